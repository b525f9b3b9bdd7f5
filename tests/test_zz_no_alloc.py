"""The allocation-free decode entry point (pvlc_attn_decode_noalloc).

Some callers can pass input and output buffers but cannot allocate device
memory (a host whose device memory is planned once by a static arena, or a
foreign-language binding without a CUDA allocator).  This variant keeps the
split-KV scratch in a fixed device array inside the library.  The test calls
it through the C ABI twice in a row and checks both calls against the
workspace-taking entry point (pvlc_attn_decode) on identical inputs, within
the decode tolerance used by the other GPU tests.  Collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

QH, KVH, HD = 16, 2, 128
ATOL = 2e-3


def _vp(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else None)


def _make(lengths, cap, seed):
    from pvlc_b200 import positions
    dev = torch.device("cuda")
    rng = np.random.default_rng(seed)
    B = len(lengths)
    host = {
        "q": rng.standard_normal((B, QH, HD)).astype(np.float16),
        "kn": rng.standard_normal((B, KVH, HD)).astype(np.float16),
        "vn": rng.standard_normal((B, KVH, HD)).astype(np.float16),
        "kc": rng.standard_normal((B, cap, KVH, HD)).astype(np.float16),
        "vc": rng.standard_normal((B, cap, KVH, HD)).astype(np.float16),
    }
    cos, sin = positions.linear_rope_tables(cap)
    t = {k: torch.from_numpy(v).to(dev) for k, v in host.items()}
    t["cos"], t["sin"] = torch.from_numpy(cos).to(dev), torch.from_numpy(sin).to(dev)
    t["ct"] = torch.tensor(lengths, dtype=torch.int32, device=dev)
    t["kp"] = torch.tensor([t["kc"][b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
    t["vp"] = torch.tensor([t["vc"][b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
    t["out"] = torch.empty((B, QH, HD), dtype=torch.float16, device=dev)
    return t


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _call_workspace(lib, t, cap, max_ct, ws, ws_bytes):
    return lib.pvlc_attn_decode(
        _vp(t["q"]), _vp(t["kn"]), _vp(t["vn"]), _vp(t["cos"]), _vp(t["sin"]), t["cos"].shape[1],
        None, _vp(t["kp"]), _vp(t["vp"]), _vp(t["ct"]), cap, max_ct, t["q"].shape[0], _vp(ws),
        ws_bytes, _vp(t["out"]), _stream())


def _call_noalloc(lib, t, cap, max_ct):
    return lib.pvlc_attn_decode_noalloc(
        _vp(t["q"]), _vp(t["kn"]), _vp(t["vn"]), _vp(t["cos"]), _vp(t["sin"]), t["cos"].shape[1],
        None, _vp(t["kp"]), _vp(t["vp"]), _vp(t["ct"]), cap, max_ct, t["q"].shape[0],
        _vp(t["out"]), _stream())


def test_noalloc_matches_workspace_entry_point_on_two_calls(cuda_lib):
    lib = cuda_lib
    # short, tile-boundary and multi-CTA sequences, so the combine path runs
    lengths = [0, 31, 32, 700, 2500, 5000, 17, 4096]
    cap = 5100
    ref = _make(lengths, cap, seed=21)
    new = _make(lengths, cap, seed=21)
    B = len(lengths)
    ws_bytes = lib.pvlc_attn_decode_workspace_bytes(B)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    assert lib.pvlc_attn_decode_workspace_init(_vp(ws), ws_bytes, _stream()) == 0

    rng = np.random.default_rng(22)
    for call in range(2):
        if call == 1:   # second call: next position, fresh query
            q2 = torch.from_numpy(rng.standard_normal((B, QH, HD)).astype(np.float16)).cuda()
            for t in (ref, new):
                t["q"].copy_(q2)
                t["ct"] += 1
        max_ct = max(lengths) + call
        assert _call_workspace(lib, ref, cap, max_ct, ws, ws_bytes) == 0
        assert _call_noalloc(lib, new, cap, max_ct) == 0
        torch.cuda.synchronize()
        a = ref["out"].float().cpu().numpy()
        b = new["out"].float().cpu().numpy()
        assert np.isfinite(b).all()
        err = np.abs(a - b).max()
        assert err <= ATOL, f"call {call}: max abs diff {err}"
        for s, L in enumerate(lengths):
            row = L + call
            assert torch.equal(ref["kc"][s, row], new["kc"][s, row])
            assert torch.equal(ref["vc"][s, row], new["vc"][s, row])


def test_noalloc_rejects_batch_beyond_its_scratch(cuda_lib):
    from pvlc_b200 import abi
    lib = cuda_lib
    B = 257   # PVLC_DECODE_NOALLOC_MAX_BATCH + 1
    t = _make([4] * B, 16, seed=5)
    before = t["kc"].clone()
    assert _call_noalloc(lib, t, 16, 4) == abi.WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert torch.equal(before, t["kc"])
