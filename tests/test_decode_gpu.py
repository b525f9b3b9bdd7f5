"""Decode path parity: CUDA split-KV decode (C ABI) vs the CPU oracle.

Oracle: decode_gqa_f32 with the append and single-row M-RoPE of the decode
step (crates/pvlc-cpu-ref/src/lib.rs:858-927,1420-1450,1648-1680) on the same
fp16-representable inputs.  Tolerance (north-star): max-abs <= 2e-3 on the fp16
outputs; cache rows written by the kernel match the oracle's rotated key within
fp16 rounding.
"""
import numpy as np
import pytest
import torch

import pvlc_oracle as O

pytestmark = pytest.mark.gpu

QH, KVH, HD = 16, 2, 128
ATOL = 2e-3


def _setup(lengths, capacity, seed, poison_tail=True, rope_rows=None):
    """lengths = cache rows BEFORE the append, per sequence."""
    from pvlc_b200 import ops, positions
    rng = np.random.default_rng(seed)
    B = len(lengths)
    q = rng.standard_normal((B, QH, HD)).astype(np.float16)
    kn = rng.standard_normal((B, KVH, HD)).astype(np.float16)
    vn = rng.standard_normal((B, KVH, HD)).astype(np.float16)
    kc = rng.standard_normal((B, capacity, KVH, HD)).astype(np.float16)
    vc = rng.standard_normal((B, capacity, KVH, HD)).astype(np.float16)
    if poison_tail:
        for b, L in enumerate(lengths):
            kc[b, L + 1:] = np.nan   # nothing past the appended row may be read
            vc[b, L + 1:] = np.nan
            kc[b, L] = np.nan        # the append slot itself is overwritten before use
            vc[b, L] = np.nan
    rows = rope_rows or capacity
    cos, sin = positions.linear_rope_tables(rows)
    dev = torch.device("cuda")
    t = dict(
        q=torch.from_numpy(q).to(dev), kn=torch.from_numpy(kn).to(dev),
        vn=torch.from_numpy(vn).to(dev), kc=torch.from_numpy(kc).to(dev),
        vc=torch.from_numpy(vc).to(dev), cos=torch.from_numpy(cos).to(dev),
        sin=torch.from_numpy(sin).to(dev),
        ct=torch.tensor(lengths, dtype=torch.int32, device=dev))
    t["kp"] = torch.tensor([t["kc"][b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
    t["vp"] = torch.tensor([t["vc"][b].data_ptr() for b in range(B)], dtype=torch.int64, device=dev)
    t["ws"] = ops.DecodeWorkspace(B)
    host = dict(q=q, kn=kn, vn=vn, kc=kc, vc=vc, cos=cos, sin=sin)
    return t, host


def _oracle(host, b, L, rope_row=None):
    kc = host["kc"][b].astype(np.float32).copy()
    vc = host["vc"][b].astype(np.float32).copy()
    out = O.decode_step(host["q"][b].astype(np.float32), host["kn"][b].astype(np.float32),
                        host["vn"][b].astype(np.float32), host["cos"], host["sin"],
                        L if rope_row is None else rope_row, kc, vc, L)
    return out.reshape(QH, HD), kc[L], vc[L]


def _run(t, capacity, max_ct):
    from pvlc_b200 import ops
    out = ops.decode(t["q"], t["kn"], t["vn"], t["cos"], t["sin"], t["kp"], t["vp"], t["ct"],
                     capacity, max_ct, t["ws"])
    torch.cuda.synchronize()
    return out


def test_decode_config1_single_sequence(cuda_lib):
    """B=1, Q16/KV2/D128, 1024 KV rows after the append."""
    L = 1023
    t, host = _setup([L], 1024, seed=0)
    out = _run(t, 1024, L).cpu().numpy().astype(np.float32)
    ref, kref, vref = _oracle(host, 0, L)
    assert np.isfinite(out).all()
    err = np.abs(out[0] - ref).max()
    assert err <= ATOL, f"max abs err {err}"
    krow = t["kc"][0, L].float().cpu().numpy()
    vrow = t["vc"][0, L].float().cpu().numpy()
    np.testing.assert_allclose(krow, kref, atol=2e-3, rtol=1e-3)
    np.testing.assert_array_equal(vrow, vref)
    assert t["ws"].errors() == 0


@pytest.mark.parametrize("lengths", [
    [0, 1, 15, 16, 31, 32, 33, 63],          # tile and half-tile boundaries
    [700, 3, 1500, 64, 65, 4000],            # ragged batch, multi-CTA sequences
    # forty one-tile sequences, ~4 per CTA: the copy warp runs several
    # sequences ahead of the sequence warp's appends
    [(7 * i) % 31 for i in range(40)],
    # one-tile sequences between long ones: append-first and q-first pieces
    [5, 900, 2, 0, 30, 1300, 17, 3, 640, 1],
])
def test_decode_ragged_batch_with_poisoned_tails(cuda_lib, lengths):
    cap = max(lengths) + 7
    t, host = _setup(lengths, cap, seed=len(lengths))
    out = _run(t, cap, max(lengths)).cpu().numpy().astype(np.float32)
    assert np.isfinite(out).all()
    for b, L in enumerate(lengths):
        ref, kref, _ = _oracle(host, b, L)
        err = np.abs(out[b] - ref).max()
        assert err <= ATOL, f"seq {b} (L={L}) max abs err {err}"
        np.testing.assert_allclose(t["kc"][b, L].float().cpu().numpy(), kref, atol=2e-3, rtol=1e-3)
    assert t["ws"].errors() == 0


def test_decode_two_steps_reuse_workspace(cuda_lib):
    """Consecutive launches on one workspace: combine tickets reset themselves."""
    lengths = [900, 2500, 17]
    cap = 2600
    t, host = _setup(lengths, cap, seed=7, poison_tail=False)
    first = _run(t, cap, max(lengths)).cpu().numpy().astype(np.float32)
    # step 2: advance the rows and append again with fresh inputs
    rng = np.random.default_rng(8)
    q2 = rng.standard_normal((3, QH, HD)).astype(np.float16)
    t["q"].copy_(torch.from_numpy(q2))
    t["ct"] += 1
    second = _run(t, cap, max(lengths) + 1).cpu().numpy().astype(np.float32)
    for b, L in enumerate(lengths):
        ref1, k1, v1 = _oracle(host, b, L)
        assert np.abs(first[b] - ref1).max() <= ATOL
        kc = host["kc"][b].astype(np.float32).copy()
        vc = host["vc"][b].astype(np.float32).copy()
        kc[L] = t["kc"][b, L].float().cpu().numpy()   # the fp16 row the GPU appended
        vc[L] = v1
        ref2 = O.decode_step(q2[b].astype(np.float32), host["kn"][b].astype(np.float32),
                             host["vn"][b].astype(np.float32), host["cos"], host["sin"], L + 1, kc,
                             vc, L + 1).reshape(QH, HD)
        assert np.abs(second[b] - ref2).max() <= ATOL
    assert t["ws"].errors() == 0


def test_decode_strided_qkv_matches_packed(cuda_lib):
    """q / k_new / v_new as column blocks of one [B, 2560] projection (row stride 2560,
    pvlc_attn_decode_strided) give exactly the packed-input results, outputs and the
    appended cache rows alike."""
    from pvlc_b200 import ops
    lengths = [5, 300, 64, 1777]
    cap = max(lengths) + 3
    t, host = _setup(lengths, cap, seed=13, poison_tail=False)
    B = len(lengths)
    qkv = torch.empty((B, 2560), dtype=torch.float16, device="cuda")
    qkv[:, :2048] = t["q"].view(B, -1)
    qkv[:, 2048:2304] = t["kn"].view(B, -1)
    qkv[:, 2304:] = t["vn"].view(B, -1)
    q, k, v = qkv[:, :2048].view(B, QH, HD), qkv[:, 2048:2304].view(B, KVH, HD), \
        qkv[:, 2304:].view(B, KVH, HD)
    kc0, vc0 = t["kc"].clone(), t["vc"].clone()
    ref = _run(t, cap, max(lengths))
    kc_ref, vc_ref = t["kc"].clone(), t["vc"].clone()
    t["kc"].copy_(kc0)
    t["vc"].copy_(vc0)
    got = ops.decode(q, k, v, t["cos"], t["sin"], t["kp"], t["vp"], t["ct"], cap, max(lengths),
                     t["ws"])
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    assert torch.equal(t["kc"], kc_ref) and torch.equal(t["vc"], vc_ref)
    assert t["ws"].errors() == 0
    with pytest.raises(ValueError):      # k_new and v_new strides must agree
        ops.decode(q, k, t["vn"], t["cos"], t["sin"], t["kp"], t["vp"], t["ct"], cap,
                   max(lengths), t["ws"])


def test_decode_large_batch_stream_k(cuda_lib):
    """64 sequences with lengths in [512, 8192] (config-4 shape), every sequence checked."""
    rng = np.random.default_rng(1)
    lengths = rng.integers(512, 8193, size=64).tolist()
    cap = 8192 + 8
    t, host = _setup(lengths, cap, seed=11, poison_tail=True)
    out = _run(t, cap, max(lengths)).cpu().numpy().astype(np.float32)
    assert np.isfinite(out).all()
    for b in range(0, 64, 3):
        ref, _, _ = _oracle(host, b, lengths[b])
        err = np.abs(out[b] - ref).max()
        assert err <= ATOL, f"seq {b} (L={lengths[b]}) err {err}"
    assert t["ws"].errors() == 0


@pytest.mark.parametrize("n,lo,hi,seed", [(600, 0, 40, 21), (300, 0, 300, 22)])
def test_decode_many_short_sequences(cuda_lib, n, lo, hi, seed):
    """Hundreds of short sequences: the work-weighted split then gives many CTAs
    an empty range (a sequence end's allowance only) and others several sequence
    ends each; two steps in a row on one workspace."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=n).tolist()
    cap = hi + 4
    t, host = _setup(lengths, cap, seed=seed, poison_tail=False)
    out = _run(t, cap, max(lengths)).cpu().numpy().astype(np.float32)
    assert np.isfinite(out).all()
    for b in range(0, n, 7):
        ref, _, _ = _oracle(host, b, lengths[b])
        err = np.abs(out[b] - ref).max()
        assert err <= ATOL, f"seq {b} (L={lengths[b]}) err {err}"
    t["ct"] += 1
    out2 = _run(t, cap, max(lengths) + 1).cpu().numpy().astype(np.float32)
    assert np.isfinite(out2).all()
    assert t["ws"].errors() == 0


def test_decode_rejects_out_of_range_rows_without_faulting(cuda_lib):
    """A device-side row past max_cache_tokens is skipped, zero-filled and flagged."""
    lengths = [10, 20]
    t, host = _setup(lengths, 64, seed=3, poison_tail=False)
    t["ct"][1] = 40            # larger than the host bound passed below
    out = _run(t, 64, 20).cpu().numpy()
    assert (out[1] == 0).all()
    ref, _, _ = _oracle(host, 0, 10)
    assert np.abs(out[0].astype(np.float32) - ref).max() <= ATOL
    assert t["ws"].errors() & 1
    assert t["ws"].errors() == 0   # reading clears the flags


def test_decode_host_validation_has_no_device_effect(cuda_lib):
    from pvlc_b200 import abi, ops
    t, _ = _setup([5], 8, seed=4, poison_tail=False)
    before = t["kc"].clone()
    with pytest.raises(abi.PvlcError) as e:
        ops.decode(t["q"], t["kn"], t["vn"], t["cos"], t["sin"], t["kp"], t["vp"], t["ct"],
                   8, 8, t["ws"])           # max_cache_tokens must be < capacity
    assert e.value.status == abi.CAPACITY_EXHAUSTED
    torch.cuda.synchronize()
    assert torch.equal(before, t["kc"])
