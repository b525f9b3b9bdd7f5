"""Vision varlen attention parity: CUDA kernel (C ABI) vs the CPU oracle.

Oracle: vision_rope_2d table form (crates/pvlc-wgsl/src/lib.rs:1691-1730) then
materialized_segmented_attention_f32 (crates/pvlc-cpu-ref/src/lib.rs:2752-2802).
Inputs are fp16-representable; tolerance max-abs <= 2e-3 on fp16 outputs
(north-star), which is looser than the reference's f32-vs-f32 native policy
(3e-4, crates/pvlc-testkit/src/m3_vision_attention.rs:13-21) by the fp16 output
rounding and fp16 P/V operands.
"""
import numpy as np
import pytest
import torch

import pvlc_oracle as O
from test_oracle_kat import m3_case

pytestmark = pytest.mark.gpu
H, D = 16, 72
ATOL = 2e-3


def _gpu(q, k, v, cu, cos=None, sin=None):
    from pvlc_b200 import ops
    dev = torch.device("cuda")
    T = q.size // (H * D)
    tq = torch.from_numpy(q.astype(np.float16).reshape(T, H, D)).to(dev)
    tk = torch.from_numpy(k.astype(np.float16).reshape(T, H, D)).to(dev)
    tv = torch.from_numpy(v.astype(np.float16).reshape(T, H, D)).to(dev)
    tc = torch.from_numpy(cos).to(dev) if cos is not None else None
    ts = torch.from_numpy(sin).to(dev) if sin is not None else None
    out = ops.vision_varlen_attention(tq, tk, tv, cu, tc, ts)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


M3_CASES = [(n, [0, n], 101 + i, None) for i, n in enumerate([8, 16, 31, 64, 127, 256])] + [
    (31, [0, 3, 11, 31], 201, None), (17, [0, 3, 9, 17], 301, None),
    (17, [0, 3, 9, 17], 301, 0), (17, [0, 3, 9, 17], 301, 1), (17, [0, 3, 9, 17], 301, 2)]


@pytest.mark.parametrize("tokens,cu,seed,poison", M3_CASES)
def test_m3_corpus(cuda_lib, tokens, cu, seed, poison):
    """The reference's 11-case M3 vision attention corpus (no RoPE)."""
    q, k, v = m3_case(tokens, cu, seed, poison)
    # the kernel consumes fp16: give the oracle the same (fp16-rounded) operands
    q, k, v = (x.astype(np.float16).astype(np.float32) for x in (q, k, v))
    ref = O.segmented_attention(q, k, v, tokens, H, D, cu).reshape(tokens, H, D)
    got = _gpu(q, k, v, cu)
    err = np.abs(got - ref).max()
    # poisoned segments hold values up to ~130 in V: scale the bound by the value range
    scale = max(1.0, float(np.abs(v).max()) / 2.0)
    assert err <= ATOL * scale, f"max abs err {err}"


def test_poisoned_segment_does_not_leak(cuda_lib):
    cu = [0, 3, 9, 17]
    q, k, v = m3_case(17, cu, 301)
    base = _gpu(q, k, v, cu)
    for seg in range(3):
        qp, kp, vp = m3_case(17, cu, 301, seg)
        got = _gpu(qp, kp, vp, cu)
        for s2 in range(3):
            rows = slice(cu[s2], cu[s2 + 1])
            if s2 != seg:
                np.testing.assert_array_equal(got[rows], base[rows])


@pytest.mark.parametrize("grids", [
    [(1, 4, 4)],
    [(1, 8, 8), (1, 6, 10), (1, 2, 2)],
    [(1, 12, 16), (1, 9, 7), (1, 16, 12)],
])
def test_packed_images_with_rope(cuda_lib, grids):
    from pvlc_b200 import positions
    rng = np.random.default_rng(len(grids))
    lens = [t * h * w for t, h, w in grids]
    cu = np.concatenate([[0], np.cumsum(lens)]).tolist()
    T = cu[-1]
    q = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    cos, sin = positions.vision_rope_tables(grids)
    ocos, osin = O.vision_rope_tables(grids)
    np.testing.assert_allclose(cos, ocos, atol=1e-7, rtol=0)
    qr, kr = O.vision_rope_apply_tables(q, k, T, H, D, ocos, osin)
    ref = O.segmented_attention(qr, kr, v, T, H, D, cu).reshape(T, H, D)
    got = _gpu(q, k, v, cu, cos, sin)
    err = np.abs(got - ref).max()
    assert err <= ATOL, f"max abs err {err}"


def _rope_case(grids, seed):
    from pvlc_b200 import positions
    lens = [t * h * w for t, h, w in grids]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32).tolist()
    T = cu[-1]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((T, H, D)).astype(np.float16).astype(np.float32)
    cos, sin = positions.vision_rope_tables(grids)
    return cu, T, q, k, v, cos, sin


def _check_every_segment(got, q, k, v, cu, cos, sin):
    T = cu[-1]
    qr, kr = O.vision_rope_apply_tables(q, k, T, H, D, cos, sin)
    ref = O.segmented_attention(qr, kr, v, T, H, D, cu).reshape(T, H, D)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        err = float(np.abs(got[a:b] - ref[a:b]).max())
        assert err <= ATOL, f"segment {s} ({b - a} tokens) err {err}"


def test_config2_shape_every_segment(cuda_lib):
    """BASELINE config 2 geometry (8000 tokens, segments 1024/2304/576/4096, 2-D RoPE):
    every row of every segment against the oracle."""
    grids = [(1, 32, 32), (1, 48, 48), (1, 24, 24), (1, 64, 64)]
    cu, T, q, k, v, cos, sin = _rope_case(grids, 2)
    assert cu == [0, 1024, 3328, 3904, 8000]
    got = _gpu(q, k, v, cu, cos, sin)
    assert np.isfinite(got).all()
    _check_every_segment(got, q, k, v, cu, cos, sin)


def test_e2e_page_segment(cuda_lib):
    """The end-to-end engine's page: a 1024x1024 image resized to 980x980 is one
    70x70 = 4900-patch segment (39 K tiles), packed after a short one; every row."""
    grids = [(1, 70, 70), (1, 5, 7)]
    cu, T, q, k, v, cos, sin = _rope_case(grids, 44)
    got = _gpu(q, k, v, cu, cos, sin)
    _check_every_segment(got, q, k, v, cu, cos, sin)


def test_lazy_rescale_branch(cuda_lib):
    """Scores that rise along the keys and jump by more than the kernel's lazy rescale
    threshold (8 log2 units) twice, in the middle and late in a segment, so the
    running max moves and O is rescaled mid-segment; heads alternate the sign of the
    query's planted component, so half of them meet their max in the first K tile and
    only see P far below 1 afterwards.  The planted component is dim 35 of head_dim 72:
    a column-position pair at the 2-D RoPE's lowest frequency (~1.7e-4 rad a patch).
    The 3000-patch image is one column wide, so dim 35 is not rotated there at all; in
    the 40x50 image it turns by at most 49 patches' worth."""
    grids = [(1, 3000, 1), (1, 40, 50)]
    cu, T, q, k, v, cos, sin = _rope_case(grids, 9)
    q *= 0.25
    k *= 0.25
    sign = np.where(np.arange(H) % 2 == 0, 1.0, -1.0).astype(np.float32)
    q[:, :, 35] = (6.0 * sign)[None, :]
    for a, b in ((cu[0], cu[1]), (cu[1], cu[2])):
        n = b - a
        k[a:b, :, 35] = np.linspace(-2.0, 6.0, n, dtype=np.float32)[:, None]
        k[a + int(0.45 * n):a + int(0.45 * n) + 32, :, 35] = 10.0
        k[a + int(0.85 * n):a + int(0.85 * n) + 64, :, 35] = 20.0
    q, k = (x.astype(np.float16).astype(np.float32) for x in (q, k))
    # a planted key value x gives a score of about 6 x / sqrt(72) nats = 1.02 x log2 units
    per_unit = 6.0 / np.sqrt(72.0) * np.log2(np.e)
    assert (10.0 - (-2.0)) * per_unit > 8.0 and (20.0 - 10.0) * per_unit > 8.0
    got = _gpu(q, k, v, cu, cos, sin)
    assert np.isfinite(got).all()
    _check_every_segment(got, q, k, v, cu, cos, sin)


def test_vision_validation_errors(cuda_lib):
    from pvlc_b200 import abi
    T = 8
    z = torch.zeros((T, H, D), dtype=torch.float16, device="cuda")
    from pvlc_b200 import ops
    for cu, code in (([0, 4, 4, 8], abi.INVALID_SEQUENCE_BOUNDARIES),
                     ([1, 8], abi.INVALID_SEQUENCE_BOUNDARIES),
                     ([0, 7], abi.INVALID_SEQUENCE_BOUNDARIES)):
        with pytest.raises(abi.PvlcError) as e:
            ops.vision_varlen_attention(z, z, z, cu)
        assert e.value.status == code


def test_workspace_entry_points_agree(cuda_lib):
    """pvlc_attn_vision_varlen (stream-ordered scratch) and pvlc_attn_vision_varlen_ws
    (caller scratch) run the same kernels: bitwise equal outputs; the _ws checks."""
    import ctypes
    from pvlc_b200 import abi, ops, positions
    grids = [(1, 8, 8), (1, 6, 10)]
    cu = np.array([0, 64, 124], np.uint32)
    T = 124
    g = torch.Generator(device="cuda")
    g.manual_seed(7)
    q, k, v = (torch.randn((T, H, D), generator=g, device="cuda").half() for _ in range(3))
    c, s = (torch.from_numpy(x).cuda() for x in positions.vision_rope_tables(grids))
    a = ops.vision_varlen_attention(q, k, v, cu, c, s)
    b = torch.empty_like(a)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = abi.lib().pvlc_attn_vision_varlen(P(q), P(k), P(v), cu.ctypes.data_as(ctypes.c_void_p),
                                           2, T, H, D, P(c), P(s), P(b), stream)
    assert st == abi.OK
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    need = ops.vision_workspace_bytes(T, H)
    assert need == 2 * T * H * D * 2
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    f = abi.lib().pvlc_attn_vision_varlen_ws
    args = (P(q), P(k), P(v), cu.ctypes.data_as(ctypes.c_void_p), 2, T, H, D, P(c), P(s))
    assert f(*args, P(ws), need - 1, P(b), stream) == abi.WORKSPACE_TOO_SMALL
    assert f(*args, P(None), need, P(b), stream) == abi.NULL_POINTER
    assert f(*args, P(ws[1:]), need - 1, P(b), stream) in (abi.MISALIGNED_POINTER,
                                                         abi.WORKSPACE_TOO_SMALL)
    # without tables no scratch is needed: NULL workspace is fine
    ref = ops.vision_varlen_attention(q, k, v, cu)
    nul = P(None)
    assert f(P(q), P(k), P(v), cu.ctypes.data_as(ctypes.c_void_p), 2, T, H, D, nul, nul, nul, 0,
             P(b), stream) == abi.OK
    torch.cuda.synchronize()
    assert torch.equal(ref, b)


@pytest.mark.parametrize("rope", [True, False])
def test_many_ragged_segments_persistent_schedule(cuda_lib, rope):
    """More work items than SMs and ragged segments (single-Q-tile items, partial K
    tiles), with and without rope tables, against the oracle; a second call on the
    same scratch gives the same bits."""
    import pvlc_oracle as O
    from pvlc_b200 import ops, positions
    rng = np.random.default_rng(21)
    lens = rng.integers(1, 700, size=48)
    lens[:4] = [1, 128, 129, 257]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    T = int(cu[-1])
    q = rng.standard_normal((T, H, D)).astype(np.float16)
    k = rng.standard_normal((T, H, D)).astype(np.float16)
    v = rng.standard_normal((T, H, D)).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(x).cuda() for x in (q, k, v))
    if rope:
        grids = [(1, 1, int(n)) for n in lens]
        c, s_ = positions.vision_rope_tables(grids)
        tc, ts = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
        ws = torch.empty(ops.vision_workspace_bytes(T, H), dtype=torch.uint8, device="cuda")
        out = ops.vision_varlen_attention(dq, dk, dv, cu, tc, ts, workspace=ws)
        out2 = ops.vision_varlen_attention(dq, dk, dv, cu, tc, ts, workspace=ws)
        qr, kr = O.vision_rope_apply_tables(q.astype(np.float32), k.astype(np.float32), T, H, D,
                                            c, s_)
    else:
        out = ops.vision_varlen_attention(dq, dk, dv, cu)
        out2 = ops.vision_varlen_attention(dq, dk, dv, cu)
        qr, kr = q.astype(np.float32), k.astype(np.float32)
    torch.cuda.synchronize()
    ref = O.segmented_attention(qr, kr, v.astype(np.float32), T, H, D, cu)
    err = float(np.abs(out.float().cpu().numpy().reshape(-1) - ref.reshape(-1)).max())
    assert err <= 2e-3, err
    assert torch.equal(out, out2)


@pytest.mark.parametrize("rope", [True, False])
def test_strided_qkv_matches_packed(cuda_lib, rope):
    """q, k, v as the three column blocks of one [T, 3 x 1152] projection output
    (pvlc_attn_vision_varlen_strided_ws) give the packed call's outputs bit for bit;
    a stride below heads x 72 or not a multiple of 8 is refused before any launch."""
    import ctypes
    from pvlc_b200 import abi, ops, positions
    grids = [(1, 12, 16), (1, 9, 7), (1, 20, 20)]
    lens = [t * h * w for t, h, w in grids]
    cu = np.concatenate([[0], np.cumsum(lens)]).tolist()
    T = cu[-1]
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    qkv = torch.randn((T, 3 * H * D), generator=g, device="cuda").half()
    q, k, v = (qkv[:, j * H * D:(j + 1) * H * D].view(T, H, D) for j in range(3))
    tabs = (None, None)
    if rope:
        tabs = tuple(torch.from_numpy(x).cuda() for x in positions.vision_rope_tables(grids))
    got = ops.vision_varlen_attention(q, k, v, cu, *tabs)
    ref = ops.vision_varlen_attention(q.contiguous(), k.contiguous(), v.contiguous(), cu, *tabs)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)
    cuh = np.asarray(cu, np.uint32)
    ws = torch.empty(ops.vision_workspace_bytes(T, H), dtype=torch.uint8, device="cuda")
    out = torch.empty((T, H, D), dtype=torch.float16, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    f = abi.lib().pvlc_attn_vision_varlen_strided_ws
    for bad in (H * D - 8, H * D + 4):
        st = f(P(q), P(k), P(v), bad, cuh.ctypes.data_as(ctypes.c_void_p), 3, T, H, D,
               P(tabs[0]), P(tabs[1]), P(ws), ws.numel(), P(out), stream)
        assert st == abi.LENGTH_MISMATCH
