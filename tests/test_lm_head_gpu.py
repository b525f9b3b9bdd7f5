"""Greedy top-1 over the LM head (pvlc_lm_head_top1, tcgen05 GEMM with an arg-max
epilogue) against the reference's rule: the largest f32 logit, equal logits to the
smaller token id (compare_top_k_entries, crates/pvlc-cpu-ref/src/lib.rs:2051-2056;
chunked_lm_head_top_k_f32 :1511-1568).

Exactness: with small-integer fp16 inputs every logit is an integer that f32 holds
exactly whatever the summation order, so the oracle's logits (linear_f32 order) and
the kernel's agree bit for bit and ties are common: the ids must be identical.  On
N(0,1)-scale inputs the ids must equal the f32 arg-max wherever the top-two margin
exceeds the f32 accumulation error, and the reported logit must be within 1e-3
relative of the f32 maximum.
"""
import ctypes

import numpy as np
import pytest
import torch

import pvlc_oracle as O

pytestmark = pytest.mark.gpu


def _ref_top1(logits):
    """compare_top_k_entries with top_k = 1 on f32 rows: max value, smallest index."""
    m = logits.max(axis=1, keepdims=True)
    return np.argmax(logits == m, axis=1)


@pytest.mark.parametrize("rows,vocab,K", [(1, 1000, 128), (3, 1000, 128), (5, 1000, 192),
                                          (129, 5000, 256), (256, 2304, 64)])
def test_integer_logits_match_the_oracle_with_ties(cuda_lib, rows, vocab, K):
    from pvlc_b200 import ops
    rng = np.random.default_rng(rows + vocab)
    h = rng.integers(-2, 3, (rows, K)).astype(np.float16)
    w = rng.integers(-2, 3, (vocab, K)).astype(np.float16)
    w[vocab - 1] = w[3]          # an exact tie across N tiles: id 3 must win over vocab - 1
    ref_logits = O.linear(h.astype(np.float32), w.astype(np.float32))
    want = _ref_top1(ref_logits)
    lg = torch.empty(rows, dtype=torch.float32, device="cuda")
    got = ops.lm_head_top1(torch.from_numpy(h).cuda(), torch.from_numpy(w).cuda(), logits=lg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    np.testing.assert_array_equal(lg.cpu().numpy(), ref_logits.max(axis=1))


@pytest.mark.parametrize("rows", [1, 32, 200, 256, 300])
def test_decoder_shape_against_f32_argmax(cuda_lib, rows):
    """The engine's shape: hidden [rows, 1024], vocab 103,424."""
    from pvlc_b200 import ops
    g = torch.Generator(device="cuda")
    g.manual_seed(rows)
    h = torch.randn((rows, 1024), generator=g, device="cuda").half()
    w = (torch.randn((103_424, 1024), generator=g, device="cuda") * 0.02).half()
    ref = torch.mm(h, w.t(), out_dtype=torch.float32)
    lg = torch.empty(rows, dtype=torch.float32, device="cuda")
    got = ops.lm_head_top1(h, w, logits=lg).long()
    top2 = torch.topk(ref, 2, dim=1).values
    margin = top2[:, 0] - top2[:, 1]
    tol = 1e-3 * top2[:, 0].abs()
    clear = margin > tol
    assert torch.equal(got[clear], ref.argmax(dim=1)[clear])
    picked = ref.gather(1, got[:, None])[:, 0]
    assert torch.all(picked >= top2[:, 0] - tol)
    assert torch.allclose(lg, top2[:, 0], rtol=1e-3, atol=0)
    # a second call on the same workspace gives the same ids
    ws = torch.empty(int(ops.abi.lib().pvlc_lm_head_top1_workspace_bytes(min(rows, 256))),
                     dtype=torch.uint8, device="cuda")
    again = ops.lm_head_top1(h, w, workspace=ws)
    again2 = ops.lm_head_top1(h, w, workspace=ws)
    assert torch.equal(again.long(), got) and torch.equal(again2, again)


def test_host_refusals_have_no_device_effect(cuda_lib):
    from pvlc_b200 import abi
    lib = abi.lib()
    h = torch.zeros((4, 128), dtype=torch.float16, device="cuda")
    w = torch.zeros((300, 128), dtype=torch.float16, device="cuda")
    ws = torch.empty(int(lib.pvlc_lm_head_top1_workspace_bytes(4)), dtype=torch.uint8,
                     device="cuda")
    tok = torch.full((4,), -7, dtype=torch.int32, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    f = lib.pvlc_lm_head_top1
    assert f(P(h), 0, P(w), 300, 128, P(ws), ws.numel(), P(tok), None, s) == abi.ZERO_DIMENSION
    assert f(P(h), 257, P(w), 300, 128, P(ws), ws.numel(), P(tok), None, s) == \
        abi.INVALID_DECODER_GEOMETRY
    assert f(P(h), 4, P(w), 300, 100, P(ws), ws.numel(), P(tok), None, s) == \
        abi.INVALID_DECODER_GEOMETRY
    assert f(P(h), 4, P(w), 300, 128, P(ws), ws.numel() - 1, P(tok), None, s) == \
        abi.WORKSPACE_TOO_SMALL
    assert f(P(h[:, 1:]), 4, P(w), 300, 128, P(ws), ws.numel(), P(tok), None, s) == \
        abi.MISALIGNED_POINTER
    assert f(P(h), 4, P(w), 300, 128, P(None), ws.numel(), P(tok), None, s) == abi.NULL_POINTER
    assert lib.pvlc_lm_head_top1_workspace_bytes(0) == 0
    assert lib.pvlc_lm_head_top1_workspace_bytes(257) == 0
    torch.cuda.synchronize()
    assert (tok == -7).all()
    # a clean call leaves the fault word clear
    assert f(P(h), 4, P(w), 300, 128, P(ws), ws.numel(), P(tok), None, s) == abi.OK
    flags = ctypes.c_uint32(99)
    assert lib.pvlc_lm_head_top1_errors(P(ws), 4, ctypes.byref(flags), s) == abi.OK
    assert flags.value == 0
