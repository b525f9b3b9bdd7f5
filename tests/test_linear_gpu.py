"""Decode-step projections on the tensor cores (pvlc_linear) against a torch fp32 reference.

out = fp16(x @ w^T) with f32 accumulation, so each output must be the fp16 rounding of the
f32 product up to the accumulation order: within half an fp16 ulp plus a small absolute
term.  The SiLU-gate form must equal fp16(silu(fp16(gate)) * fp16(up)), the numerics of an
fp16 projection followed by the SiLU-gate glue pass (crates/pvlc-cpu-ref/src/lib.rs:
1385-1390).  Shapes cover the pinned decoder's four projections at decode batch 1..256,
every split, pitched inputs and outputs, and more than 256 rows."""
import pytest
import torch

from pvlc_b200 import ops

pytestmark = pytest.mark.gpu

RTOL = 2.0 ** -10          # one fp16 ulp relative (half an ulp of rounding + accumulation order)
ATOL = 1e-4


def _data(rows, n, k, seed, ldx=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    ldx = ldx or k
    xbuf = torch.randn(rows, ldx, generator=g, device="cuda").half()
    w = (torch.randn(n, k, generator=g, device="cuda") * (1.0 / k ** 0.5)).half()
    return xbuf[:, :k], w


def _ref(x, w):
    return x.float() @ w.float().t()


def _silu_ref(gate16, up16):
    g = gate16.float()
    return (g / (1.0 + torch.exp(-g))) * up16.float()


def _check(out, ref):
    err = (out.float() - ref).abs()
    bound = ref.abs() * RTOL + ATOL
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} of {ref.numel()} outside bound, max err {err.max().item():.3g}"


@pytest.mark.parametrize("rows,n,k", [
    (1, 128, 64), (5, 256, 128), (16, 128, 1024), (32, 2560, 1024), (32, 1024, 2048),
    (32, 1024, 3072), (100, 384, 320), (200, 2560, 1024), (256, 1024, 2048),
    (256, 1024, 3072), (256, 6144, 1024),
])
def test_projection_matches_fp32(cuda_lib, rows, n, k):
    x, w = _data(rows, n, k, seed=rows * 7 + n + k)
    out = ops.linear(x, w)
    _check(out, _ref(x, w))


@pytest.mark.parametrize("split", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("rows", [3, 32, 144])
def test_every_split(cuda_lib, split, rows):
    x, w = _data(rows, 512, 1024, seed=split * 31 + rows)
    out = ops.linear(x, w, split=split)
    _check(out, _ref(x, w))


@pytest.mark.parametrize("rows,i,k,split", [
    (32, 3072, 1024, 0), (1, 64, 64, 1), (7, 192, 256, 2), (256, 3072, 1024, 0),
    (48, 512, 512, 1), (130, 1024, 1024, 8),
])
def test_silu_gate(cuda_lib, rows, i, k, split):
    g = torch.Generator(device="cuda").manual_seed(rows + i + k)
    x = torch.randn(rows, k, generator=g, device="cuda").half()
    wg = (torch.randn(i, k, generator=g, device="cuda") * (2.0 / k ** 0.5)).half()
    wu = (torch.randn(i, k, generator=g, device="cuda") * (1.0 / k ** 0.5)).half()
    w = ops.gate_up_blocks(wg, wu)
    out = ops.linear(x, w, gate=True, split=split)
    assert out.shape == (rows, i)
    g16 = _ref(x, wg).half()
    u16 = _ref(x, wu).half()
    ref = _silu_ref(g16, u16)
    err = (out.float() - ref).abs()
    # a sum on an fp16 rounding boundary may round the other way: one ulp of g or u
    bound = ref.abs() * 3e-3 + 2e-4
    assert (err > bound).sum().item() == 0, err.max().item()
    # and it agrees with the SiLU-gate glue pass over the fp16 projections except where
    # a sum sits on a rounding boundary
    unfused = ops.silu_mul(torch.cat((g16, u16), dim=1))
    assert (out != unfused).float().mean().item() < 0.01


def test_pitched_input_and_output(cuda_lib):
    rows, n, k = 40, 256, 512
    x, w = _data(rows, n, k, seed=5, ldx=k + 64)          # x rows 576 elements apart
    assert x.stride(0) == k + 64
    big = torch.full((rows, 3 * n), float("nan"), dtype=torch.float16, device="cuda")
    out = big[:, n:2 * n]                                   # a column block of a wider row
    ops.linear(x, w, out=out)
    _check(out, _ref(x, w))
    assert torch.isnan(big[:, :n]).all() and torch.isnan(big[:, 2 * n:]).all()


def test_more_than_256_rows(cuda_lib):
    x, w = _data(300, 256, 256, seed=11)
    _check(ops.linear(x, w), _ref(x, w))


def test_reproducible_and_rows_independent(cuda_lib):
    """Slice sums run in slice order: repeated calls are bitwise equal, and with the same
    split a row's output does not depend on the other rows of the call."""
    x, w = _data(64, 2560, 1024, seed=3)
    a = ops.linear(x, w, split=8)
    b = ops.linear(x, w, split=8)
    assert torch.equal(a, b)
    c = ops.linear(x[:17].contiguous(), w, split=8)
    assert torch.equal(a[:17], c)


def test_graph_capture_and_fault_word_clear(cuda_lib):
    """Captured in a CUDA graph behind other work on the stream (programmatic dependent
    launch: the weights are read before the wait, the activations after it)."""
    x, w = _data(32, 1024, 3072, seed=9)
    w2 = (torch.randn(2560, 1024, device="cuda") * 0.03).half()
    y = torch.empty(32, 1024, dtype=torch.float16, device="cuda")
    z = torch.empty(32, 2560, dtype=torch.float16, device="cuda")
    xs = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        ops.fault_flags()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            xs.copy_(x)
            xs.mul_(0.5)                        # a kernel ahead that writes the activations
            ops.linear(xs, w, out=y)
            ops.linear(y, w2, out=z)   # reads the previous projection's output
        for _ in range(3):
            y.zero_()
            z.zero_()
            graph.replay()
        s.synchronize()
        assert ops.fault_flags() == 0
    ref_y = _ref(x * 0.5, w)
    _check(y, ref_y)
    _check(z, _ref(y, w2))
