"""Engine glue kernels (residual add + LayerNorm / RMSNorm, GELU, SiLU gate) vs torch fp32.

Floating-point elementwise kernels: the reference is the plain fp32 computation of
crates/pvlc-cpu-ref/src/lib.rs:280-367 (torch on the same device), rounded to fp16 once.
Tolerance: 2e-3 absolute + 2e-3 relative on the fp16 outputs; the updated f32 residual
stream is compared exactly (the same single f32 addition).
"""
import pytest
import torch

from pvlc_b200 import ops

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("rows,width,layer,with_delta", [
    (3, 1152, True, False), (257, 1152, True, True), (5, 1024, False, True),
    (1000, 1024, False, False), (9, 8, True, True), (17, 2048, False, True),
    (4, 2056, True, True), (2, 4608, True, True),
    # from 4096 rows, widths 1152 / 1024 take the warp-per-row kernel (8 rows per CTA;
    # 8191 leaves a partial last CTA)
    (5000, 1152, True, True), (8191, 1152, True, False), (4096, 1024, False, True),
    (4100, 1024, False, False)])
def test_add_norm(cuda_lib, rows, width, layer, with_delta):
    g = torch.Generator(device="cuda")
    g.manual_seed(rows + width)
    h = torch.randn((rows, width), generator=g, device="cuda") * 3 + 0.5
    d = (torch.randn((rows, width), generator=g, device="cuda")).half() if with_delta else None
    w = 1 + 0.1 * torch.randn(width, generator=g, device="cuda")
    b = 0.1 * torch.randn(width, generator=g, device="cuda") if layer else None
    eps = 1e-6 if layer else 1e-5
    ref_h = h + d.float() if with_delta else h.clone()
    if layer:
        mean = ref_h.mean(-1, keepdim=True)
        var = ((ref_h - mean) ** 2).mean(-1, keepdim=True)
        ref = (ref_h - mean) / torch.sqrt(var + eps) * w + b
    else:
        ref = ref_h / torch.sqrt((ref_h * ref_h).mean(-1, keepdim=True) + eps) * w
    out = ops.add_norm(h, w, eps, bias=b, delta=d)
    torch.cuda.synchronize()
    assert torch.equal(h, ref_h)
    torch.testing.assert_close(out.float(), ref.half().float(), **TOL)


@pytest.mark.parametrize("erf", [False, True])
@pytest.mark.parametrize("n", [4304 * 3, 4304 * 3 + 6, 2])
def test_gelu(cuda_lib, erf, n):
    # n % 8 != 0 runs the pair tail after the 16-byte body
    x = (torch.linspace(-8, 8, n, device="cuda")).half()
    ref = torch.nn.functional.gelu(x.float(), approximate="none" if erf else "tanh").half()
    got = ops.gelu_(x.clone(), erf=erf)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), ref.float(), **TOL)


@pytest.mark.parametrize("width", [3072, 6])   # 8-wide and pair accesses
def test_silu_mul(cuda_lib, width):
    g = torch.Generator(device="cuda")
    g.manual_seed(4)
    gu = (torch.randn((77, 2 * width), generator=g, device="cuda") * 4).half()
    ref = (torch.nn.functional.silu(gu[:, :width].float()) * gu[:, width:].float()).half()
    got = ops.silu_mul(gu)
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float(), ref.float(), **TOL)


def test_glue_rejects_bad_shapes_before_launch(cuda_lib):
    from pvlc_b200 import abi
    import ctypes
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)
    h = torch.zeros((2, 12), device="cuda")
    w = torch.ones(12, device="cuda")
    o = torch.empty((2, 12), dtype=torch.float16, device="cuda")
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # width 12 is not a multiple of 8
    assert abi.lib().pvlc_add_norm(P(h), P(None), 2, 12, P(w), P(None), 1e-5, P(o), s) == \
        abi.LENGTH_MISMATCH
    assert abi.lib().pvlc_add_norm(P(h), P(None), 0, 8, P(w), P(None), 1e-5, P(o), s) == \
        abi.ZERO_DIMENSION
    assert abi.lib().pvlc_gelu(P(o), 3, 0, s) == abi.LENGTH_MISMATCH
