"""The C ABI library loads, exports every symbol the header declares, and its
host-side plans validate geometry like the reference's runtime-core contract
(no GPU needed: plans never touch a device)."""
import ctypes
import re

import numpy as np
import pytest

from pvlc_b200 import abi


def _header_functions():
    text = open(abi.HEADER_PATH).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pvlc_(?:attn|plan|image|add_norm|gelu|silu_mul|bf16_to_f16|lm_head|blake3|linear)\w*)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = abi.lib()
    declared = _header_functions()
    assert len(declared) >= 12
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(abi.EXPORTED) == declared


def test_status_strings_mirror_invocation_error_codes():
    # crates/pvlc-runtime-core/src/lib.rs:5335-5351 declaration order
    assert abi.status_string(abi.ZERO_DIMENSION) == "ZeroDimension"
    assert abi.status_string(abi.LENGTH_MISMATCH) == "LengthMismatch"
    assert abi.status_string(abi.UNSUPPORTED_HEAD_DIMENSION) == "UnsupportedHeadDimension"
    assert abi.status_string(abi.INVALID_DECODER_GEOMETRY) == "InvalidDecoderGeometry"
    assert abi.status_string(abi.INVALID_SEQUENCE_BOUNDARIES) == "InvalidSequenceBoundaries"
    assert abi.status_string(abi.NON_FINITE_INPUT) == "NonFiniteInput"
    assert abi.status_string(12345) == "Unknown"


def _vision_plan(cu, tokens, heads=16, head_dim=72):
    arr = np.asarray(cu, dtype=np.uint32)
    plan = abi.Plan()
    st = abi.lib().pvlc_plan_vision_varlen(arr.ctypes.data_as(ctypes.c_void_p), len(cu) - 1,
                                           tokens, heads, head_dim, ctypes.byref(plan))
    return st, plan


def test_vision_plan_config2():
    st, plan = _vision_plan([0, 1024, 3328, 3904, 8000], 8000)
    assert st == abi.OK
    assert plan.flops == pytest.approx(1.0813e11, rel=1e-4)      # 4*72*16*sum n_i^2
    assert plan.output_elements == 8000 * 16 * 72
    assert plan.work_items == plan.grid[0] * plan.grid[1]
    # scratch for the rotated q and k of the two-pass rotation + attention
    assert plan.workspace_bytes == 2 * 8000 * 16 * 72 * 2
    assert abi.lib().pvlc_attn_vision_workspace_bytes(8000, 16, 72) == plan.workspace_bytes
    assert abi.lib().pvlc_attn_vision_workspace_bytes(8000, 16, 80) == 0


@pytest.mark.parametrize("args,code", [
    (([0, 8], 0, 16, 72), abi.ZERO_DIMENSION),
    (([0, 8], 8, 0, 72), abi.ZERO_DIMENSION),
    (([0, 8], 8, 16, 0), abi.ZERO_DIMENSION),
    (([0, 8], 8, 16, 80), abi.UNSUPPORTED_HEAD_DIMENSION),     # > MAX_VISION_HEAD_DIM
    (([0, 4, 4, 8], 8, 16, 72), abi.INVALID_SEQUENCE_BOUNDARIES),
    (([1, 8], 8, 16, 72), abi.INVALID_SEQUENCE_BOUNDARIES),
    (([0, 7], 8, 16, 72), abi.INVALID_SEQUENCE_BOUNDARIES),
])
def test_vision_plan_rejections(args, code):
    # precedence as in crates/pvlc-runtime-core/src/lib.rs:443-478: zero dims,
    # head-dim limit, then sequence boundaries
    st, _ = _vision_plan(*args)
    assert st == code


def test_decoder_prefill_plan():
    plan = abi.Plan()
    assert abi.lib().pvlc_plan_decoder_prefill(1564, 1820, 1820, ctypes.byref(plan)) == abi.OK
    assert plan.flops == pytest.approx(1.00256e10, rel=1e-4)   # 4*128*16*T(T+1)/2
    # 98 Q tiles per KV head: the 48 lightest paired, so 2 x (50 + 24) = 148 CTAs
    assert plan.work_items == 2 * 98
    assert (plan.grid[0], plan.grid[1]) == (2, 74)
    assert abi.lib().pvlc_plan_decoder_prefill(0, 10, 10, ctypes.byref(plan)) == abi.ZERO_DIMENSION
    assert abi.lib().pvlc_plan_decoder_prefill(11, 10, 20, ctypes.byref(plan)) == abi.CAPACITY_EXHAUSTED
    assert (abi.lib().pvlc_plan_decoder_prefill(11, 20, 10, ctypes.byref(plan))
            == abi.INVALID_DECODER_GEOMETRY)


@pytest.mark.parametrize("geom,code", [
    ((16, 2, 128, 5, 10), abi.OK),
    ((0, 2, 128, 5, 10), abi.ZERO_DIMENSION),
    ((16, 2, 128, 0, 10), abi.ZERO_DIMENSION),
    ((16, 2, 256, 5, 10), abi.UNSUPPORTED_HEAD_DIMENSION),
    ((16, 4, 128, 5, 10), abi.INVALID_DECODER_GEOMETRY),       # pinned Q16/KV2/D128
    ((15, 2, 128, 5, 10), abi.INVALID_DECODER_GEOMETRY),
    ((16, 2, 64, 5, 10), abi.INVALID_DECODER_GEOMETRY),
    ((16, 2, 128, 10, 10), abi.INVALID_DECODER_GEOMETRY),      # no append slot
])
def test_kv_session_plan_mirrors_reference(geom, code):
    # crates/pvlc-runtime-core/src/lib.rs:1091-1159 plan_decoder_kv_session_geometry
    plan = abi.Plan()
    assert abi.lib().pvlc_plan_decoder_kv_session(*geom, ctypes.byref(plan)) == code


def test_decode_plan_balances_tiles():
    rng = np.random.default_rng(1)
    ct = rng.integers(512, 8193, size=64).astype(np.uint32)
    plan = abi.Plan()
    st = abi.lib().pvlc_plan_decode(ct.ctypes.data_as(ctypes.c_void_p), 64, 8192 + 257,
                                    ctypes.byref(plan))
    assert st == abi.OK
    tiles = int(((ct + 1 + 31) // 32).sum())
    assert plan.work_items == tiles
    assert plan.grid[0] == min(tiles, 148)
    assert plan.hbm_bytes == pytest.approx(float((ct + 1).sum()) * 1024 + 64 * 9216)
    assert plan.workspace_bytes > 0
    bad = np.array([5, 9000], np.uint32)
    assert abi.lib().pvlc_plan_decode(bad.ctypes.data_as(ctypes.c_void_p), 2, 9000,
                                      ctypes.byref(plan)) == abi.CAPACITY_EXHAUSTED


@pytest.mark.parametrize("q_stride,kv_stride", [(2047, 256), (2048, 255), (2052, 256),
                                                (2560, 260)])
def test_decode_strided_rejects_bad_strides_before_any_device_call(q_stride, kv_stride):
    """Row strides below one row or not a 16-byte multiple return LengthMismatch from the
    host-side checks (no device is touched: this runs without a GPU)."""
    fake = ctypes.c_void_p(256)     # never dereferenced: the call returns first
    st = abi.lib().pvlc_attn_decode_strided(
        fake, q_stride, fake, fake, kv_stride, fake, fake, 64, None, fake, fake, fake,
        64, 10, 4, fake, 1 << 20, fake, None)
    assert st == abi.LENGTH_MISMATCH


def test_batched_prefill_host_validation():
    """Geometry errors of pvlc_attn_decoder_prefill_batch come from host checks, before
    any device call (this runs without a GPU)."""
    fake = ctypes.c_void_p(256)
    tab = (ctypes.c_void_p * 2)(256, 512)
    rows = (ctypes.c_uint32 * 2)(64, 64)
    fn = abi.lib().pvlc_attn_decoder_prefill_batch

    def call(offsets, prompts, stride=64 * 256, cap=64):
        offs = (ctypes.c_uint32 * len(offsets))(*offsets)
        return fn(fake, fake, fake, offs, prompts, tab, tab, rows, fake, fake, stride, cap,
                  fake, None)

    assert call([0, 10, 20], 0) == abi.ZERO_DIMENSION
    assert call([0, 10, 20], 257) == abi.INVALID_DECODER_GEOMETRY
    assert call([1, 10, 20], 2) == abi.INVALID_SEQUENCE_BOUNDARIES
    assert call([0, 10, 10], 2) == abi.INVALID_SEQUENCE_BOUNDARIES     # empty prompt
    assert call([0, 10, 90], 2) == abi.CAPACITY_EXHAUSTED               # 80 tokens > 64
    assert call([0, 10, 20], 2, stride=64 * 256 - 8) == abi.LENGTH_MISMATCH


def test_linear_host_validation():
    """pvlc_linear rejects bad geometry and splits before any device call."""
    lib = abi.lib()
    p = ctypes.c_void_p(1 << 20)     # aligned, never dereferenced: every case fails first
    def call(rows=32, ldx=1024, n=2560, k=1024, gate=0, split=8, ldo=2560, x=p, w=p, out=p):
        return lib.pvlc_linear(x, rows, ldx, w, n, k, gate, split, out, ldo, None)
    assert call(rows=0) == abi.ZERO_DIMENSION
    assert call(n=0) == abi.ZERO_DIMENSION
    for bad in (dict(rows=257), dict(n=2500, ldo=2500), dict(k=1000, ldx=1000), dict(ldx=1020),
                dict(ldo=2552), dict(ldo=2564), dict(gate=2), dict(split=3), dict(split=32),
                dict(k=128, ldx=128, split=4), dict(gate=1, n=6144, ldo=3068)):
        assert call(**bad) == abi.INVALID_DECODER_GEOMETRY, bad
    assert call(x=None) == abi.NULL_POINTER
    assert call(out=None) == abi.NULL_POINTER
    assert call(w=ctypes.c_void_p((1 << 20) + 8)) == abi.MISALIGNED_POINTER
    assert call(out=ctypes.c_void_p((1 << 20) + 2)) == abi.MISALIGNED_POINTER
