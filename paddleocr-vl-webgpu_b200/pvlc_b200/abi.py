"""ctypes binding of ``libpvlc_cuda_attn.so`` (the C ABI in include/pvlc_cuda_attn.h).

This is the reference-facing boundary: the same entry points a Rust
``extern "C"`` block or a cgo stub would bind.  Loading fails loudly when the
library is missing -- there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpvlc_cuda_attn.so")
HEADER_PATH = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include",
                           "pvlc_cuda_attn.h")

# Status codes (mirror include/pvlc_cuda_attn.h; 1..15 follow the reference's
# InvocationErrorCode order, crates/pvlc-runtime-core/src/lib.rs:5335-5351).
OK = 0
ZERO_DIMENSION = 1
LENGTH_MISMATCH = 2
ARITHMETIC_OVERFLOW = 3
INVALID_ROTARY_DIMENSION = 5
INVALID_ROPE_BASE = 6
UNSUPPORTED_HEAD_DIMENSION = 7
INVALID_DECODER_GEOMETRY = 8
INVALID_VISION_GEOMETRY = 9
INVALID_SEQUENCE_BOUNDARIES = 11
NON_FINITE_INPUT = 15
NULL_POINTER = 64
MISALIGNED_POINTER = 65
WORKSPACE_TOO_SMALL = 66
CAPACITY_EXHAUSTED = 67
CUDA_ERROR = 68
DEVICE_UNSUPPORTED = 69
DEVICE_FAULT_FLAG = 70


class PvlcError(RuntimeError):
    """A nonzero status from the library (the reference's InvocationError)."""

    def __init__(self, status: int, where: str = ""):
        self.status = status
        self.name = status_string(status)
        super().__init__(f"{where}: {self.name} ({status})" if where else f"{self.name} ({status})")


class Plan(ctypes.Structure):
    _fields_ = [
        ("grid", ctypes.c_uint32 * 3),
        ("block", ctypes.c_uint32 * 3),
        ("shared_bytes", ctypes.c_uint32),
        ("work_items", ctypes.c_uint32),
        ("output_elements", ctypes.c_uint64),
        ("output_bytes", ctypes.c_uint64),
        ("workspace_bytes", ctypes.c_uint64),
        ("flops", ctypes.c_double),
        ("hbm_bytes", ctypes.c_double),
    ]


_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_SIGNATURES = {
    "pvlc_attn_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "pvlc_attn_device_check": (ctypes.c_int, []),
    "pvlc_attn_vision_varlen": (ctypes.c_int, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _P, _P,
                                               _P, _P]),
    "pvlc_attn_vision_workspace_bytes": (ctypes.c_size_t, [_U32, _U32, _U32]),
    "pvlc_attn_vision_varlen_ws": (ctypes.c_int, [_P, _P, _P, _P, _U32, _U32, _U32, _U32, _P, _P,
                                                  _P, ctypes.c_size_t, _P, _P]),
    "pvlc_attn_vision_varlen_strided_ws": (ctypes.c_int, [_P, _P, _P, _U32, _P, _U32, _U32, _U32,
                                                          _U32, _P, _P, _P, ctypes.c_size_t, _P,
                                                          _P]),
    "pvlc_attn_decoder_prefill": (ctypes.c_int, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _P, _P,
                                                 _P, _P]),
    "pvlc_attn_decoder_prefill_batch": (ctypes.c_int, [_P, _P, _P, _P, _U32, _P, _P, _P, _P, _P,
                                                       ctypes.c_uint64, _U32, _P, _P]),
    "pvlc_attn_decode_workspace_bytes": (ctypes.c_size_t, [_U32]),
    "pvlc_attn_decode_workspace_init": (ctypes.c_int, [_P, ctypes.c_size_t, _P]),
    "pvlc_attn_decode": (ctypes.c_int, [_P, _P, _P, _P, _P, _U32, _P, _P, _P, _P, _U32, _U32,
                                        _U32, _P, ctypes.c_size_t, _P, _P]),
    "pvlc_attn_decode_strided": (ctypes.c_int, [_P, _U32, _P, _P, _U32, _P, _P, _U32, _P, _P,
                                                _P, _P, _U32, _U32, _U32, _P, ctypes.c_size_t,
                                                _P, _P]),
    "pvlc_attn_decode_errors": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_uint32), _P]),
    "pvlc_attn_fault_flags": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _P]),
    "pvlc_blake3_workspace_bytes": (ctypes.c_size_t, [ctypes.c_uint64]),
    "pvlc_blake3": (ctypes.c_int, [_P, ctypes.c_uint64, _P, ctypes.c_size_t, _P, _P]),
    "pvlc_attn_decode_noalloc": (ctypes.c_int, [_P, _P, _P, _P, _P, _U32, _P, _P, _P, _P, _U32,
                                                _U32, _U32, _P, _P]),
    "pvlc_image_patches_workspace_bytes": (ctypes.c_size_t, [_U32, _U32, _U32, _U32]),
    "pvlc_image_patches": (ctypes.c_int, [_P, _U32, _U32, _U32, _U32, _U32, _P, ctypes.c_size_t,
                                          _P, _P]),
    "pvlc_add_norm": (ctypes.c_int, [_P, _P, _U32, _U32, _P, _P, ctypes.c_float, _P, _P]),
    "pvlc_gelu": (ctypes.c_int, [_P, ctypes.c_uint64, ctypes.c_int, _P]),
    "pvlc_silu_mul": (ctypes.c_int, [_P, _U32, _U32, _P, _P]),
    "pvlc_bf16_to_f16": (ctypes.c_int, [_P, _P, ctypes.c_uint64, ctypes.c_uint64, _P, _P]),
    "pvlc_lm_head_top1_workspace_bytes": (ctypes.c_size_t, [_U32]),
    "pvlc_lm_head_top1": (ctypes.c_int, [_P, _U32, _P, _U32, _U32, _P, ctypes.c_size_t, _P, _P,
                                         _P]),
    "pvlc_lm_head_top1_errors": (ctypes.c_int, [_P, _U32, ctypes.POINTER(ctypes.c_uint32), _P]),
    "pvlc_linear": (ctypes.c_int, [_P, _U32, _U32, _P, _U32, _U32, _U32, _U32, _P, _U32, _P]),
    "pvlc_plan_vision_varlen": (ctypes.c_int, [_P, _U32, _U32, _U32, _U32, ctypes.POINTER(Plan)]),
    "pvlc_plan_decoder_prefill": (ctypes.c_int, [_U32, _U32, _U32, ctypes.POINTER(Plan)]),
    "pvlc_plan_decoder_kv_session": (ctypes.c_int, [_U32, _U32, _U32, _U32, _U32,
                                                    ctypes.POINTER(Plan)]),
    "pvlc_plan_decode": (ctypes.c_int, [_P, _U32, _U32, ctypes.POINTER(Plan)]),
}
EXPORTED = tuple(_SIGNATURES)

_lib = None


def lib() -> ctypes.CDLL:
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                               "(make -C paddleocr-vl-webgpu_b200); there is no CPU fallback")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def status_string(status: int) -> str:
    return lib().pvlc_attn_status_string(status).decode()


def check(status: int, where: str = "") -> None:
    if status != OK:
        raise PvlcError(status, where)
