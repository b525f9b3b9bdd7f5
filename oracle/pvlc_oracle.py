"""ctypes view of the CPU oracle (``libpvlc_oracle.so``) -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference legs may import this module; it is the checker, never the measured
or shipped path.  Each wrapper takes and returns float32 / uint32 / int64 numpy
arrays and raises ``OracleError`` carrying the reference's ``CpuRefErrorCode``
number (crates/pvlc-cpu-ref/src/lib.rs:15-29).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libpvlc_oracle.so")

ERROR_NAMES = {
    1: "DimensionMismatch",
    3: "AllMasked",
    4: "InvalidRotaryDimension",
    5: "InvalidRopeBase",
    7: "NonFiniteInput",
    8: "InvalidImageGeometry",
    11: "InvalidSequenceBoundaries",
    12: "InvalidTileSize",
}


class OracleError(RuntimeError):
    def __init__(self, code: int):
        super().__init__(f"oracle error {code} ({ERROR_NAMES.get(code, '?')})")
        self.code = code
        self.name = ERROR_NAMES.get(code, "?")


def build() -> str:
    """Compile the oracle with its Makefile (only when the library is missing or stale)."""
    src = os.path.join(_HERE, "pvlc_oracle.cpp")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.pvlc_oracle_threads.restype = ctypes.c_int
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a):
    return np.ascontiguousarray(a, dtype=np.uint32)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(status: int):
    if status != 0:
        raise OracleError(status)


def threads() -> int:
    return lib().pvlc_oracle_threads()


def set_threads(n: int) -> None:
    lib().pvlc_oracle_set_threads(ctypes.c_int(n))


def vision_rope_2d(query, key, tokens, heads, head_dim, pos_hw, base=10000.0):
    q, k = _f32(query), _f32(key)
    pos = _u32(pos_hw).reshape(-1)
    qo, ko = np.empty_like(q), np.empty_like(k)
    _check(lib().pvlc_oracle_vision_rope_2d(_p(q), _p(k), ctypes.c_uint32(tokens),
                                            ctypes.c_uint32(heads), ctypes.c_uint32(head_dim),
                                            _p(pos), ctypes.c_float(base), _p(qo), _p(ko)))
    return qo, ko


def vision_rope_tables(grids_thw, head_dim=72, theta=10000.0):
    g = _u32(grids_thw).reshape(-1, 3)
    tokens = int(sum(int(t) * int(h) * int(w) for t, h, w in g))
    c = np.empty((tokens, head_dim // 2), np.float32)
    s = np.empty_like(c)
    _check(lib().pvlc_oracle_vision_rope_tables(_p(g), ctypes.c_uint32(len(g)),
                                                ctypes.c_uint32(head_dim), ctypes.c_double(theta),
                                                _p(c), _p(s)))
    return c, s


def vision_rope_apply_tables(query, key, tokens, heads, head_dim, cos_t, sin_t):
    q, k, c, s = _f32(query), _f32(key), _f32(cos_t), _f32(sin_t)
    qo, ko = np.empty_like(q), np.empty_like(k)
    _check(lib().pvlc_oracle_vision_rope_apply_tables(
        _p(q), _p(k), ctypes.c_uint32(tokens), ctypes.c_uint32(heads), ctypes.c_uint32(head_dim),
        _p(c), _p(s), _p(qo), _p(ko)))
    return qo, ko


def segmented_attention(query, key, value, tokens, heads, head_dim, cu_seqlens):
    q, k, v = _f32(query), _f32(key), _f32(value)
    cu = _u32(cu_seqlens)
    out = np.empty_like(q)
    _check(lib().pvlc_oracle_segmented_attention(
        _p(q), _p(k), _p(v), ctypes.c_uint32(tokens), ctypes.c_uint32(heads),
        ctypes.c_uint32(head_dim), _p(cu), ctypes.c_uint32(len(cu)), _p(out)))
    return out


def streaming_segmented_attention(query, key, value, tokens, heads, head_dim, cu_seqlens,
                                  key_tile=16, reverse=False):
    q, k, v = _f32(query), _f32(key), _f32(value)
    cu = _u32(cu_seqlens)
    out = np.empty_like(q)
    _check(lib().pvlc_oracle_streaming_segmented_attention(
        _p(q), _p(k), _p(v), ctypes.c_uint32(tokens), ctypes.c_uint32(heads),
        ctypes.c_uint32(head_dim), _p(cu), ctypes.c_uint32(len(cu)), ctypes.c_uint32(key_tile),
        ctypes.c_int(1 if reverse else 0), _p(out)))
    return out


def apply_multimodal_rope(query, key, tokens, query_heads, kv_heads, head_dim, raw_cos, raw_sin,
                          sections=(16, 24, 24)):
    q, k, c, s = _f32(query), _f32(key), _f32(raw_cos), _f32(raw_sin)
    sec = _u32(sections)
    qo, ko = np.empty_like(q), np.empty_like(k)
    _check(lib().pvlc_oracle_apply_multimodal_rope(
        _p(q), _p(k), ctypes.c_uint32(tokens), ctypes.c_uint32(query_heads),
        ctypes.c_uint32(kv_heads), ctypes.c_uint32(head_dim), _p(c), _p(s), _p(sec), _p(qo),
        _p(ko)))
    return qo, ko


def rope_tables(positions, rope_delta, capacity=None, theta=500000.0, head_dim=128):
    pos = np.ascontiguousarray(positions, dtype=np.int64).reshape(3, -1)
    prompt = pos.shape[1]
    cap = prompt if capacity is None else int(capacity)
    c = np.empty((3, cap, head_dim), np.float32)
    s = np.empty_like(c)
    _check(lib().pvlc_oracle_rope_tables(_p(pos), ctypes.c_uint32(prompt),
                                         ctypes.c_int64(int(rope_delta)), ctypes.c_uint32(cap),
                                         ctypes.c_double(theta), ctypes.c_uint32(head_dim), _p(c),
                                         _p(s)))
    return c, s


def causal_gqa(query, key, value, tokens, query_heads, kv_heads, head_dim):
    q, k, v = _f32(query), _f32(key), _f32(value)
    out = np.empty_like(q)
    _check(lib().pvlc_oracle_causal_gqa(_p(q), _p(k), _p(v), ctypes.c_uint32(tokens),
                                        ctypes.c_uint32(query_heads), ctypes.c_uint32(kv_heads),
                                        ctypes.c_uint32(head_dim), _p(out)))
    return out


def decode_gqa(query, key, value, cache_tokens, query_heads, kv_heads, head_dim):
    q, k, v = _f32(query), _f32(key), _f32(value)
    out = np.empty(query_heads * head_dim, np.float32)
    _check(lib().pvlc_oracle_decode_gqa(_p(q), _p(k), _p(v), ctypes.c_uint32(cache_tokens),
                                        ctypes.c_uint32(query_heads), ctypes.c_uint32(kv_heads),
                                        ctypes.c_uint32(head_dim), _p(out)))
    return out


def decode_step(query, key_new, value_new, rope_cos, rope_sin, rope_row, key_cache, value_cache,
                prefix_tokens, sections=(16, 24, 24), query_heads=16, kv_heads=2, head_dim=128):
    """Rotate, append at row ``prefix_tokens`` (in place on the f32 caches), attend."""
    q, kn, vn = _f32(query), _f32(key_new), _f32(value_new)
    c, s = _f32(rope_cos), _f32(rope_sin)
    assert key_cache.dtype == np.float32 and key_cache.flags.c_contiguous
    assert value_cache.dtype == np.float32 and value_cache.flags.c_contiguous
    rope_rows = c.size // (3 * head_dim)
    capacity = key_cache.size // (kv_heads * head_dim)
    sec = _u32(sections)
    out = np.empty(query_heads * head_dim, np.float32)
    _check(lib().pvlc_oracle_decode_step(
        _p(q), _p(kn), _p(vn), _p(c), _p(s), ctypes.c_uint32(rope_rows), ctypes.c_uint32(rope_row),
        _p(sec), _p(key_cache), _p(value_cache), ctypes.c_uint32(prefix_tokens),
        ctypes.c_uint32(capacity), ctypes.c_uint32(query_heads), ctypes.c_uint32(kv_heads),
        ctypes.c_uint32(head_dim), _p(out)))
    return out


def decoder_prefill(query, key, value, rope_cos, rope_sin, tokens, key_cache, value_cache,
                    sections=(16, 24, 24), query_heads=16, kv_heads=2, head_dim=128):
    q, k, v = _f32(query), _f32(key), _f32(value)
    c, s = _f32(rope_cos), _f32(rope_sin)
    rope_rows = c.size // (3 * head_dim)
    capacity = key_cache.size // (kv_heads * head_dim)
    sec = _u32(sections)
    out = np.empty((tokens, query_heads, head_dim), np.float32)
    _check(lib().pvlc_oracle_decoder_prefill(
        _p(q), _p(k), _p(v), _p(c), _p(s), ctypes.c_uint32(rope_rows), _p(sec),
        ctypes.c_uint32(tokens), ctypes.c_uint32(query_heads), ctypes.c_uint32(kv_heads),
        ctypes.c_uint32(head_dim), _p(key_cache), _p(value_cache), ctypes.c_uint32(capacity),
        _p(out)))
    return out


def mrope_position_ids(input_ids, grids_thw, image_token_id=100295, vision_start_token_id=101305,
                       spatial_merge_size=2):
    ids = _u32(input_ids)
    g = _u32(grids_thw).reshape(-1)
    pos = np.empty((3, len(ids)), np.int64)
    delta = ctypes.c_int64(0)
    _check(lib().pvlc_oracle_mrope_position_ids(
        _p(ids), ctypes.c_uint32(len(ids)), _p(g), ctypes.c_uint32(len(g) // 3),
        ctypes.c_uint32(image_token_id), ctypes.c_uint32(vision_start_token_id),
        ctypes.c_uint32(spatial_merge_size), _p(pos), ctypes.byref(delta)))
    return pos, int(delta.value)


def decode_mrope_position(cache_position, rope_delta):
    out = ctypes.c_int64(0)
    _check(lib().pvlc_oracle_decode_mrope_position(ctypes.c_uint32(cache_position),
                                                   ctypes.c_int64(rope_delta), ctypes.byref(out)))
    return int(out.value)
