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
    srcs = [os.path.join(_HERE, f) for f in ("pvlc_oracle.cpp", "pvlc_model_oracle.cpp",
                                                  "pvlc_checkpoint_oracle.cpp")]
    if not os.path.exists(_LIB_PATH) or \
            os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
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


# ----------------------------------------------------------------- model level
def linear(x, weight, bias=None):
    """x [rows, in] @ weight[out, in]^T (+ bias): the reference's linear_f32 order."""
    x, w = _f32(x), _f32(weight)
    rows, iw = x.reshape(-1, x.shape[-1]).shape
    ow = w.shape[0]
    b = None if bias is None else _f32(bias)
    out = np.empty((rows, ow), np.float32)
    _check(lib().pvlc_oracle_linear(_p(x), ctypes.c_uint32(rows), ctypes.c_uint32(iw), _p(w),
                                    _p(b) if b is not None else None, ctypes.c_uint32(ow),
                                    _p(out)))
    return out


def rms_norm(x, weight, eps):
    x, w = _f32(x), _f32(weight)
    out = np.empty_like(x)
    rows, width = x.reshape(-1, x.shape[-1]).shape
    _check(lib().pvlc_oracle_rms_norm(_p(x), ctypes.c_uint32(rows), ctypes.c_uint32(width), _p(w),
                                      ctypes.c_float(eps), _p(out)))
    return out


def layer_norm(x, weight, bias, eps):
    x, w, b = _f32(x), _f32(weight), _f32(bias)
    out = np.empty_like(x)
    rows, width = x.reshape(-1, x.shape[-1]).shape
    _check(lib().pvlc_oracle_layer_norm(_p(x), ctypes.c_uint32(rows), ctypes.c_uint32(width),
                                        _p(w), _p(b), ctypes.c_float(eps), _p(out)))
    return out


def prefill_last_logits(final_norm, lm_head):
    fn, w = _f32(final_norm), _f32(lm_head)
    tokens, hidden = fn.reshape(-1, w.shape[1]).shape
    out = np.empty(w.shape[0], np.float32)
    _check(lib().pvlc_oracle_prefill_last_logits(_p(fn), ctypes.c_uint32(tokens),
                                                 ctypes.c_uint32(hidden), _p(w),
                                                 ctypes.c_uint32(w.shape[0]), _p(out)))
    return out


DECODER_TRACE_FIELDS = ("norm1", "query", "key", "value", "mrope_query", "mrope_key",
                        "attention_context", "attention_output", "attention_residual", "norm2",
                        "mlp_gate", "mlp_up", "mlp_activation", "mlp_down", "output")


def decoder_layer_prefill(x, tokens, hidden, intermediate, query_heads, kv_heads, head_dim, eps,
                          sections, raw_cos, raw_sin, weights):
    """One f32 decoder prefill layer; weights = (input_norm, q, k, v, o, post_norm, gate, up,
    down).  Returns the trace as a dict of the reference's field names."""
    x, c, s = _f32(x), _f32(raw_cos), _f32(raw_sin)
    ws = [_f32(w) for w in weights]
    qw, kw = query_heads * head_dim, kv_heads * head_dim
    widths = {"norm1": hidden, "query": qw, "key": kw, "value": kw, "mrope_query": qw,
              "mrope_key": kw, "attention_context": qw, "attention_output": hidden,
              "attention_residual": hidden, "norm2": hidden, "mlp_gate": intermediate,
              "mlp_up": intermediate, "mlp_activation": intermediate, "mlp_down": hidden,
              "output": hidden}
    trace = {k: np.empty(tokens * widths[k], np.float32) for k in DECODER_TRACE_FIELDS}
    wp = (ctypes.c_void_p * 9)(*[w.ctypes.data for w in ws])
    tp = (ctypes.c_void_p * 15)(*[trace[k].ctypes.data for k in DECODER_TRACE_FIELDS])
    sec = _u32(sections)
    _check(lib().pvlc_oracle_decoder_layer_prefill(
        _p(x), ctypes.c_uint32(tokens), ctypes.c_uint32(hidden), ctypes.c_uint32(intermediate),
        ctypes.c_uint32(query_heads), ctypes.c_uint32(kv_heads), ctypes.c_uint32(head_dim),
        ctypes.c_float(eps), _p(sec), _p(c), _p(s), wp, tp))
    return trace


class ModelDims(ctypes.Structure):
    """Mirror of pvlc_oracle_model_dims (oracle/pvlc_model_oracle.cpp)."""
    _fields_ = [("vision_theta", ctypes.c_double), ("decoder_theta", ctypes.c_double),
                ("vision_eps", ctypes.c_float), ("projector_eps", ctypes.c_float),
                ("decoder_eps", ctypes.c_float), ("reserved", ctypes.c_float)] + \
               [(n, ctypes.c_uint32) for n in (
                   "vision_layers", "vision_hidden", "vision_heads", "vision_head_dim",
                   "vision_intermediate", "patch_input", "pos_side", "merge", "decoder_layers",
                   "decoder_hidden", "query_heads", "kv_heads", "head_dim",
                   "decoder_intermediate", "vocab", "eos_token_id", "image_token_id",
                   "vision_start_token_id")] + \
               [("sections", ctypes.c_uint32 * 3), ("reserved2", ctypes.c_uint32)]


def generate(dims: dict, vision_w, projector_w, decoder_w, patches, grids, input_ids,
             max_new_tokens, fp16_storage=True, want_logits=False, want_features=False):
    """One request end to end (pvlc_oracle_generate).  Weight lists hold fp16 numpy arrays in
    the documented order.  Returns dict(tokens, logits?, vision?, projector?)."""
    d = ModelDims()
    for k, v in dims.items():
        if k == "sections":
            d.sections[:] = list(v)
        else:
            setattr(d, k, v)
    keep = []

    def table(ws):
        arrs = [np.ascontiguousarray(w).view(np.uint16) for w in ws]
        keep.extend(arrs)
        return (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])

    vt, pt, dt = table(vision_w), table(projector_w), table(decoder_w)
    p = _f32(patches)
    g = _u32(grids).reshape(-1)
    ids = _u32(input_ids)
    toks = np.zeros(max_new_tokens, np.uint32)
    n = ctypes.c_uint32(0)
    logits = np.empty((max_new_tokens, d.vocab), np.float32) if want_logits else None
    n_patches = int(sum(int(g[i]) * int(g[i + 1]) * int(g[i + 2]) for i in range(0, len(g), 3)))
    vis = np.empty((n_patches, d.vision_hidden), np.float32) if want_features else None
    proj = (np.empty((n_patches // (d.merge * d.merge), d.decoder_hidden), np.float32)
            if want_features else None)
    _check(lib().pvlc_oracle_generate(
        ctypes.byref(d), vt, pt, dt, _p(p), _p(g), ctypes.c_uint32(len(g) // 3), _p(ids),
        ctypes.c_uint32(len(ids)), ctypes.c_uint32(max_new_tokens),
        ctypes.c_int(1 if fp16_storage else 0), _p(toks), ctypes.byref(n),
        _p(logits) if logits is not None else None, _p(vis) if vis is not None else None,
        _p(proj) if proj is not None else None))
    out = {"tokens": toks[: n.value].astype(np.int64).tolist()}
    if want_logits:
        out["logits"] = logits[: n.value]
    if want_features:
        out["vision"], out["projector"] = vis, proj
    return out


def bf16_to_f16_bits(bits):
    """crates/pvlc-safetensors/src/fp16.rs:171-210 element-wise over uint16 BF16 bit
    patterns: returns (f16 bits uint16, status uint8: 0 converted, 1 non-finite,
    2 out of the f16 range)."""
    src = np.ascontiguousarray(bits, dtype=np.uint16).reshape(-1)
    dst = np.zeros_like(src)
    status = np.zeros(src.shape, np.uint8)
    lib().pvlc_oracle_bf16_to_f16_bits(_p(src), _p(dst), _p(status), ctypes.c_uint64(src.size))
    return dst, status


def stream_bf16_to_f16(bits):
    """crates/pvlc-safetensors/src/fp16.rs:212-276: converts in order, stopping at the
    first rejected element.  Returns (f16 bits, None) or (None, (index, status))."""
    src = np.ascontiguousarray(bits, dtype=np.uint16).reshape(-1)
    dst = np.zeros_like(src)
    index = ctypes.c_uint64(0)
    status = lib().pvlc_oracle_stream_bf16_to_f16(_p(src), _p(dst), ctypes.c_uint64(src.size),
                                                  ctypes.byref(index))
    if status:
        return None, (index.value, status)
    return dst, None
