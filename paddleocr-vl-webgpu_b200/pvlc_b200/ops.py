"""Torch-facing wrappers over the C ABI (device tensors in, device tensors out).

Each function checks tensor placement, dtype and shape, then calls the C
entry point on the current CUDA stream; the library itself re-validates the
geometry and returns the reference's error code before any device effect.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import abi

QH, KVH, HD = 16, 2, 128
VISION_HD = 72


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(None)


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _need(t, dtype, shape=None, name="tensor"):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


def vision_workspace_bytes(tokens: int, heads: int, head_dim: int = VISION_HD) -> int:
    """Device scratch of a vision call with rope tables (the rotated q and k)."""
    return int(abi.lib().pvlc_attn_vision_workspace_bytes(tokens, heads, head_dim))


def vision_varlen_attention(q, k, v, cu_seqlens, rope_cos=None, rope_sin=None, out=None,
                            workspace=None):
    """Bidirectional block-diagonal attention over packed images with the 2-D RoPE.

    q, k, v: [T, H, 72] fp16 CUDA, each either contiguous or all three views whose
    token rows sit the same number of elements apart (e.g. column blocks of one
    [T, 3 * H * 72] QKV projection: pvlc_attn_vision_varlen_strided_ws);
    cu_seqlens: host sequence of segment boundaries; rope_cos/rope_sin: [T, 36] f32
    CUDA tables or None; workspace: optional uint8 CUDA tensor of at least
    vision_workspace_bytes (taken from torch's allocator when omitted).  Returns
    [T, H, 72] fp16 (contiguous).
    """
    T, H, D = q.shape
    row_stride = H * D
    strided = any(not t.is_contiguous() for t in (q, k, v))
    if strided:
        row_stride = q.stride(0)
        for name, t in (("q", q), ("k", k), ("v", v)):
            if (t.dtype != torch.float16 or tuple(t.shape) != (T, H, D) or not t.is_cuda or
                    t.stride() != (row_stride, D, 1)):
                raise ValueError(f"{name}: expected [T, H, {D}] fp16 CUDA rows {row_stride} "
                                 f"elements apart, got {tuple(t.shape)} strides {t.stride()}")
    else:
        for name, t in (("q", q), ("k", k), ("v", v)):
            _need(t, torch.float16, (T, H, D), name)
    if rope_cos is not None:
        _need(rope_cos, torch.float32, (T, D // 2), "rope_cos")
        _need(rope_sin, torch.float32, (T, D // 2), "rope_sin")
    cu = np.ascontiguousarray(np.asarray(cu_seqlens, dtype=np.uint32))
    if out is None:
        out = torch.empty((T, H, D), dtype=torch.float16, device=q.device)
    ws_bytes = 0
    if rope_cos is not None:
        ws_bytes = vision_workspace_bytes(T, H, D)
        if workspace is None:
            workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        _need(workspace, torch.uint8, None, "workspace")
        ws_bytes = workspace.numel()
    wsp = _ptr(workspace if rope_cos is not None else None)
    if strided:
        st = abi.lib().pvlc_attn_vision_varlen_strided_ws(
            _ptr(q), _ptr(k), _ptr(v), row_stride, cu.ctypes.data_as(ctypes.c_void_p),
            max(len(cu) - 1, 0), T, H, D, _ptr(rope_cos), _ptr(rope_sin), wsp, ws_bytes,
            _ptr(out), _stream())
        abi.check(st, "pvlc_attn_vision_varlen_strided_ws")
        return out
    st = abi.lib().pvlc_attn_vision_varlen_ws(
        _ptr(q), _ptr(k), _ptr(v), cu.ctypes.data_as(ctypes.c_void_p), max(len(cu) - 1, 0), T, H,
        D, _ptr(rope_cos), _ptr(rope_sin), wsp, ws_bytes, _ptr(out), _stream())
    abi.check(st, "pvlc_attn_vision_varlen_ws")
    return out


def decoder_prefill(q, k, v, rope_cos, rope_sin, k_cache, v_cache, out=None):
    """Causal GQA prefill of one decoder layer; writes rotated K / raw V into the caches.

    q: [T,16,128] fp16; k, v: [T,2,128] fp16; rope tables [3, R, 128] f32 (R >= T);
    k_cache, v_cache: [capacity, 2, 128] fp16.  Returns [T,16,128] fp16.
    """
    T = q.shape[0]
    _need(q, torch.float16, (T, QH, HD), "q")
    _need(k, torch.float16, (T, KVH, HD), "k")
    _need(v, torch.float16, (T, KVH, HD), "v")
    R = rope_cos.shape[1]
    _need(rope_cos, torch.float32, (3, R, HD), "rope_cos")
    _need(rope_sin, torch.float32, (3, R, HD), "rope_sin")
    cap = k_cache.shape[0]
    _need(k_cache, torch.float16, (cap, KVH, HD), "k_cache")
    _need(v_cache, torch.float16, (cap, KVH, HD), "v_cache")
    if out is None:
        out = torch.empty_like(q)
    st = abi.lib().pvlc_attn_decoder_prefill(
        _ptr(q), _ptr(k), _ptr(v), _ptr(rope_cos), _ptr(rope_sin), R, T, cap, _ptr(k_cache),
        _ptr(v_cache), _ptr(out), _stream())
    abi.check(st, "pvlc_attn_decoder_prefill")
    return out


MAX_PREFILL_PROMPTS = 256       # PVLC_PREFILL_MAX_PROMPTS
MAX_PREFILL_TILES = 65535       # 16-token Q tiles of one batched launch


def decoder_prefill_packed(q, k, v, offsets, tables, k_caches, v_caches, out):
    """decoder_prefill over B prompts packed back to back: pvlc_attn_decoder_prefill_batch,
    one launch pair per group of at most 256 prompts (and 65535 Q tiles).

    q: [NT,16,128], k, v: [NT,2,128] fp16 with prompt b at rows offsets[b]:offsets[b+1]
    (host integers); tables: B (rope_cos, rope_sin) pairs as decoder_prefill takes them;
    k_caches, v_caches: [B, capacity, 2, 128] fp16 (prompt b's cache at [b]); out like q."""
    NT = q.shape[0]
    _need(q, torch.float16, (NT, QH, HD), "q")
    _need(k, torch.float16, (NT, KVH, HD), "k")
    _need(v, torch.float16, (NT, KVH, HD), "v")
    _need(out, torch.float16, (NT, QH, HD), "out")
    B, cap = k_caches.shape[0], k_caches.shape[1]
    _need(k_caches, torch.float16, (B, cap, KVH, HD), "k_caches")
    _need(v_caches, torch.float16, (B, cap, KVH, HD), "v_caches")
    offs = [int(x) for x in offsets]
    if len(offs) != B + 1 or len(tables) != B or offs[0] != 0 or offs[-1] != NT:
        raise ValueError("offsets / tables do not describe the packed prompts")
    for rc, rs in tables:
        _need(rc, torch.float32, (3, rc.shape[1], HD), "rope_cos")
        _need(rs, torch.float32, (3, rc.shape[1], HD), "rope_sin")
    fn, st = abi.lib().pvlc_attn_decoder_prefill_batch, _stream()
    cstride = cap * KVH * HD             # elements
    b0 = 0
    while b0 < B:
        b1, tiles = b0, 0
        while b1 < B and b1 - b0 < MAX_PREFILL_PROMPTS:
            t = (offs[b1 + 1] - offs[b1] + 15) // 16
            if b1 > b0 and tiles + t > MAX_PREFILL_TILES:
                break
            tiles += t
            b1 += 1
        n = b1 - b0
        r0 = offs[b0]
        offs_c = (ctypes.c_uint32 * (n + 1))(*[x - r0 for x in offs[b0:b1 + 1]])
        cos_c = (ctypes.c_void_p * n)(*[tables[i][0].data_ptr() for i in range(b0, b1)])
        sin_c = (ctypes.c_void_p * n)(*[tables[i][1].data_ptr() for i in range(b0, b1)])
        rows_c = (ctypes.c_uint32 * n)(*[tables[i][0].shape[1] for i in range(b0, b1)])
        status = fn(q.data_ptr() + r0 * QH * HD * 2, k.data_ptr() + r0 * KVH * HD * 2,
                    v.data_ptr() + r0 * KVH * HD * 2, offs_c, n, cos_c, sin_c, rows_c,
                    k_caches.data_ptr() + b0 * cstride * 2, v_caches.data_ptr() + b0 * cstride * 2,
                    cstride, cap, out.data_ptr() + r0 * QH * HD * 2, st)
        abi.check(status, f"pvlc_attn_decoder_prefill_batch (prompts {b0}..{b1 - 1})")
        b0 = b1
    return out


class DecodeWorkspace:
    """Device scratch for batched decode (split partials + combine tickets + fault flags)."""

    def __init__(self, batch: int, device=None):
        self.batch = int(batch)
        self.nbytes = int(abi.lib().pvlc_attn_decode_workspace_bytes(self.batch))
        self.buffer = torch.empty(self.nbytes, dtype=torch.uint8,
                                  device=device or torch.device("cuda"))
        abi.check(abi.lib().pvlc_attn_decode_workspace_init(_ptr(self.buffer), self.nbytes,
                                                            _stream()),
                  "pvlc_attn_decode_workspace_init")

    def errors(self) -> int:
        flags = ctypes.c_uint32(0)
        abi.lib().pvlc_attn_decode_errors(_ptr(self.buffer), ctypes.byref(flags), _stream())
        return int(flags.value)


def blake3(data, digest=None, workspace=None):
    """BLAKE3 (plain hash, 32 bytes) of a contiguous CUDA uint8 tensor, computed on the
    device (pvlc_blake3); returns the [32] uint8 device digest (no host sync)."""
    if not isinstance(data, torch.Tensor) or not data.is_cuda or data.dtype != torch.uint8:
        raise TypeError("data must be a CUDA uint8 tensor")
    if not data.is_contiguous():
        raise ValueError("data must be contiguous")
    n = data.numel()
    need = int(abi.lib().pvlc_blake3_workspace_bytes(n))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=data.device)
    if digest is None:
        digest = torch.empty(32, dtype=torch.uint8, device=data.device)
    st = abi.lib().pvlc_blake3(_ptr(data) if n else None, n, _ptr(workspace), workspace.numel(),
                               _ptr(digest), _stream())
    abi.check(st, "pvlc_blake3")
    return digest


FAULT_VISION, FAULT_PREFILL, FAULT_PREFILL_BATCH, FAULT_LINEAR = 1, 2, 4, 8


def fault_flags() -> int:
    """Read and clear the current device's sticky fault word of the vision, prefill and
    projection kernels (FAULT_* bits: a launch whose bounded pipeline wait ran out and whose output
    is incomplete).  Synchronizes the current stream."""
    flags = ctypes.c_uint32(0)
    st = abi.lib().pvlc_attn_fault_flags(ctypes.byref(flags), _stream())
    if st not in (abi.OK, abi.DEVICE_FAULT_FLAG):
        abi.check(st, "pvlc_attn_fault_flags")
    return int(flags.value)


def _rows(t, dtype, shape, name):
    """Check a [B, H, 128] tensor whose rows may sit at any 16-byte multiple apart (the
    inner [H, 128] contiguous); returns the row stride in elements."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    if t.stride(2) != 1 or t.stride(1) != shape[2] or (shape[0] > 1 and t.stride(0) % 8):
        raise ValueError(f"{name} rows must be contiguous and 16-byte aligned")
    return t.stride(0) if shape[0] > 1 else shape[1] * shape[2]


def decode(q, k_new, v_new, rope_cos, rope_sin, k_cache_ptrs, v_cache_ptrs, cache_tokens,
           capacity: int, max_cache_tokens: int, workspace: DecodeWorkspace, rope_row=None,
           out=None):
    """Batched single-token decode with fused M-RoPE and KV append.

    q: [B,16,128] fp16; k_new/v_new: [B,2,128] fp16 -- each may be a row-strided view
    (e.g. column slices of one [B, 2560] QKV projection; rows contiguous, k_new and v_new
    with the same stride), passed through pvlc_attn_decode_strided; rope tables
    [3, R, 128] f32; k_cache_ptrs/v_cache_ptrs: int64 CUDA tensors of B device pointers
    to [capacity, 2, 128] fp16 caches; cache_tokens: int32 CUDA [B] rows before the
    append; rope_row: optional int32 CUDA [B] (defaults to cache_tokens).
    Returns [B,16,128] fp16.
    """
    B = q.shape[0]
    qs = _rows(q, torch.float16, (B, QH, HD), "q")
    ks = _rows(k_new, torch.float16, (B, KVH, HD), "k_new")
    vs = _rows(v_new, torch.float16, (B, KVH, HD), "v_new")
    if ks != vs:
        raise ValueError("k_new and v_new must share one row stride")
    R = rope_cos.shape[1]
    _need(rope_cos, torch.float32, (3, R, HD), "rope_cos")
    _need(rope_sin, torch.float32, (3, R, HD), "rope_sin")
    _need(k_cache_ptrs, torch.int64, (B,), "k_cache_ptrs")
    _need(v_cache_ptrs, torch.int64, (B,), "v_cache_ptrs")
    _need(cache_tokens, torch.int32, (B,), "cache_tokens")
    if rope_row is not None:
        _need(rope_row, torch.int32, (B,), "rope_row")
    if out is None:
        out = torch.empty((B, QH, HD), dtype=torch.float16, device=q.device)
    _need(out, torch.float16, (B, QH, HD), "out")
    st = abi.lib().pvlc_attn_decode_strided(
        _ptr(q), qs, _ptr(k_new), _ptr(v_new), ks, _ptr(rope_cos), _ptr(rope_sin), R,
        _ptr(rope_row), _ptr(k_cache_ptrs), _ptr(v_cache_ptrs), _ptr(cache_tokens),
        int(capacity), int(max_cache_tokens), B, _ptr(workspace.buffer), workspace.nbytes,
        _ptr(out), _stream())
    abi.check(st, "pvlc_attn_decode_strided")
    return out


def image_patches(rgb, out_height: int, out_width: int, patch_size: int = 14, out=None,
                  workspace=None):
    """Bicubic resample of an [H, W, 3] uint8 CUDA image to (out_height, out_width) and its
    normalised patch-major values [(out_height/p)*(out_width/p), 3*p*p] f32 (the
    reference's canonical_rgb8_to_patches after smart_resize)."""
    if not isinstance(rgb, torch.Tensor) or not rgb.is_cuda or rgb.dtype != torch.uint8 or \
            rgb.dim() != 3 or rgb.shape[2] != 3 or not rgb.is_contiguous():
        raise TypeError("rgb must be a contiguous [H, W, 3] uint8 CUDA tensor")
    H, W = int(rgb.shape[0]), int(rgb.shape[1])
    n = (out_height // patch_size) * (out_width // patch_size)
    if out is None:
        out = torch.empty((n, 3 * patch_size * patch_size), dtype=torch.float32,
                          device=rgb.device)
    _need(out, torch.float32, (n, 3 * patch_size * patch_size), "out")
    need = int(abi.lib().pvlc_image_patches_workspace_bytes(H, W, out_height, out_width))
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=rgb.device)
    _need(workspace, torch.uint8, None, "workspace")
    st = abi.lib().pvlc_image_patches(_ptr(rgb), H, W, out_height, out_width, patch_size,
                                      _ptr(workspace), workspace.numel(), _ptr(out), _stream())
    abi.check(st, "pvlc_image_patches")
    return out


def add_norm(residual, weight, eps: float, bias=None, delta=None, out=None):
    """residual [rows, width] f32 CUDA (+= delta [rows, width] fp16 in place when given), then
    LayerNorm (with bias) or RMSNorm (bias None) of each row * weight (+ bias), as fp16."""
    rows, width = residual.shape
    _need(residual, torch.float32, (rows, width), "residual")
    _need(weight, torch.float32, (width,), "weight")
    if bias is not None:
        _need(bias, torch.float32, (width,), "bias")
    if delta is not None:
        _need(delta, torch.float16, (rows, width), "delta")
    if out is None:
        out = torch.empty((rows, width), dtype=torch.float16, device=residual.device)
    _need(out, torch.float16, (rows, width), "out")
    st = abi.lib().pvlc_add_norm(_ptr(residual), _ptr(delta), rows, width, _ptr(weight),
                                 _ptr(bias), float(eps), _ptr(out), _stream())
    abi.check(st, "pvlc_add_norm")
    return out


def gelu_(x, erf: bool = False):
    """In-place GELU (tanh form, or erf form) of an fp16 CUDA tensor."""
    _need(x, torch.float16, None, "x")
    abi.check(abi.lib().pvlc_gelu(_ptr(x), x.numel(), 1 if erf else 0, _stream()), "pvlc_gelu")
    return x


def silu_mul(gate_up, out=None):
    """[rows, 2I] fp16 (gate | up) -> [rows, I] fp16 silu(gate) * up."""
    rows, w2 = gate_up.shape
    _need(gate_up, torch.float16, (rows, w2), "gate_up")
    if out is None:
        out = torch.empty((rows, w2 // 2), dtype=torch.float16, device=gate_up.device)
    _need(out, torch.float16, (rows, w2 // 2), "out")
    abi.check(abi.lib().pvlc_silu_mul(_ptr(gate_up), rows, w2 // 2, _ptr(out), _stream()),
              "pvlc_silu_mul")
    return out


LINEAR_MAX_ROWS = 256           # PVLC_LINEAR_MAX_ROWS


def _rows_view(t, name):
    """A 2-D fp16 CUDA tensor whose rows may be pitched (stride(1) == 1)."""
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float16:
        raise TypeError(f"{name} must be torch.float16, got {t.dtype}")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with unit column stride")
    return t.stride(0) if t.shape[0] > 1 else max(t.stride(0), t.shape[1])


def gate_up_blocks(gate_w, up_w):
    """The gate-up weight of the fused SiLU projection: 128-row blocks of 64 gate rows
    followed by the 64 up rows of the same output columns ([2I, K] from two [I, K])."""
    i, k = gate_w.shape
    if up_w.shape != (i, k) or i % 64:
        raise ValueError("gate and up weights must both be [I, K] with I a multiple of 64")
    return torch.stack((gate_w.view(i // 64, 64, k), up_w.view(i // 64, 64, k)),
                       dim=1).reshape(2 * i, k).contiguous()


def linear(x, w, out=None, gate=False, split=0):
    """Decode-step projection on the tensor cores (pvlc_linear): x [rows, K] fp16 (rows
    may be pitched) times w [N, K] fp16 -> out [rows, N] fp16 with f32 accumulation, or
    with gate=True (w laid out by gate_up_blocks) out [rows, N / 2] =
    fp16(silu(fp16(gate)) * fp16(up)).  Rows beyond 256 are taken in groups of 256.
    split: K slices per 128-feature tile (0: the library's choice)."""
    rows, K = x.shape
    ldx = _rows_view(x, "x")
    N = w.shape[0]
    _need(w, torch.float16, (N, K), "w")
    width = N // 2 if gate else N
    if out is None:
        out = torch.empty((rows, width), dtype=torch.float16, device=x.device)
    ldo = _rows_view(out, "out")
    if tuple(out.shape) != (rows, width):
        raise ValueError(f"out has shape {tuple(out.shape)}, expected {(rows, width)}")
    for r0 in range(0, rows, LINEAR_MAX_ROWS):
        r1 = min(rows, r0 + LINEAR_MAX_ROWS)
        st = abi.lib().pvlc_linear(
            _ptr(x[r0:r1]), r1 - r0, ldx, _ptr(w), N, K, int(bool(gate)), split,
            _ptr(out[r0:r1]), ldo, _stream())
        abi.check(st, "pvlc_linear")
    return out


LM_HEAD_MAX_ROWS = 256          # PVLC_LM_HEAD_MAX_ROWS


def lm_head_top1(hidden, lm_head, tokens=None, logits=None, workspace=None):
    """Greedy top-1 over the LM head without materialising the logits
    (pvlc_lm_head_top1): hidden [rows, K] fp16 (the final-norm output), lm_head
    [vocab, K] fp16 -> int32 token ids [rows] (the largest f32 logit; equal logits go to
    the smaller id).  logits, when given, is a [rows] f32 tensor that receives the
    winning logit.  Rows beyond 256 are taken in groups of 256."""
    rows, K = hidden.shape
    V = lm_head.shape[0]
    _need(hidden, torch.float16, (rows, K), "hidden")
    _need(lm_head, torch.float16, (V, K), "lm_head")
    if tokens is None:
        tokens = torch.empty(rows, dtype=torch.int32, device=hidden.device)
    _need(tokens, torch.int32, (rows,), "tokens")
    if logits is not None:
        _need(logits, torch.float32, (rows,), "logits")
    need = int(abi.lib().pvlc_lm_head_top1_workspace_bytes(min(rows, LM_HEAD_MAX_ROWS)))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=hidden.device)
    _need(workspace, torch.uint8, None, "workspace")
    for r0 in range(0, rows, LM_HEAD_MAX_ROWS):
        r1 = min(rows, r0 + LM_HEAD_MAX_ROWS)
        st = abi.lib().pvlc_lm_head_top1(
            _ptr(hidden[r0:r1]), r1 - r0, _ptr(lm_head), V, K, _ptr(workspace),
            workspace.numel(), _ptr(tokens[r0:r1]),
            _ptr(logits[r0:r1] if logits is not None else None), _stream())
        abi.check(st, "pvlc_lm_head_top1")
    return tokens
