"""Host-side position and RoPE-table preparation for the attention paths.

Product code (numpy), restating the reference engine's host math:
  * vision 2-D RoPE tables  -- web/engine/multimodal_ocr.mjs:98-155 (visionRope2dTables)
  * decoder M-RoPE tables   -- web/engine/multimodal_ocr.mjs:937-986 (ropeTables)
  * M-RoPE position ids     -- crates/pvlc-cpu-ref/src/multimodal.rs:28-78,249-373
  * decode position         -- crates/pvlc-cpu-ref/src/multimodal.rs:80-113
All angles are computed in float64 and stored as float32, as the reference host does.
"""
from __future__ import annotations

import numpy as np

IMAGE_TOKEN_ID = 100295
VISION_START_TOKEN_ID = 101305
SPATIAL_MERGE_SIZE = 2
DECODER_ROPE_THETA = 500000.0
VISION_ROPE_THETA = 10000.0
DECODER_HEAD_DIM = 128
VISION_HEAD_DIM = 72
MROPE_SECTIONS = (16, 24, 24)


class PositionError(ValueError):
    """Malformed prompt / geometry (the reference's InvalidSequenceBoundaries)."""


def vision_rope_tables(grids_thw, head_dim: int = VISION_HEAD_DIM,
                       theta: float = VISION_ROPE_THETA):
    """[tokens, head_dim/2] cos/sin tables for patch grids (t, h, w); pair p < hd/4 uses the
    row index, the rest the column index; frequency index p mod hd/4."""
    if head_dim <= 0 or head_dim % 4:
        raise PositionError("vision RoPE head_dim must be positive and divisible by four")
    pair_count = head_dim // 2
    freq_count = pair_count // 2
    pairs = np.arange(pair_count)
    inv = float(theta) ** (-(2.0 * (pairs % freq_count)) / pair_count)
    rows = []
    for t, h, w in grids_thw:
        if min(t, h, w) <= 0:
            raise PositionError("vision grid dimensions must be positive")
        y, x = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
        y = np.tile(y.reshape(-1), t)
        x = np.tile(x.reshape(-1), t)
        pos = np.where(pairs[None, :] < freq_count, y[:, None], x[:, None]).astype(np.float64)
        rows.append(pos * inv[None, :])
    ang = np.concatenate(rows, axis=0)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def mrope_position_ids(input_ids, grids_thw, image_token_id: int = IMAGE_TOKEN_ID,
                       vision_start_token_id: int = VISION_START_TOKEN_ID,
                       spatial_merge_size: int = SPATIAL_MERGE_SIZE):
    """(positions [3, n] int64, rope_delta) for a prompt of text and image runs."""
    ids = [int(v) for v in input_ids]
    if not ids or image_token_id == vision_start_token_id:
        raise PositionError("empty prompt")
    grids = []
    for t, h, w in grids_thw:
        if min(t, h, w) <= 0 or h % spatial_merge_size or w % spatial_merge_size:
            raise PositionError("invalid image geometry")
        hm, wm = h // spatial_merge_size, w // spatial_merge_size
        grids.append((t, hm, wm, t * hm * wm))
    n = len(ids)
    if not grids:
        if any(v in (image_token_id, vision_start_token_id) for v in ids):
            raise PositionError("image tokens without image grids")
        pos = np.tile(np.arange(n, dtype=np.int64), (3, 1))
        return pos, int(pos.max()) + 1 - n
    axes = [[], [], []]
    cursor, gi, nxt = 0, 0, 0
    while True:
        try:
            vs = ids.index(vision_start_token_id, cursor)
        except ValueError:
            break
        if image_token_id in ids[cursor:vs] or gi >= len(grids):
            raise PositionError("image run outside a vision_start block")
        t, hm, wm, tokens = grids[gi]
        start, end = vs + 1, vs + 1 + tokens
        if end > n or any(v != image_token_id for v in ids[start:end]) or (
                end < n and ids[end] == image_token_id):
            raise PositionError("image run length does not match its grid")
        text_len = start - cursor
        for a in axes:
            a.extend(range(nxt, nxt + text_len))
        vstart = nxt + text_len
        yy, xx = np.meshgrid(np.arange(hm), np.arange(wm), indexing="ij")
        axes[0].extend([vstart] * tokens)
        axes[1].extend(np.tile(vstart + yy.reshape(-1), t).tolist())
        axes[2].extend(np.tile(vstart + xx.reshape(-1), t).tolist())
        nxt = vstart + max(hm - 1, wm - 1) + 1
        cursor, gi = end, gi + 1
    if gi != len(grids) or any(v in (image_token_id, vision_start_token_id) for v in ids[cursor:]):
        raise PositionError("unused image grids or trailing image tokens")
    for a in axes:
        a.extend(range(nxt, nxt + n - cursor))
    pos = np.array(axes, dtype=np.int64)
    return pos, int(pos.max()) + 1 - n


def decode_position(cache_position: int, rope_delta: int) -> int:
    p = int(cache_position) + int(rope_delta)
    if p < 0:
        raise PositionError("decode position is negative")
    return p


def mrope_tables(positions, rope_delta: int, capacity: int | None = None,
                 theta: float = DECODER_ROPE_THETA, head_dim: int = DECODER_HEAD_DIM):
    """Axis-major [3, capacity, head_dim] cos/sin tables; rows past the prompt continue
    at (row + rope_delta) on every axis."""
    pos = np.asarray(positions, dtype=np.int64).reshape(3, -1)
    prompt = pos.shape[1]
    cap = prompt if capacity is None else int(capacity)
    if prompt == 0 or cap < prompt:
        raise PositionError("rope table capacity is smaller than the prompt")
    half = head_dim // 2
    inv = float(theta) ** (-(2.0 * np.arange(half)) / head_dim)
    rows = np.arange(cap, dtype=np.int64)
    full = np.empty((3, cap), np.float64)
    for a in range(3):
        full[a, :prompt] = pos[a]
        full[a, prompt:] = rows[prompt:] + rope_delta
    ang = full[:, :, None] * inv[None, None, :]
    ang = np.concatenate([ang, ang], axis=2)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def linear_rope_tables(rows: int, theta: float = DECODER_ROPE_THETA,
                       head_dim: int = DECODER_HEAD_DIM):
    """Tables whose row p holds position p on all three axes (text-only / decode rows)."""
    pos = np.tile(np.arange(rows, dtype=np.int64), (3, 1))
    return mrope_tables(pos, 0, rows, theta, head_dim)
