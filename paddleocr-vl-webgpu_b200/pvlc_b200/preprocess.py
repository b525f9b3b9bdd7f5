"""Image preprocessing for the vision encoder: smart resize, Pillow bicubic, patches.

Restates the reference's canonical RGB8 path
(crates/pvlc-cpu-ref/src/lib.rs:2427-2563, 3066-3273):

* ``smart_resize`` (:2442-2513): round both sides to multiples of
  patch_size x merge_size (Python ties-to-even rounding), then rescale into
  [min_pixels, max_pixels] by floor / ceil of the scaled sides;
* ``pillow_bicubic_rgb8`` (:3092-3273): Pillow's separable bicubic (a = -0.5)
  with 22-bit fixed-point coefficients and int64 accumulation, horizontal pass
  first; exact integer arithmetic, vectorised with numpy;
* ``canonical_rgb8_to_patches`` (:2515-2563): patch-major
  [patch_y, patch_x, channel, y, x] values (byte / 255 in f64, stored f32,
  then (v - 0.5) / 0.5 in f32).

``device_patches`` runs the same resample and patchify on the GPU through
the library's bicubic kernel (bit-identical to the host version).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

INVALID_IMAGE_GEOMETRY = 8
INVALID_PREPROCESS_CONFIG = 9
DIMENSION_MISMATCH = 1


class PreprocessError(ValueError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


@dataclass(frozen=True)
class VisionPreprocessConfig:
    patch_size: int = 14
    merge_size: int = 2
    min_pixels: int = 112_896
    max_pixels: int = 1_003_520


MODEL_CONFIG = VisionPreprocessConfig()


def _validate(config: VisionPreprocessConfig) -> None:
    # crates/pvlc-cpu-ref/src/lib.rs:3066-3076
    if (config.patch_size == 0 or config.merge_size == 0 or config.min_pixels == 0
            or config.max_pixels < config.min_pixels):
        raise PreprocessError(INVALID_PREPROCESS_CONFIG, "invalid preprocess config")


def _round_half_even(v: float) -> int:
    if not math.isfinite(v) or v < 0:
        raise PreprocessError(INVALID_IMAGE_GEOMETRY, "invalid image geometry")
    return int(round(v))          # Python round() is ties-to-even, as f64::round_ties_even


def smart_resize(height: int, width: int, config: VisionPreprocessConfig = MODEL_CONFIG):
    """crates/pvlc-cpu-ref/src/lib.rs:2442-2513 -> (resized_height, resized_width)."""
    _validate(config)
    if height == 0 or width == 0:
        raise PreprocessError(INVALID_IMAGE_GEOMETRY, "empty image")
    factor = config.patch_size * config.merge_size
    h, w = height, width
    if h < factor:
        w = _round_half_even(w * float(factor) / h)
        h = factor
    if w < factor:
        h = _round_half_even(h * float(factor) / w)
        w = factor
    if max(h, w) / min(h, w) > 200.0:
        raise PreprocessError(INVALID_IMAGE_GEOMETRY, "aspect ratio above 200")
    ff = float(factor)
    rh = _round_half_even(h / ff) * factor
    rw = _round_half_even(w / ff) * factor
    if rh * rw > config.max_pixels:
        beta = math.sqrt(float(h * w) / config.max_pixels)
        rh = int(math.floor(h / beta / ff)) * factor
        rw = int(math.floor(w / beta / ff)) * factor
    elif rh * rw < config.min_pixels:
        beta = math.sqrt(config.min_pixels / float(h * w))
        rh = int(math.ceil(h * beta / ff)) * factor
        rw = int(math.ceil(w * beta / ff)) * factor
    if rh == 0 or rw == 0:
        raise PreprocessError(INVALID_IMAGE_GEOMETRY, "resized to nothing")
    return rh, rw


def _bicubic_filter(x: np.ndarray) -> np.ndarray:
    # crates/pvlc-cpu-ref/src/lib.rs:3198-3208 (a = -0.5)
    a = -0.5
    x = np.abs(x)
    near = ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0
    far = (((x - 5.0) * x + 8.0) * x - 4.0) * a
    return np.where(x < 1.0, near, np.where(x < 2.0, far, 0.0))


def bicubic_coefficients(input_size: int, output_size: int):
    """crates/pvlc-cpu-ref/src/lib.rs:3141-3196 -> (kernel_size, first [out], count [out],
    weights int32 [out, kernel_size]); weights beyond `count` are zero."""
    scale = input_size / output_size
    filter_scale = max(scale, 1.0)
    support = 2.0 * filter_scale
    ksize = int(math.ceil(support)) * 2 + 1
    inv = 1.0 / filter_scale
    centers = (np.arange(output_size, dtype=np.float64) + 0.5) * scale
    lo = np.maximum(np.trunc(centers - support + 0.5), 0).astype(np.int64)
    hi = np.minimum(np.trunc(centers + support + 0.5), input_size).astype(np.int64)
    count = np.maximum(hi - lo, 0)
    offs = np.arange(ksize, dtype=np.float64)
    dist = (offs[None, :] + lo[:, None].astype(np.float64) - centers[:, None] + 0.5) * inv
    w = _bicubic_filter(dist)
    w = np.where(offs[None, :] < count[:, None], w, 0.0)
    total = np.zeros(output_size, dtype=np.float64)
    for j in range(ksize):              # left-to-right sum, as the reference loop
        total = total + w[:, j]
    w = np.where(total[:, None] != 0.0, w / np.where(total == 0.0, 1.0, total)[:, None], w)
    scaled = w * float(1 << 22)
    fixed = np.where(w < 0.0, np.trunc(-0.5 + scaled), np.trunc(0.5 + scaled)).astype(np.int32)
    return ksize, lo.astype(np.int32), count.astype(np.int32), fixed


def _resample_axis(img: np.ndarray, axis: int, coeffs) -> np.ndarray:
    ksize, lo, count, w = coeffs
    n_in = img.shape[axis]
    idx = lo[:, None] + np.arange(ksize)[None, :]
    idx = np.minimum(idx, n_in - 1)            # padded taps carry weight 0
    src = np.take(img.astype(np.int64), idx, axis=axis)   # axis expands to (out, k)
    wshape = [1] * src.ndim
    wshape[axis], wshape[axis + 1] = w.shape
    acc = (1 << 21) + (src * w.astype(np.int64).reshape(wshape)).sum(axis=axis + 1)
    return np.clip(acc >> 22, 0, 255).astype(np.uint8)


def pillow_bicubic_rgb8(rgb: np.ndarray, out_h: int, out_w: int) -> np.ndarray:
    """crates/pvlc-cpu-ref/src/lib.rs:3092-3139: [H, W, 3] uint8 -> [out_h, out_w, 3] uint8."""
    h, w = rgb.shape[:2]
    if (h, w) == (out_h, out_w):
        return rgb.copy()
    out = rgb
    if w != out_w:
        out = _resample_axis(out, 1, bicubic_coefficients(w, out_w))
    if h != out_h:
        out = _resample_axis(out, 0, bicubic_coefficients(h, out_h))
    return out


@dataclass
class PreprocessedVisionInput:
    resized_height: int
    resized_width: int
    image_grid_thw: tuple
    values: np.ndarray              # [patches, 3 * patch * patch] f32


def patchify(resized: np.ndarray, patch: int) -> np.ndarray:
    """Normalised patch-major values of a resized [H, W, 3] uint8 image (:2534-2553)."""
    gh, gw = resized.shape[0] // patch, resized.shape[1] // patch
    r = (resized.astype(np.float64) / 255.0).astype(np.float32)
    v = (r - np.float32(0.5)) / np.float32(0.5)
    v = v.reshape(gh, patch, gw, patch, 3).transpose(0, 2, 4, 1, 3)
    return np.ascontiguousarray(v.reshape(gh * gw, 3 * patch * patch))


def canonical_rgb8_to_patches(rgb: np.ndarray, config: VisionPreprocessConfig = MODEL_CONFIG):
    """crates/pvlc-cpu-ref/src/lib.rs:2515-2563 on an [H, W, 3] uint8 image."""
    _validate(config)
    rgb = np.asarray(rgb)
    if rgb.dtype != np.uint8 or rgb.ndim != 3 or rgb.shape[2] != 3:
        raise PreprocessError(DIMENSION_MISMATCH, "expected an [H, W, 3] uint8 image")
    rh, rw = smart_resize(rgb.shape[0], rgb.shape[1], config)
    resized = pillow_bicubic_rgb8(rgb, rh, rw)
    p = config.patch_size
    return PreprocessedVisionInput(rh, rw, (1, rh // p, rw // p), patchify(resized, p))
