"""End-to-end greedy OCR on the GPU engine vs the CPU oracle (BASELINE configs[4] shapes).

The engine (pvlc_b200.model.OcrEngine) runs the full PaddleOCR-VL architecture
with random-init fp16 weights: image -> patches on the device -> 27-layer vision
encoder (this library's varlen attention) -> projector -> 18-layer decoder
prefill (this library's causal prefill, KV cache written in place) -> batched
greedy decode (this library's split-KV decode in a CUDA graph).  The oracle
(oracle/pvlc_model_oracle.cpp) composes the reference's f32 CPU functions over
the same fp16 weights and patches.

Tolerances (the north star's): generated tokens identical; logits within 1e-2
relative error (max |gpu - cpu| / max |cpu| per step).  The tokens are held to
two oracle runs: the plain f32 composition of the reference, and the same
composition rounded to fp16 at the engine's storage points (which also bounds the
logits of every step).
"""
import numpy as np
import pytest
import torch

import pvlc_oracle as O
from pvlc_b200 import model as M
from pvlc_b200 import ops, preprocess as P

pytestmark = pytest.mark.gpu

MAX_NEW = 20


def _formula_image(h, w):
    y, x = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
    rgb = np.empty((h, w, 3), np.uint8)
    rgb[..., 0] = (x * 17 + y * 3) % 256
    rgb[..., 1] = (x * 5 + y * 29 + 7) % 256
    rgb[..., 2] = (x * 11 + y * 13 + 19) % 256
    return rgb


@pytest.mark.parametrize("shape,cfg", [
    ((1024, 1024), P.MODEL_CONFIG),                                  # configs[4] page
    ((29, 31), P.MODEL_CONFIG),                                      # upscale (digest case)
    ((29, 31), P.VisionPreprocessConfig(min_pixels=784, max_pixels=784)),   # downscale
    ((28, 56), P.VisionPreprocessConfig(min_pixels=1568, max_pixels=1568)),  # identity
])
def test_image_patch_kernel_is_bit_exact(cuda_lib, shape, cfg):
    rng = np.random.default_rng(11)
    if shape == (29, 31):
        rgb = _formula_image(*shape)
    else:
        rgb = rng.integers(0, 256, (*shape, 3), dtype=np.uint8)
    ref = P.canonical_rgb8_to_patches(rgb, cfg)
    dev = torch.from_numpy(rgb).cuda()
    got = ops.image_patches(dev, ref.resized_height, ref.resized_width, cfg.patch_size)
    torch.cuda.synchronize()
    assert np.array_equal(got.cpu().numpy().view(np.uint32), ref.values.view(np.uint32))


@pytest.fixture(scope="module")
def engine_and_weights(cuda_lib):
    cfg = M.ModelConfig()
    w = M.init_weights(cfg, seed=0, device="cuda")
    eng = M.OcrEngine(cfg, w)
    host = [[t.cpu().numpy() for t in part] for part in (w.vision, w.projector, w.decoder)]
    return cfg, eng, host


def _requests():
    """Two pages of seeded noise with small patch grids (8x8 and 8x12), so that the
    CPU oracle finishes each request in seconds."""
    rng = np.random.default_rng(5)
    out = []
    for h, w in [(112, 112), (112, 168)]:
        rgb = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
        cfg = P.VisionPreprocessConfig(min_pixels=h * w, max_pixels=h * w)
        pre = P.canonical_rgb8_to_patches(rgb, cfg)
        out.append((rgb, pre))
    return out


def test_e2e_greedy_matches_oracle(engine_and_weights):
    cfg, eng, (vw, pw, dw) = engine_and_weights
    reqs = _requests()
    patches, grids = [], []
    for rgb, pre in reqs:
        dev = torch.from_numpy(rgb).cuda()
        patches.append(ops.image_patches(dev, pre.resized_height, pre.resized_width))
        grids.append(pre.image_grid_thw)
    res = eng.generate(patches, grids, MAX_NEW, chunk=8, record_logits=True)
    # the serving path: greedy top-1 straight from the LM head (pvlc_lm_head_top1)
    fused = eng.generate(patches, grids, MAX_NEW, chunk=8, record_logits=False)
    dims = cfg.oracle_dims()
    report = []
    for b, (rgb, pre) in enumerate(reqs):
        g = pre.image_grid_thw
        ids = M.ocr_prompt_ids(g[0] * g[1] * g[2] // 4, cfg)
        ref = O.generate(dims, vw, pw, dw, pre.values, [g], ids, MAX_NEW, fp16_storage=True,
                         want_logits=True)
        got_logits = res["logits"][b].numpy()
        assert res["tokens"][b] == ref["tokens"], (b, res["tokens"][b], ref["tokens"])
        errs, margins = [], []
        for s in range(len(ref["tokens"])):
            r = ref["logits"][s]
            errs.append(float(np.abs(got_logits[s] - r).max() / np.abs(r).max()))
            top2 = np.sort(r)[-2:]
            margins.append(float(top2[1] - top2[0]))
        assert max(errs) <= 1e-2, (b, errs)
        # the plain f32 reference composition
        f32 = O.generate(dims, vw, pw, dw, pre.values, [g], ids, MAX_NEW, fp16_storage=False,
                         want_logits=True)
        r0 = f32["logits"][0]
        err0 = float(np.abs(got_logits[0] - r0).max() / np.abs(r0).max())
        assert err0 <= 1e-2, err0
        # the north star's rule: the same tokens as the plain f32 reference, every step
        assert res["tokens"][b] == f32["tokens"], (b, res["tokens"][b], f32["tokens"])
        assert list(fused["tokens"][b]) == f32["tokens"], (b, fused["tokens"][b])
        same = len(f32["tokens"])
        report.append(dict(request=b, tokens=len(ref["tokens"]), max_rel_logit_err=max(errs),
                           min_margin=min(margins), f32_prefill_rel_err=err0,
                           f32_tokens_agree=same))
    print("e2e parity:", report)


def test_e2e_config4_page_matches_f32_oracle(engine_and_weights):
    """One configs[4] request at full size: a 1024x1024 seeded-noise page -> 980x980 ->
    4900 patches -> 1225 image tokens in a 1238-token prompt, through the 27-layer
    encoder, the projector and the 18-layer decoder, then greedy tokens.  The tokens
    must equal the plain f32 reference composition's; the prefill logits must be
    within 1e-2 relative of it."""
    cfg, eng, (vw, pw, dw) = engine_and_weights
    steps = 4
    rng = np.random.default_rng(4)
    rgb = rng.integers(0, 256, (1024, 1024, 3), dtype=np.uint8)
    pre = P.canonical_rgb8_to_patches(rgb, P.MODEL_CONFIG)
    g = pre.image_grid_thw
    assert tuple(g) == (1, 70, 70)
    patches = ops.image_patches(torch.from_numpy(rgb).cuda(), pre.resized_height,
                                pre.resized_width)
    res = eng.generate([patches], [g], steps, chunk=steps, record_logits=True)
    fused = eng.generate([patches], [g], steps, chunk=steps, record_logits=False)
    ids = M.ocr_prompt_ids(g[0] * g[1] * g[2] // 4, cfg)
    assert len(ids) == 1238
    f32 = O.generate(cfg.oracle_dims(), vw, pw, dw, pre.values, [g], ids, steps,
                     fp16_storage=False, want_logits=True)
    got0, r0 = res["logits"][0].numpy()[0], f32["logits"][0]
    rel0 = float(np.abs(got0 - r0).max() / np.abs(r0).max())
    top2 = np.sort(r0)[-2:]
    print("configs[4] page:", dict(tokens=res["tokens"][0], f32_tokens=f32["tokens"],
                                   prefill_rel_err=rel0, top1_margin=float(top2[1] - top2[0])))
    assert rel0 <= 1e-2, rel0
    assert res["tokens"][0] == f32["tokens"], (res["tokens"][0], f32["tokens"])
    assert list(fused["tokens"][0]) == f32["tokens"], (fused["tokens"][0], f32["tokens"])
