"""Decoder causal-GQA prefill parity: CUDA kernel (C ABI) vs the CPU oracle.

Oracle: apply_multimodal_rope_f32 -> write_decoder_prefill_kv_f32 ->
causal_gqa_f32 (crates/pvlc-cpu-ref/src/lib.rs:562-672,976-991,782-853) with
M-RoPE positions from mrope_position_ids (multimodal.rs:28-78) and the
reference host's ropeTables (web/engine/multimodal_ocr.mjs:937-986).
Tolerance: max-abs <= 2e-3 on fp16 outputs; the fp16 cache rows match the
oracle's f32 rows within fp16 rounding.
"""
import numpy as np
import pytest
import torch

import pvlc_oracle as O

pytestmark = pytest.mark.gpu
QH, KVH, HD = 16, 2, 128
ATOL = 2e-3


def image_prompt(prefix_text, grid_hw_merged, suffix_text):
    """Token ids: text ... vision_start, image run, text ...; grid in merged tokens."""
    h, w = grid_hw_merged
    ids = [7] * (prefix_text - 1) + [101305] + [100295] * (h * w) + [9] * suffix_text
    return ids, [(1, 2 * h, 2 * w)]


def _run_case(ids, grids, capacity, seed):
    from pvlc_b200 import ops, positions
    T = len(ids)
    pos, delta = positions.mrope_position_ids(ids, grids)
    opos, odelta = O.mrope_position_ids(ids, grids)
    np.testing.assert_array_equal(pos, opos)
    assert delta == odelta
    cos, sin = positions.mrope_tables(pos, delta, capacity)
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, QH, HD)).astype(np.float16)
    k = rng.standard_normal((T, KVH, HD)).astype(np.float16)
    v = rng.standard_normal((T, KVH, HD)).astype(np.float16)
    kc_o = np.zeros((capacity, KVH, HD), np.float32)
    vc_o = np.zeros((capacity, KVH, HD), np.float32)
    ref = O.decoder_prefill(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), cos,
                            sin, T, kc_o, vc_o)
    dev = torch.device("cuda")
    kc = torch.full((capacity, KVH, HD), float("nan"), dtype=torch.float16, device=dev)
    vc = torch.full((capacity, KVH, HD), float("nan"), dtype=torch.float16, device=dev)
    out = ops.decoder_prefill(torch.from_numpy(q).to(dev), torch.from_numpy(k).to(dev),
                              torch.from_numpy(v).to(dev), torch.from_numpy(cos).to(dev),
                              torch.from_numpy(sin).to(dev), kc, vc)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err <= ATOL, f"T={T} max abs err {err}"
    kcg = kc.float().cpu().numpy()
    vcg = vc.float().cpu().numpy()
    np.testing.assert_allclose(kcg[:T], kc_o[:T], atol=2e-3, rtol=1e-3)
    np.testing.assert_array_equal(vcg[:T], vc_o[:T])
    assert np.isnan(kcg[T:]).all(), "rows past the prompt must not be written"


@pytest.mark.parametrize("T", [1, 5, 63, 64, 65, 200])
def test_text_only_prefill(cuda_lib, T):
    _run_case(list(range(3, 3 + T)), [], T + 3, seed=T)


@pytest.mark.parametrize("pre,grid,post", [(5, (4, 6), 7), (20, (10, 9), 64), (2, (16, 16), 1)])
def test_image_prompt_prefill(cuda_lib, pre, grid, post):
    ids, grids = image_prompt(pre, grid, post)
    _run_case(ids, grids, len(ids) + 16, seed=pre)


def test_config3_prefill(cuda_lib):
    """20 text + 40x37 image tokens + 64 text = 1564 positions."""
    ids, grids = image_prompt(20, (40, 37), 64)
    assert len(ids) == 1564
    _run_case(ids, grids, 1564 + 256, seed=3)


@pytest.mark.parametrize("T", [1190, 2500, 4100])
def test_long_prefill_paired_tiles(cuda_lib, T):
    """Past 74 Q tiles per KV head the lightest tiles run two per CTA (one per
    stream, sharing K/V tiles): one pair (1190), many pairs (2500), and every
    tile paired with more CTAs than SMs (4100)."""
    _run_case(list(range(3, 3 + T)), [], T + 5, seed=T)
