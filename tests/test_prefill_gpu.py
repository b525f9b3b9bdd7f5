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


def _run_case(ids, grids, capacity, seed, plant=None, fp16_rotated=False):
    from pvlc_b200 import ops, positions
    T = len(ids)
    pos, delta = positions.mrope_position_ids(ids, grids)
    opos, odelta = O.mrope_position_ids(ids, grids)
    np.testing.assert_array_equal(pos, opos)
    assert delta == odelta
    cos, sin = positions.mrope_tables(pos, delta, capacity)
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, QH, HD)).astype(np.float32)
    k = rng.standard_normal((T, KVH, HD)).astype(np.float32)
    v = rng.standard_normal((T, KVH, HD)).astype(np.float16)
    if plant is not None:
        plant(q, k)
    q, k = q.astype(np.float16), k.astype(np.float16)
    kc_o = np.zeros((capacity, KVH, HD), np.float32)
    vc_o = np.zeros((capacity, KVH, HD), np.float32)
    ref = O.decoder_prefill(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), cos,
                            sin, T, kc_o, vc_o)
    if fp16_rotated:
        # attention over the rotated q and k rounded to fp16, as the fp16 KV cache (and the
        # staged Q tile) hold them: the reference composition with that storage point
        kc_o[:T] = kc_o[:T].astype(np.float16).astype(np.float32)
        qr, _ = O.apply_multimodal_rope(q.astype(np.float32), k.astype(np.float32), T, QH, KVH,
                                        HD, np.ascontiguousarray(cos[:, :T]),
                                        np.ascontiguousarray(sin[:, :T]))
        qr = qr.astype(np.float16).astype(np.float32)
        ref = O.causal_gqa(qr, kc_o[:T].copy(), v.astype(np.float32), T, QH, KVH, HD)
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


@pytest.mark.parametrize("T", [1190, 1600, 1800, 2500, 4100])
def test_long_prefill_schedules(cuda_lib, T):
    """Past 74 Q tiles per KV head: one pair of light tiles (1190), the most pairs
    that keep one wave (1600, 52 light tiles), and split CTAs only, in several waves
    heaviest first, where pairing would outlast the heaviest CTA (1800, 2500, 4100)."""
    _run_case(list(range(3, 3 + T)), [], T + 5, seed=T)


def test_lazy_rescale_branch(cuda_lib):
    """Scores that rise along the keys and jump by more than the kernel's lazy rescale
    threshold (8 log2 units) twice, at 45 % and 85 % of the prompt, so queries past
    each jump rescale O in the middle of their key range; query heads alternate the
    sign of the planted component, so half of them meet their max in the first K
    tile.  The planted component is dim 63 (partner 127), the M-RoPE's lowest
    frequency (500000^(-126/128) ~ 2.5e-6 rad a position), so it survives rotation.
    Planted scores of ~14 nats make the fp16 rounding of the rotated q and k (the fp16
    cache's storage point) worth ~1e-2 nats a score, so the reference here attends over
    the rotated operands rounded to fp16: the test isolates the rescale logic."""
    T = 1800
    sign = np.where(np.arange(QH) % 2 == 0, 1.0, -1.0).astype(np.float32)

    def plant(q, k):
        q *= 0.25
        k *= 0.25
        q[:, :, 63] = (8.0 * sign)[None, :]
        k[:, :, 63] = np.linspace(-2.0, 6.0, T, dtype=np.float32)[:, None]
        k[int(0.45 * T):int(0.45 * T) + 32, :, 63] = 10.0
        k[int(0.85 * T):int(0.85 * T) + 64, :, 63] = 20.0

    per_unit = 8.0 / np.sqrt(128.0) * np.log2(np.e)
    assert (10.0 - (-2.0)) * per_unit > 8.0 and (20.0 - 10.0) * per_unit > 8.0
    _run_case(list(range(3, 3 + T)), [], T + 4, seed=17, plant=plant, fp16_rotated=True)


def test_packed_prompts_match_single_calls(cuda_lib):
    """ops.decoder_prefill_packed (the engine's path: prompts back to back, one cache
    slab per prompt, adjacent Q tiles paired in a CTA) gives the per-prompt
    decoder_prefill results within the fp16 output tolerance and the same caches bit for
    bit."""
    from pvlc_b200 import ops, positions
    dev = torch.device("cuda")
    prompts = [image_prompt(3, (4, 5), 6), image_prompt(20, (12, 10), 40), image_prompt(1, (2, 2), 1)]
    Ts = [len(ids) for ids, _ in prompts]
    offs = np.concatenate([[0], np.cumsum(Ts)])
    NT, cap = int(offs[-1]), max(Ts) + 8
    rng = np.random.default_rng(11)
    q = torch.from_numpy(rng.standard_normal((NT, QH, HD)).astype(np.float16)).to(dev)
    k = torch.from_numpy(rng.standard_normal((NT, KVH, HD)).astype(np.float16)).to(dev)
    v = torch.from_numpy(rng.standard_normal((NT, KVH, HD)).astype(np.float16)).to(dev)
    tables = []
    for ids, grids in prompts:
        pos, delta = positions.mrope_position_ids(ids, grids)
        c, s_ = positions.mrope_tables(pos, delta, cap)
        tables.append((torch.from_numpy(c).to(dev), torch.from_numpy(s_).to(dev)))
    kc = torch.zeros((len(prompts), cap, KVH, HD), dtype=torch.float16, device=dev)
    vc = torch.zeros_like(kc)
    out = torch.empty_like(q)
    ops.decoder_prefill_packed(q, k, v, offs, tables, kc, vc, out)
    for b in range(len(prompts)):
        s, e = int(offs[b]), int(offs[b + 1])
        kc1 = torch.zeros((cap, KVH, HD), dtype=torch.float16, device=dev)
        vc1 = torch.zeros_like(kc1)
        ref = ops.decoder_prefill(q[s:e].contiguous(), k[s:e].contiguous(), v[s:e].contiguous(),
                                  tables[b][0], tables[b][1], kc1, vc1)
        assert (out[s:e].float() - ref.float()).abs().max().item() <= ATOL
        assert torch.equal(kc[b], kc1) and torch.equal(vc[b], vc1)
    with pytest.raises(ValueError):
        ops.decoder_prefill_packed(q, k, v, offs[:-1], tables, kc, vc, out)


def _packed_case(Ts, cap, seed):
    from pvlc_b200 import positions
    dev = torch.device("cuda")
    offs = np.concatenate([[0], np.cumsum(Ts)]).astype(np.int64)
    NT = int(offs[-1])
    rng = np.random.default_rng(seed)
    host = dict(q=rng.standard_normal((NT, QH, HD)).astype(np.float16),
                k=rng.standard_normal((NT, KVH, HD)).astype(np.float16),
                v=rng.standard_normal((NT, KVH, HD)).astype(np.float16))
    tables, host_tables = [], []
    for b, T in enumerate(Ts):
        ids = list(range(3 + b, 3 + b + T))
        pos, delta = positions.mrope_position_ids(ids, [])
        c, s_ = positions.mrope_tables(pos, delta, cap)
        host_tables.append((c, s_))
        tables.append((torch.from_numpy(c).to(dev), torch.from_numpy(s_).to(dev)))
    t = {n: torch.from_numpy(a).to(dev) for n, a in host.items()}
    kc = torch.full((len(Ts), cap, KVH, HD), float("nan"), dtype=torch.float16, device=dev)
    vc = torch.full_like(kc, float("nan"))
    return offs, host, host_tables, t, tables, kc, vc


def test_batched_prefill_long_and_short_prompts_vs_oracle(cuda_lib):
    """One batched launch over a configs[2]-length prompt (1564 tokens: 98 Q tiles, paired
    adjacent here, heaviest split in the single call), a short one and a 1190-token one:
    each prompt's output within tolerance of the oracle, caches written only up to its
    length (the NaN tails stay untouched)."""
    from pvlc_b200 import ops
    Ts = [1564, 40, 1190]
    cap = 1600
    offs, host, host_tables, t, tables, kc, vc = _packed_case(Ts, cap, seed=17)
    out = torch.empty_like(t["q"])
    ops.decoder_prefill_packed(t["q"], t["k"], t["v"], offs, tables, kc, vc, out)
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    for b, T in enumerate(Ts):
        s, e = int(offs[b]), int(offs[b + 1])
        kc_o = np.zeros((cap, KVH, HD), np.float32)
        vc_o = np.zeros((cap, KVH, HD), np.float32)
        ref = O.decoder_prefill(host["q"][s:e].astype(np.float32), host["k"][s:e].astype(np.float32),
                                host["v"][s:e].astype(np.float32), host_tables[b][0],
                                host_tables[b][1], T, kc_o, vc_o)
        err = np.abs(got[s:e] - ref).max()
        assert err <= ATOL, f"prompt {b} (T={T}) max abs err {err}"
        kcg = kc[b].float().cpu().numpy()
        np.testing.assert_allclose(kcg[:T], kc_o[:T], atol=2e-3, rtol=1e-3)
        assert np.isnan(kcg[T:]).all()


def test_batched_prefill_many_prompts_in_groups(cuda_lib):
    """300 short prompts (two launches of at most 256 prompts, odd and even Q-tile counts)
    match the per-prompt calls, every prompt: outputs within the fp16 tolerance, caches bit
    for bit (the persistent kernel's work items cross prompt boundaries on every CTA, and an
    odd prompt's last item leaves one stream idle)."""
    from pvlc_b200 import ops
    rng = np.random.default_rng(4)
    Ts = [int(x) for x in rng.integers(1, 300, size=300)]
    cap = 304
    offs, host, host_tables, t, tables, kc, vc = _packed_case(Ts, cap, seed=5)
    out = torch.empty_like(t["q"])
    ops.decoder_prefill_packed(t["q"], t["k"], t["v"], offs, tables, kc, vc, out)
    for b in range(len(Ts)):
        s, e = int(offs[b]), int(offs[b + 1])
        kc1 = torch.full((cap, KVH, HD), float("nan"), dtype=torch.float16, device="cuda")
        vc1 = torch.full_like(kc1, float("nan"))
        ref = ops.decoder_prefill(t["q"][s:e].contiguous(), t["k"][s:e].contiguous(),
                                  t["v"][s:e].contiguous(), tables[b][0], tables[b][1], kc1, vc1)
        assert (out[s:e].float() - ref.float()).abs().max().item() <= ATOL, b
        assert torch.equal(kc[b].nan_to_num(7.0), kc1.nan_to_num(7.0)), b


def test_fault_word_clear_after_clean_calls(cuda_lib):
    """pvlc_attn_fault_flags: after clean vision, single-prompt and batched prefill calls
    the device's sticky fault word of those kernels reads zero (status OK), and a read
    clears it."""
    from pvlc_b200 import ops
    ops.fault_flags()                         # whatever earlier tests left
    dev = torch.device("cuda")
    rng = np.random.default_rng(21)
    T, H, D = 300, 16, 72
    qv = [torch.from_numpy(rng.standard_normal((T, H, D)).astype(np.float16)).to(dev)
          for _ in range(3)]
    ops.vision_varlen_attention(*qv, np.array([0, 100, 300]))
    _run_case(list(range(3, 3 + 200)), [], 208, seed=3)
    Ts = [40, 17]
    offs, host, host_tables, t, tables, kc, vc = _packed_case(Ts, 48, seed=9)
    out = torch.empty_like(t["q"])
    ops.decoder_prefill_packed(t["q"], t["k"], t["v"], offs, tables, kc, vc, out)
    assert ops.fault_flags() == 0
    assert ops.fault_flags() == 0
