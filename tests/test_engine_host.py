"""Host-side helpers of the end-to-end engine (no GPU needed)."""
import numpy as np
import torch

from pvlc_b200 import model as M


def test_join_rows_is_a_view_for_consecutive_blocks_else_a_copy():
    a = torch.arange(60.0).reshape(20, 3)
    blocks = [a[0:5], a[5:12], a[12:20]]
    j = M._join_rows(blocks)
    assert torch.equal(j, a) and j.data_ptr() == a.data_ptr()
    gap = [a[0:5], a[6:12]]                       # not adjacent
    assert torch.equal(M._join_rows(gap), torch.cat(gap))
    other = [a[0:2], torch.zeros(4, 3)]           # different buffers
    assert torch.equal(M._join_rows(other), torch.cat(other))
    assert M._join_rows([a[3:7]]).data_ptr() == a[3:7].data_ptr()


def test_prompt_ids_hold_one_placeholder_per_merged_patch():
    cfg = M.ModelConfig()
    ids = M.ocr_prompt_ids(1225, cfg)
    assert sum(1 for t in ids if t == cfg.image_token_id) == 1225
    assert len(ids) == 1238
    assert np.asarray(ids).dtype.kind == "i"


def test_gate_up_blocks_layout():
    """The fused SiLU-gate projection's weight: 128-row blocks of 64 gate rows followed by
    the 64 up rows of the same output columns (pvlc_linear with gate = 1)."""
    from pvlc_b200 import ops
    i, k = 192, 8
    g = torch.arange(i * k, dtype=torch.float32).reshape(i, k)
    u = -torch.arange(i * k, dtype=torch.float32).reshape(i, k) - 1
    w = ops.gate_up_blocks(g, u)
    assert w.shape == (2 * i, k) and w.is_contiguous()
    for blk in range(i // 64):
        assert torch.equal(w[128 * blk:128 * blk + 64], g[64 * blk:64 * blk + 64])
        assert torch.equal(w[128 * blk + 64:128 * blk + 128], u[64 * blk:64 * blk + 64])
    import pytest
    with pytest.raises(ValueError):
        ops.gate_up_blocks(g[:100], u[:100])
    with pytest.raises(ValueError):
        ops.gate_up_blocks(g, u[:64])
