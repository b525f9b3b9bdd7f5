"""Host-side table / position preparation (product numpy code) vs the oracle."""
import numpy as np
import pytest

import pvlc_oracle as O
from pvlc_b200 import positions


@pytest.mark.parametrize("grids", [[(1, 32, 32)], [(1, 4, 6), (1, 3, 3), (2, 2, 5)]])
def test_vision_tables_match_oracle(grids):
    c, s = positions.vision_rope_tables(grids)
    oc, os_ = O.vision_rope_tables(grids)
    np.testing.assert_allclose(c, oc, atol=1e-7, rtol=0)
    np.testing.assert_allclose(s, os_, atol=1e-7, rtol=0)


@pytest.mark.parametrize("ids,grids", [
    ([1, 2, 101305] + [100295] * 6 + [7, 8], [(1, 4, 6)]),
    ([5] * 19 + [101305] + [100295] * 1480 + [9] * 64, [(1, 80, 74)]),
    ([3, 101305] + [100295] * 4 + [4, 101305] + [100295] * 9 + [1], [(1, 4, 4), (1, 6, 6)]),
    (list(range(10, 40)), []),
])
def test_mrope_positions_match_oracle(ids, grids):
    pos, delta = positions.mrope_position_ids(ids, grids)
    opos, odelta = O.mrope_position_ids(ids, grids)
    np.testing.assert_array_equal(pos, opos)
    assert delta == odelta


def test_mrope_positions_reject_malformed_prompts():
    for ids, grids in (([1, 100295, 2], [(1, 2, 2)]),
                       ([101305, 100295, 100295], [(1, 2, 2)]),
                       ([101305] + [100295] * 2, [(1, 2, 4), (1, 2, 2)])):
        with pytest.raises(positions.PositionError):
            positions.mrope_position_ids(ids, grids)
        with pytest.raises(O.OracleError):
            O.mrope_position_ids(ids, grids)


def test_mrope_tables_match_oracle():
    ids = [5] * 19 + [101305] + [100295] * 1480 + [9] * 64
    pos, delta = positions.mrope_position_ids(ids, [(1, 80, 74)])
    c, s = positions.mrope_tables(pos, delta, 1564 + 256)
    oc, os_ = O.rope_tables(pos, delta, 1564 + 256)
    np.testing.assert_allclose(c, oc, atol=1e-7, rtol=0)
    np.testing.assert_allclose(s, os_, atol=1e-7, rtol=0)
    assert positions.decode_position(1564, delta) == O.decode_mrope_position(1564, delta)
