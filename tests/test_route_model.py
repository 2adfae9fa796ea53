"""The decode kernel's routing-table algorithm (a warp bitonic sort plus scans,
modelled in tests/route_model.py) builds exactly the reference's grouping for
every post size the slice accepts, with padding, bad ids and hot experts."""

import numpy as np
import pytest

import route_model as RM


def _ids(rows, rng, hot=False, pad=False, n_experts=384, topk=6):
    ids = np.stack([rng.choice(n_experts, topk, replace=False) for _ in range(rows)]).astype(np.int64)
    if hot:
        ids[:, :3] = rng.integers(0, 4, size=(rows, 3))       # a few experts take many pairs
    if pad:
        ids[rng.random(ids.shape) < 0.15] = -1
        ids[0, 0] = n_experts + 7                             # an id outside [0, E): skipped
    return ids.reshape(-1)


@pytest.mark.parametrize("rows", [1, 2, 3, 6, 10, 11, 16, 21, 42, 48, 64])
def test_sorted_tables_equal_direct_grouping(rows):
    rng = np.random.default_rng(rows)
    for trial in range(6):
        ids = _ids(rows, rng, hot=trial % 2 == 1, pad=trial % 3 == 2)
        for n_tiles in (5, 36):
            assert RM.route_sort(ids, rows, n_tiles, 384) == RM.direct_grouping(ids, rows, n_tiles, 384)


def test_all_padding_gives_no_group():
    ids = np.full(36, -1, dtype=np.int64)
    assert RM.route_sort(ids, 6, 36, 384) == ([], [], 0)
