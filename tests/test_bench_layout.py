"""bench.py's dp x tp rank layout (host logic, no GPU)."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_auto_layout_is_pure_data_parallel_when_the_batch_divides():
    for world in (1, 2, 4, 8):
        seen = []
        for rank in range(world):
            tp, dp, groups, (a, b) = bench.dp_tp_layout(world, rank, 8)
            assert (tp, dp) == (1, world) and groups == [[r] for r in range(world)]
            seen.extend(range(a, b))
        assert seen == list(range(8))                    # every sequence exactly once


def test_tensor_parallel_groups_share_sequences():
    layouts = [bench.dp_tp_layout(8, r, 8, tp=2) for r in range(8)]
    assert all(l[:3] == (2, 4, [[0, 1], [2, 3], [4, 5], [6, 7]]) for l in layouts)
    assert [l[3] for l in layouts] == [(0, 2), (0, 2), (2, 4), (2, 4), (4, 6), (4, 6), (6, 8), (6, 8)]
    assert bench.dp_tp_layout(3, 1, 8)[:2] == (3, 1)         # 8 sequences do not split over 3 ranks: all shard


def test_invalid_layout_is_rejected():
    with pytest.raises(SystemExit):
        bench.dp_tp_layout(8, 0, 8, tp=3)
