"""bench.py's request sharding of the decode_sweep workload across N GPUs
(strong scaling): every row lands on exactly one rank, a rank's block
tables address only its own pool, each row's pages are distinct, and the
ranks' attended tokens are balanced."""
import numpy as np
import pytest

import bench
import workloads as W


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_every_row_on_exactly_one_rank_with_its_own_pool(world):
    g = W.decode_sweep(seed=4, batch=256)
    seen = []
    sums = []
    for rank in range(world):
        case, rows = bench.shard_case(g, world, rank)
        assert case.num_layers == g.num_layers
        assert np.array_equal(case.lens, g.lens[rows])
        seen += list(rows)
        sums.append(int(case.lens.astype(np.int64).sum()))
        used = []
        for b, L in enumerate(case.lens):
            n = W.pages_for(int(L))
            pages = case.tables[b, :n]
            assert (pages >= 0).all() and (pages < case.num_pages).all()
            assert (case.tables[b, n:] == -1).all()
            used += list(pages)
        assert len(used) == len(set(used))  # no page shared by two rows
    assert sorted(seen) == list(range(256))
    assert max(sums) / (sum(sums) / world) < 1.01


def test_one_rank_is_the_global_workload():
    g = W.decode_sweep(seed=4, batch=256)
    case, rows = bench.shard_case(g, 1, 0)
    assert case is g and np.array_equal(rows, np.arange(256))
