"""Host model of the decode plan's split-K partition (tvp_decode.cu:
decode_plan_kernel and the page ranges of paged_decode_kernel /
paged_decode_heads_kernel), in exact integer arithmetic.

The plan cuts the step's T pages, laid end to end, into C = min(grid, T)
ranges; CTA c takes pages [floor(c T / C), floor((c + 1) T / C)).  It writes
CTA c's start record {s, cu[s], cu[s + 1]} from sequence s's side, for the c
with ceil(cu[s] C / T) <= c < ceil(cu[s + 1] C / T).  The kernels rely on:
  * every CTA c < C gets exactly one record, and empty sequences write none;
  * the record's sequence holds CTA c's first page;
  * the ranges partition [0, T), every range non-empty;
  * a sequence's pieces are exactly the CTAs its pages span, which is the
    arrival count its last-arriver merge waits for.
No GPU is needed."""
import numpy as np
import pytest


def plan(lens, grid):
    pages = [(int(L) + 15) // 16 for L in lens]
    cu = np.concatenate([[0], np.cumsum(pages)]).astype(np.int64).tolist()
    T = cu[-1]
    C = min(grid, T)
    records = {}
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        for c in range((a * C + T - 1) // T if T else 0, (b * C + T - 1) // T if T else 0):
            assert c not in records, "two sequences wrote one CTA's record"
            records[c] = (s, a, b)
    return cu, T, C, records


def check(lens, grid):
    cu, T, C, records = plan(lens, grid)
    assert sorted(records) == list(range(C))
    covered = []
    for c in range(C):
        lo, hi = c * T // C, (c + 1) * T // C
        assert hi > lo, "a CTA below C without pages"
        s, a, b = records[c]
        assert a <= lo < b, "record's sequence does not hold the CTA's first page"
        covered.extend(range(lo, hi))
    assert covered == list(range(T))
    for s in range(len(lens)):
        a, b = cu[s], cu[s + 1]
        if a == b:
            assert all(r[0] != s for r in records.values())
            continue
        spanning = [c for c in range(C) if c * T // C < b and (c + 1) * T // C > a]
        assert spanning == list(range(spanning[0], spanning[-1] + 1))
        # the first CTA of the sequence's pieces holds page a or starts before it
        assert spanning[0] * T // C <= a


@pytest.mark.parametrize("grid", [1, 2, 7, 148, 296, 1000])
def test_partition_random_lengths(grid):
    rng = np.random.default_rng(grid)
    for _ in range(40):
        n = int(rng.integers(1, 40))
        lens = rng.integers(0, 4000, n)
        lens[rng.random(n) < 0.2] = 0  # empty sequences
        check(lens.tolist(), grid)


@pytest.mark.parametrize("lens", [[1], [16], [17], [0, 0, 5], [32768] * 16, [1] * 300,
                                  [17, 64, 129, 256], [1024] * 4])
@pytest.mark.parametrize("grid", [1, 148, 4096])
def test_partition_edge_cases(lens, grid):
    check(lens, grid)


def test_all_sequences_empty_write_nothing():
    cu, T, C, records = plan([0, 0, 0], 148)
    assert T == 0 and C == 0 and records == {}
