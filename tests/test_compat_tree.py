"""Host model of COMPAT's chunked pairwise sum (no GPU).

The reference sums a softmax row with a pairwise tree (src/model/softmax.cu:
35-42): for i = 1, 2, 4, ...: e[t] += e[t + i] where t % 2i == 0 and
t + i < L.  The COMPAT decode kernel holds 4096 tokens of a row at a time; it
runs the same tree inside each aligned 4096-token chunk and then over the
chunk sums.  This checks, in FP32 with numpy, that both give the same bits for
any row length, including lengths just off the chunk boundaries."""
import numpy as np
import pytest


def whole_row_tree(e: np.ndarray) -> np.float32:
    e = e.copy()
    L = e.size
    i = 1
    while i < L:
        t = np.arange(0, L, 2 * i)
        t = t[t + i < L]
        e[t] = e[t] + e[t + i]
        i *= 2
    return e[0]


def chunked_tree(e: np.ndarray, chunk: int) -> np.float32:
    sums = np.array([whole_row_tree(e[b:b + chunk]) for b in range(0, e.size, chunk)],
                    dtype=np.float32)
    return whole_row_tree(sums)


@pytest.mark.parametrize("L", [1, 2, 3, 4095, 4096, 4097, 8191, 8192, 8193, 12289, 20000,
                               32768, 65535, 100003])
def test_chunked_tree_equals_whole_row_tree(L):
    rng = np.random.default_rng(L)
    # expf(s - max) values of BF16 scores: in (0, 1], max at 1
    s = rng.standard_normal(L).astype(np.float32) * 3
    e = np.exp(s - s.max()).astype(np.float32)
    assert chunked_tree(e, 4096).view(np.uint32) == whole_row_tree(e).view(np.uint32)


def test_chunk_size_must_be_a_power_of_two():
    """The split is exact only at aligned power-of-two chunks; a 3000-token
    chunk regroups the additions (shown here, so the model can fail)."""
    rng = np.random.default_rng(1)
    e = np.exp(rng.standard_normal(9000).astype(np.float32)).astype(np.float32)
    diffs = sum(chunked_tree(np.roll(e, k), 3000) != whole_row_tree(np.roll(e, k)) for k in range(8))
    assert diffs > 0
