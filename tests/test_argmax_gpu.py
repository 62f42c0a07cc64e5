"""tvp_greedy_argmax on the GPU against the oracle (the reference engine's
selection rule, src/model/argmax.cu:16-45): the reference's own known-answer
rows in one launch, rows with many BF16 ties, strided rows, short
vocabularies, and repeated calls on one workspace.  Token ids must be
identical."""
import numpy as np
import pytest
import torch

import oracle
from test_argmax import VOCAB, known_answer_cases
from vllm_b200 import _native as N
from vllm_b200 import ops

pytestmark = pytest.mark.gpu


def run(host, stride=None, workspace=None):
    rows, vocab = host.shape
    stride = stride or vocab
    buf = torch.full((rows, stride), float("nan"), dtype=torch.float32, device="cuda")
    buf[:, :vocab] = torch.from_numpy(host).cuda()
    out = ops.greedy_argmax(buf[:, :vocab], workspace=workspace)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_reference_known_answers_in_one_launch():
    cases = known_answer_cases()
    logits = np.stack([c for c, _ in cases])
    want = np.array([t for _, t in cases], np.int32)
    assert np.array_equal(oracle.greedy_argmax(logits), want)
    assert np.array_equal(run(logits), want)


def test_random_bit_patterns():
    rng = np.random.default_rng(20261015)
    x = rng.integers(0, 2**32, size=(8, VOCAB), dtype=np.uint64).astype(np.uint32).view(np.float32)
    assert np.array_equal(run(x), oracle.greedy_argmax(x))


def test_many_bf16_ties_and_strided_rows():
    rng = np.random.default_rng(5)
    # logits on a coarse grid: the maximum is shared by many tokens per row
    x = (rng.integers(-40, 41, size=(64, VOCAB)) / 8.0).astype(np.float32)
    x += rng.uniform(-1e-3, 1e-3, size=x.shape).astype(np.float32)  # below BF16 resolution at 5
    assert np.array_equal(run(x, stride=VOCAB + 96), oracle.greedy_argmax(x))


@pytest.mark.parametrize("vocab", [1, 5, 31, 32, 33, 257, 4097])
def test_short_vocabularies(vocab):
    rng = np.random.default_rng(vocab)
    x = rng.normal(size=(3, vocab)).astype(np.float32)
    x[1, :] = x[1, 0]  # all tied
    assert np.array_equal(run(x), oracle.greedy_argmax(x))


def test_workspace_is_reusable():
    rng = np.random.default_rng(9)
    lib = N.load()
    ws = torch.zeros(lib.tvp_greedy_argmax_workspace_bytes(4), dtype=torch.uint8, device="cuda")
    for _ in range(5):
        x = rng.normal(size=(4, VOCAB)).astype(np.float32)
        assert np.array_equal(run(x, workspace=ws), oracle.greedy_argmax(x))
    counters = ws[-4 * 4:].view(torch.int32)  # the per-row counters end the workspace
    assert int(counters.abs().sum()) == 0


def test_workspace_serves_calls_of_any_row_count():
    """A decode loop's batch shrinks and grows as requests finish and slots
    refill; one workspace sized for the largest batch serves every call.  Rows
    4, then 1, 3, 2, 4, 1: each call's tokens are the oracle's."""
    rng = np.random.default_rng(19)
    lib = N.load()
    ws = torch.zeros(lib.tvp_greedy_argmax_workspace_bytes(4), dtype=torch.uint8, device="cuda")
    for rows in (4, 1, 3, 2, 4, 1):
        x = rng.normal(size=(rows, VOCAB)).astype(np.float32)
        assert np.array_equal(run(x, workspace=ws), oracle.greedy_argmax(x)), rows
    counters = ws[-4 * 4:].view(torch.int32)
    assert int(counters.abs().sum()) == 0
