"""End to end: the reference engine with the B200 paged-KV path dropped in
(its paged_transformer.cu replaced by vllm_b200/csrc/integration/
paged_transformer_tvp.cu) against the unmodified engine, on the e2e workload:
Llama-3.2-1B geometry with seeded N(0, 0.02) weights, 4 requests x 128 prompt
tokens, 128 greedy tokens each, the reference's own scheduler.

Greedy identity.  The reference rounds its logits to BF16 before the argmax
(src/model/argmax.cu:24) and keeps the lowest index on ties.  With
random-init weights the top two logits of a 128,256-entry row are within a
few BF16 ulps of each other at about one step in ten, and often equal after
rounding.  Any change in the FP32 summation order anywhere in the step moves
the logits by a few FP32 ulps and can flip such a tie.  The reference's
attention sums its dot products inside cuBLAS GEMVs, in an order cuBLAS does
not specify; this path sums them in its own order (COMPAT keeps every other
rounding point of the reference).  So the sequences cannot be pinned to
identity.  What is checked instead, per mode:

  * free-running sequences are identical to the reference's up to exactly the
    step where the teacher-forced argmax first differs (both runs decode the
    same inputs until then);
  * every teacher-forced disagreement is a near-tie in the reference's own
    BF16-rounded logits (gap in BF16 ulps, 0 = an exact tie after rounding);
  * the teacher-forced agreement is at least what the path achieves on this
    workload (measured on a B200: compat 0.949, fast and batched 0.911,
    native 0.907; free-running divergence of compat at tokens 58, 9, 8, 57).
"""
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu

# teacher-forced agreement floors and widest allowed gap (BF16 ulps of the
# reference's top logit), just under what the path measures on this workload
FLOORS = {"compat": (0.94, 3.0), "fast": (0.90, 4.0), "batched": (0.90, 4.0),
          "native": (0.90, 4.0)}


@pytest.fixture(scope="module")
def summary():
    for name in ("ref", "tvp"):
        if not (ROOT / "oracle" / "_ref" / f"libtvp_e2e_{name}.so").exists():
            pytest.skip("end-to-end engines not built (make -C oracle e2e)")
    import e2e_compare
    s = e2e_compare.compare()
    print("e2e identity summary:", json.dumps(
        {m: {k: s[m][k] for k in ("argmax_agreement", "disagreements",
                                   "free_running_first_divergence")}
         for m in FLOORS}))
    return s


def test_reference_engine_is_deterministic_under_teacher_forcing(summary):
    assert summary["reference_free_running_matches_teacher_forced"]


@pytest.mark.parametrize("mode", sorted(FLOORS))
def test_free_running_sequences_match_until_the_first_near_tie(summary, mode):
    """A free-running sequence equals the reference's token for token up to
    the first teacher-forced disagreement, and that disagreement is a near-tie."""
    s = summary[mode]
    assert s["free_running_first_divergence"] == s["teacher_forced_first_disagreement"]
    floor, max_gap = FLOORS[mode]
    assert max(s["gap_at_disagreement_bf16_ulps"], default=0.0) <= max_gap


@pytest.mark.parametrize("mode", sorted(FLOORS))
def test_dropped_in_path_matches_reference_up_to_bf16_ties(summary, mode):
    """batched: fast's attention and prefill, plus the decode projections and
    LM head as one GEMM over the batch, the greedy tokens from one batched
    argmax launch, and the step replayed as a CUDA graph.  native: batched
    with the projections and the LM head on tvp_decode_projections."""
    s = summary[mode]
    if mode == "compat":
        assert s["first_tokens_match"]      # prefill: RoPE + pages bit-exact, reference attention
    else:
        # FAST prefill uses the paged prefill kernel: a first token may differ
        # only at a near-tie of the reference's own prefill logits
        assert max(s["first_token_gap_bf16_ulps"], default=0.0) <= 8.0
    floor, max_gap = FLOORS[mode]
    assert s["argmax_agreement"] >= floor
    assert max(s["gap_at_disagreement_bf16_ulps"], default=0.0) <= max_gap
    assert s["max_abs_logit_diff"] <= 0.05 * s["max_abs_reference_logit"]
