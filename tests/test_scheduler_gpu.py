"""Continuous batching through the drop-in engine: the reference's own
scheduler (generateContinuous, src/engine/scheduler.cu:17-169) serves more
requests than it has slots, with ragged prompt and output lengths, so the
decode batch shrinks and grows, freed slots are refilled mid-run and freed
pages are handed to the next request.  Mirrors the reference's batch test
(tests/paged_inference_test.cu:149-224) on the e2e model geometry with seeded
random weights:

  * the three first requests are admitted together; every later one takes the
    slot freed in the same iteration; freed pages are reused;
  * every slot ends empty, every finished request holds no page, and the pool
    ends full (24 pages: 3 slots x 128 tokens / 16), or the scheduler's own
    leak check throws;
  * a 0-token request performs no inference; a 1-token request stops after
    prefill;
  * the scheduler's event log (iterations, slots, page ids, free counts) of
    the engine with the path dropped in is identical to the unmodified
    engine's, in every mode: the allocator is the reference's, page for page;
  * compat: every request's tokens under continuous batching equal the same
    request served alone (the reference's own criterion for its batch test):
    no step of its decode math depends on the other rows of the batch;
  * native: the same holds here, where the rows are short enough that every
    page is its own split-K piece (a piece boundary never depends on the
    other rows) and the projections compute each row's dot products alone.
The unmodified engine's tokens are compared with its single runs and
reported, not pinned: each head's scores sit at multiples of the batch's
padded score stride (the longest row), so the operand addresses of its P.V
GEMVs, and with them the kernel cuBLAS may pick and its FP32 summation order,
can change with the other rows of the batch, which flips random-weight
near-ties.  fast matches as native does;
batched sums its projections in one cuBLAS GEMM over the batch, whose order
depends on the row count, so it is reported only."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
RUNNER = ROOT / "tests" / "e2e_runner.py"
pytestmark = pytest.mark.gpu
MODES = ("compat", "fast", "batched", "native")


def _run(engine, mode="compat"):
    out = subprocess.run([sys.executable, str(RUNNER), "--engine", engine, "--mode", mode,
                          "--scheduler-case"], capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stderr[-3000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.fixture(scope="module")
def runs():
    for name in ("ref", "tvp"):
        if not (ROOT / "oracle" / "_ref" / f"libtvp_e2e_{name}.so").exists():
            pytest.skip("end-to-end engines not built (make -C oracle e2e)")
    res = {"ref": _run("ref")}
    for m in MODES:
        res[m] = _run("tvp", m)
    print("scheduler case, continuous == alone per request:",
          {k: [a == b for a, b in zip(v["continuous"], v["single"])] for k, v in res.items()})
    return res


def _check_events(r):
    slots = r["slots"]
    n = len(r["max_new"])
    active = [-1] * slots
    released_at = [-1] * slots
    released_pages, admitted = set(), set()
    reused, admissions = False, 0
    for e in r["events"]:
        if e["admitted"]:
            assert active[e["slot"]] == -1 and e["request_id"] not in admitted
            admitted.add(e["request_id"])
            if admissions < slots:
                assert e["iteration"] == 0 and e["request_id"] == admissions
            else:
                assert released_at[e["slot"]] == e["iteration"], "freed slot not refilled at once"
            active[e["slot"]] = e["request_id"]
            reused |= any(b in released_pages for b in e["blocks"])
            admissions += 1
        else:
            assert active[e["slot"]] == e["request_id"]
            active[e["slot"]] = -1
            released_at[e["slot"]] = e["iteration"]
            released_pages.update(e["blocks"])
    assert admissions == n and reused, "waiting queue or page reuse not exercised"
    assert all(a == -1 for a in active)
    assert r["events"][-1]["free_blocks"] == slots * r["max_seq_len"] // 16


@pytest.mark.parametrize("engine", ("ref",) + MODES)
def test_slots_and_pages_are_reused_and_returned(runs, engine):
    r = runs[engine]
    _check_events(r)
    assert [len(t) for t in r["continuous"]] == r["max_new"]
    assert len(set(r["max_new"])) >= 4
    assert r["edge_tokens"][0] == []                          # 0 tokens: no inference
    assert r["edge_tokens"][1] == r["continuous"][0][:1]      # 1 token: prefill only


@pytest.mark.parametrize("mode", MODES)
def test_event_log_matches_the_unmodified_engine(runs, mode):
    assert runs[mode]["events"] == runs["ref"]["events"]
    assert runs[mode]["edge_events"] == runs["ref"]["edge_events"]


@pytest.mark.parametrize("engine", ("compat", "fast", "native"))
def test_continuous_tokens_equal_each_request_alone(runs, engine):
    r = runs[engine]
    assert r["continuous"] == r["single"]
