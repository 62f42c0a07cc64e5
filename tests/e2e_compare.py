"""Teacher-forced comparison of the engine with the B200 paged-KV path dropped
in against the unmodified engine (e2e workload).  Test infrastructure only;
runs on a GPU machine with oracle/_ref/libtvp_e2e_{ref,tvp}.so built.

1. The unmodified engine generates 128 greedy tokens per request (scheduler).
2. Both engines then decode the same forced inputs (those tokens), and every
   step's logits are compared: argmax agreement, logit differences, and, where
   the argmax differs, the gap between the two candidates in the reference's own
   logits after its BF16 rounding (src/model/argmax.cu:24), in BF16 ulps.

3. Every engine mode also generates freely, and its sequences are compared
   with the reference's: a free-running sequence can only leave the
   reference's at the first step where the teacher-forced argmax differed,
   since up to that step both runs decode the same inputs.

Prints one JSON summary line."""
from __future__ import annotations

import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
RUNNER = ROOT / "tests" / "e2e_runner.py"


def bf16_round(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    e = np.floor(np.log2(np.maximum(np.abs(x), 1e-30)))
    return np.exp2(e - 7)


def runner(args):
    out = subprocess.run([sys.executable, str(RUNNER), *args], capture_output=True, text=True,
                         timeout=1200)
    if out.returncode != 0:
        raise SystemExit(out.stderr[-3000:])
    return json.loads(out.stdout.strip().splitlines()[-1])


def compare() -> dict:
    tmp = Path(tempfile.mkdtemp())
    free = runner(["--engine", "ref", "--runs", "1"])
    gen = np.array(free["tokens"], np.int32)            # [4][128]
    free_runs = {m: np.array(runner(["--engine", "tvp", "--mode", m, "--runs", "1"])["tokens"],
                             np.int32) for m in ("compat", "fast", "batched", "native")}
    forced = gen[:, :-1]                                 # inputs of decode steps 0..126
    (tmp / "forced.json").write_text(json.dumps(forced.tolist()))
    logs = {}
    results = {}
    for name, args in {"ref": ["--engine", "ref"], "compat": ["--engine", "tvp", "--mode", "compat"],
                       "fast": ["--engine", "tvp", "--mode", "fast"],
                       "batched": ["--engine", "tvp", "--mode", "batched"],
                       "native": ["--engine", "tvp", "--mode", "native"]}.items():
        path = tmp / f"{name}.npy"
        results[name] = runner([*args, "--teacher-forced", str(tmp / "forced.json"),
                                "--logits-out", str(path)])
        logs[name] = np.load(path, mmap_mode="r")
        logs[name + "_prefill"] = np.load(str(path) + ".prefill.npy")
    ref = logs["ref"]
    summary = {"workload": "e2e: 4 requests x 128 prompt tokens, 127 teacher-forced decode steps",
               "reference_free_running_matches_teacher_forced":
                   bool(np.array_equal(np.array(results["ref"]["step_tokens"]), gen[:, 1:]))}
    rtok = np.array(results["ref"]["step_tokens"])        # [4][127]

    def gap(lr, top_tok, other_tok):
        b = bf16_round(lr)
        top = b[top_tok]
        return float((top - b[other_tok]) / bf16_ulp(np.array([top]))[0])

    for name in ("compat", "fast", "batched", "native"):
        ours = np.array(results[name]["step_tokens"])
        agree = ours == rtok
        gaps = []
        max_diff = 0.0
        for step in range(ref.shape[0]):
            lr = np.asarray(ref[step], np.float32)
            lo = np.asarray(logs[name][step], np.float32)
            max_diff = max(max_diff, float(np.abs(lr - lo).max()))
            for r in range(ref.shape[1]):
                if ours[r, step] != rtok[r, step]:
                    b = bf16_round(lr[r])
                    top = b[rtok[r, step]]
                    gaps.append(float((top - b[ours[r, step]]) / bf16_ulp(np.array([top]))[0]))
        rfirst, ofirst = results["ref"]["first_tokens"], results[name]["first_tokens"]
        first_gaps = [gap(np.asarray(logs["ref_prefill"][r], np.float32), rfirst[r], ofirst[r])
                      for r in range(len(rfirst)) if rfirst[r] != ofirst[r]]
        # first differing index of each free-running sequence (None: identical),
        # and the first teacher-forced disagreement, as a token index (step + 1)
        free_div, forced_div = [], []
        for r in range(gen.shape[0]):
            d = np.nonzero(free_runs[name][r] != gen[r])[0]
            free_div.append(int(d[0]) if d.size else None)
            if rfirst[r] != ofirst[r]:
                forced_div.append(0)
            else:
                e = np.nonzero(ours[r] != rtok[r])[0]
                forced_div.append(int(e[0]) + 1 if e.size else None)
        summary[name] = {
            "free_running_identical": [d is None for d in free_div],
            "free_running_first_divergence": free_div,
            "teacher_forced_first_disagreement": forced_div,
            "first_tokens_match": rfirst == ofirst,
            "first_token_gap_bf16_ulps": sorted(first_gaps),
            "argmax_agreement": float(agree.mean()),
            "disagreements": int((~agree).sum()),
            "gap_at_disagreement_bf16_ulps": sorted(gaps),
            "max_abs_logit_diff": max_diff,
            "max_abs_reference_logit": float(max(np.abs(np.asarray(ref[s], np.float32)).max()
                                                 for s in range(0, ref.shape[0], 16))),
        }
    for path in tmp.iterdir():
        path.unlink()
    tmp.rmdir()
    return summary


if __name__ == "__main__":
    print(json.dumps(compare()))
