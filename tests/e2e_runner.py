"""Runs the e2e workload (Llama-3.2-1B geometry, seeded random weights) through
one build of the engine and prints JSON: generated tokens per request and wall
seconds per run.  One engine per process (both builds define the same symbols).

  python tests/e2e_runner.py --engine ref|tvp [--mode compat|fast] [--runs 2]

The `ref` engine is the unmodified reference (oracle/_ref/libtvp_e2e_ref.so);
`tvp` is the reference with the B200 paged-KV path dropped in
(oracle/_ref/libtvp_e2e_tvp.so).  Test infrastructure only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
LIBS = {"ref": ROOT / "oracle" / "_ref" / "libtvp_e2e_ref.so",
        "tvp": ROOT / "oracle" / "_ref" / "libtvp_e2e_tvp.so"}


def prompts(requests: int, length: int, seed: int) -> np.ndarray:
    """Seeded random prompt token IDs below the EOS ids."""
    return np.random.default_rng(seed).integers(0, 128000, size=(requests, length)).astype(np.int32)


# Continuous-batching scenario: 7 requests with ragged prompts and output
# lengths through 3 slots (as the reference's batch test drives its scheduler,
# tests/paged_inference_test.cu:149-224), context cap 128.
SCHED_PROMPTS = [37, 12, 64, 5, 90, 23, 48]
SCHED_NEW = [9, 3, 14, 1, 6, 11, 4]
SCHED_SLOTS = 3
SCHED_MAX_SEQ = 128


def generate_requests(lib, prompt_list, max_new, slots, max_seq):
    i32p = ctypes.POINTER(ctypes.c_int32)
    flat = np.ascontiguousarray(np.concatenate([np.asarray(x, np.int32) for x in prompt_list]),
                                np.int32)
    offs = np.concatenate([[0], np.cumsum([len(x) for x in prompt_list])]).astype(np.int32)
    new = np.asarray(max_new, np.int32)
    n = len(prompt_list)
    max_out = max(1, int(new.max()))
    out = np.zeros((n, max_out), np.int32)
    counts = np.zeros(n, np.int32)
    ev = np.zeros(1 << 16, np.int32)
    ev_len = ctypes.c_int(0)
    lib.e2e_generate_requests.argtypes = [i32p, i32p, i32p, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, i32p, i32p, i32p,
                                          ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    rc = lib.e2e_generate_requests(flat.ctypes.data_as(i32p), offs.ctypes.data_as(i32p),
                                   new.ctypes.data_as(i32p), n, slots, max_seq, max_out,
                                   out.ctypes.data_as(i32p), counts.ctypes.data_as(i32p),
                                   ev.ctypes.data_as(i32p), ev.size, ctypes.byref(ev_len))
    if rc != 0:
        raise SystemExit(f"generateContinuous failed ({rc})")
    events, i = [], 0
    while i < ev_len.value:
        it, slot, rid, adm, free, nb = (int(x) for x in ev[i:i + 6])
        events.append({"iteration": it, "slot": slot, "request_id": rid, "admitted": bool(adm),
                       "free_blocks": free, "blocks": ev[i + 6:i + 6 + nb].tolist()})
        i += 6 + nb
    tokens = [out[r, :counts[r]].tolist() for r in range(n)]
    return tokens, events


def scheduler_case(lib, seed):
    rng = np.random.default_rng(seed + 17)
    plist = [rng.integers(0, 128000, size=L).astype(np.int32) for L in SCHED_PROMPTS]
    tokens, events = generate_requests(lib, plist, SCHED_NEW, SCHED_SLOTS, SCHED_MAX_SEQ)
    single = [generate_requests(lib, [plist[r]], [SCHED_NEW[r]], 1, SCHED_MAX_SEQ)[0][0]
              for r in range(len(plist))]
    edge_tokens, edge_events = generate_requests(lib, [np.array([128000], np.int32), plist[0]],
                                                 [0, 1], 1, SCHED_MAX_SEQ)
    return {"slots": SCHED_SLOTS, "max_seq_len": SCHED_MAX_SEQ, "max_new": SCHED_NEW,
            "prompt_lens": SCHED_PROMPTS, "continuous": tokens, "events": events,
            "single": single, "edge_tokens": edge_tokens, "edge_events": edge_events}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--engine", choices=sorted(LIBS), required=True)
    ap.add_argument("--mode", choices=["compat", "fast", "batched", "native"], default="compat")
    ap.add_argument("--requests", type=int, default=4)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--new", type=int, default=128)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--runs", type=int, default=2)
    ap.add_argument("--teacher-forced", help="JSON file: tokens [requests][steps] fed as decode inputs")
    ap.add_argument("--logits-out", help="with --teacher-forced: .npy of FP32 logits [steps][requests][vocab]")
    ap.add_argument("--scheduler-case", action="store_true",
                    help="continuous batching of ragged requests through fewer slots, each "
                         "request alone, and the 0- and 1-token edge requests (JSON out)")
    args = ap.parse_args()
    os.environ["TVP_DECODE_MODE"] = args.mode
    lib = ctypes.CDLL(os.fspath(LIBS[args.engine]))
    lib.e2e_init.argtypes = [ctypes.c_ulonglong]
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib.e2e_generate.argtypes = [i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, i32p, i32p, ctypes.POINTER(ctypes.c_double)]
    if lib.e2e_init(args.seed) != 0:
        raise SystemExit("weight setup failed")
    if args.scheduler_case:
        json.dump(scheduler_case(lib, args.seed), sys.stdout)
        print()
        return
    p = prompts(args.requests, args.prompt, args.seed)
    if args.teacher_forced:
        forced = np.ascontiguousarray(json.load(open(args.teacher_forced)), dtype=np.int32)
        steps = forced.shape[1]
        lib.e2e_teacher_forced.argtypes = [i32p, ctypes.c_int, ctypes.c_int, i32p, ctypes.c_int,
                                           ctypes.c_int, i32p, i32p, ctypes.c_void_p,
                                           ctypes.c_void_p]
        first = np.zeros(args.requests, np.int32)
        step_tokens = np.zeros((steps, args.requests), np.int32)
        logits = np.zeros((steps, args.requests, 128256), np.float32) if args.logits_out else None
        first_logits = np.zeros((args.requests, 128256), np.float32) if args.logits_out else None
        rc = lib.e2e_teacher_forced(p.ctypes.data_as(i32p), args.requests, args.prompt,
                                    forced.ctypes.data_as(i32p), steps, args.prompt + steps + 1,
                                    first.ctypes.data_as(i32p), step_tokens.ctypes.data_as(i32p),
                                    logits.ctypes.data if logits is not None else None,
                                    first_logits.ctypes.data if first_logits is not None else None)
        if rc != 0:
            raise SystemExit(f"teacher-forced decode failed ({rc})")
        if logits is not None:
            np.save(args.logits_out, logits)
            np.save(str(args.logits_out) + ".prefill.npy", first_logits)
        json.dump({"engine": args.engine, "mode": args.mode, "first_tokens": first.tolist(),
                   "step_tokens": step_tokens.T.tolist()}, sys.stdout)
        print()
        return
    out = np.zeros((args.requests, args.new), np.int32)
    counts = np.zeros(args.requests, np.int32)
    seconds = []
    for _ in range(args.runs):
        sec = ctypes.c_double(0.0)
        rc = lib.e2e_generate(p.ctypes.data_as(i32p), args.requests, args.prompt, args.new,
                              args.batch, args.prompt + args.new, out.ctypes.data_as(i32p),
                              counts.ctypes.data_as(i32p), ctypes.byref(sec))
        if rc != 0:
            raise SystemExit(f"generation failed ({rc})")
        seconds.append(sec.value)
    json.dump({"engine": args.engine, "mode": args.mode, "tokens": out.tolist(),
               "counts": counts.tolist(), "seconds": seconds,
               "tokens_generated": int(counts.sum())}, sys.stdout)
    print()


if __name__ == "__main__":
    main()
