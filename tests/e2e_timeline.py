"""Live kernel timeline of the e2e workload through the engine with the paged-KV
path dropped in (oracle/_ref/libtvp_e2e_tvp.so), recorded with torch.profiler
(CUPTI kernel records: real start and end times, kernels of replayed graphs
included, programmatic-launch overlap visible).  Test infrastructure only.

  python tests/e2e_timeline.py [--mode native] [--new 24] [--trace out.json]

Prints, for the decode step in the middle of the run, every kernel with its
start (relative to the step's plan kernel) and duration, and per layer the
critical path: for each launch, the time from the end of the launch before it
to its own end.  Then the medians over all steps, and the prefill kernels'
totals.  Times carry the profiler's overhead on the host side; kernel
durations do not.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import tempfile
from collections import defaultdict
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
import e2e_runner as R  # noqa: E402

SHORT = [("decode_plan", "plan"), ("paged_decode_kernel", "K2"), ("decode_projection_kernel", "K5"),
         ("greedy_argmax", "K4"), ("embeddingGather", "embedding"), ("rmsNormKernel", "rmsnorm"),
         ("rope_append", "K1"), ("paged_prefill", "K3")]


def short(name: str) -> str:
    for key, tag in SHORT:
        if key in name:
            if tag in ("K5", "K2") and "<" in name:
                return tag + name[name.find("<"):name.find(">") + 1]
            return tag
    return name[:48]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", default="native", choices=["compat", "fast", "batched", "native"])
    ap.add_argument("--new", type=int, default=24, help="tokens generated per request")
    ap.add_argument("--trace", help="also keep the chrome trace here")
    args = ap.parse_args()
    os.environ["TVP_DECODE_MODE"] = args.mode
    torch.zeros(1, device="cuda")  # the profiler's context first
    lib = ctypes.CDLL(os.fspath(R.LIBS["tvp"]))
    lib.e2e_init.argtypes = [ctypes.c_ulonglong]
    i32p = ctypes.POINTER(ctypes.c_int32)
    lib.e2e_generate.argtypes = [i32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_int, i32p, i32p, ctypes.POINTER(ctypes.c_double)]
    if lib.e2e_init(3) != 0:
        raise SystemExit("weight setup failed")
    p = R.prompts(4, 128, 3)
    out = np.zeros((4, args.new), np.int32)
    counts = np.zeros(4, np.int32)

    def generate():
        sec = ctypes.c_double(0)
        if lib.e2e_generate(p.ctypes.data_as(i32p), 4, 128, args.new, 4, 128 + args.new,
                            out.ctypes.data_as(i32p), counts.ctypes.data_as(i32p),
                            ctypes.byref(sec)) != 0:
            raise SystemExit("generation failed")
        return sec.value

    generate()
    generate()  # graphs recorded: the profiled run replays them
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
        wall = generate()
    path = args.trace or tempfile.mktemp(suffix=".json")
    prof.export_chrome_trace(path)
    events = json.load(open(path))["traceEvents"]
    if not args.trace:
        os.unlink(path)
    k = sorted((e for e in events if e.get("cat") == "kernel"), key=lambda e: e["ts"])
    plans = [i for i, e in enumerate(k) if "decode_plan" in e["name"]]
    print(f"mode {args.mode}: wall {wall * 1e3:.2f} ms under the profiler, {len(k)} kernels, "
          f"{len(plans)} decode steps")
    pre = k[:plans[0]] if plans else k
    agg = defaultdict(lambda: [0, 0.0])
    for e in pre:
        agg[short(e["name"])][0] += 1
        agg[short(e["name"])][1] += e["dur"]
    print(f"prefill phase: span {pre[-1]['ts'] + pre[-1]['dur'] - pre[0]['ts']:.1f} us, "
          f"kernels busy {sum(v[1] for v in agg.values()):.1f} us")
    for name, (n, d) in sorted(agg.items(), key=lambda x: -x[1][1])[:8]:
        print(f"  {d:9.1f} us {n:5d}x {d / n:7.2f}  {name}")
    if len(plans) < 3:
        return
    steps = [k[a:b] for a, b in zip(plans, plans[1:])]
    mid = steps[len(steps) // 2]
    t0 = mid[0]["ts"]
    print("middle step (start, duration, critical-path share = own end - previous end):")
    prev_end = None
    for e in mid:
        end = e["ts"] + e["dur"]
        crit = end - prev_end if prev_end is not None else e["dur"]
        print(f"  {e['ts'] - t0:9.2f} {e['dur']:7.2f} {crit:7.2f}  {short(e['name'])} "
              f"grid={e['args'].get('grid')}")
        prev_end = max(prev_end or 0, end)
    # per position in the step: the median critical-path share over steps
    by_pos = defaultdict(list)
    for s in steps:
        prev_end = None
        for j, e in enumerate(s):
            end = e["ts"] + e["dur"]
            by_pos[(j, short(e["name"]))].append(end - prev_end if prev_end is not None else e["dur"])
            prev_end = max(prev_end or 0, end)
    kinds = defaultdict(list)
    for (j, name), v in by_pos.items():
        kinds[name].append(statistics.median(v))
    print("median critical-path share per launch, by kernel:")
    for name, v in sorted(kinds.items(), key=lambda x: -sum(x[1])):
        print(f"  {name:24s} {len(v):3d} launches/step  {statistics.median(v):7.2f} us each, "
              f"{sum(v):8.1f} us per step")
    spans = [s[-1]["ts"] + s[-1]["dur"] - s[0]["ts"] for s in steps]
    gaps = [steps[i + 1][0]["ts"] - (steps[i][-1]["ts"] + steps[i][-1]["dur"]) for i in range(len(steps) - 1)]
    print(f"step: kernels span {statistics.median(spans):.1f} us (median), "
          f"then {statistics.median(gaps):.1f} us to the next step's plan (host, under the profiler)")


if __name__ == "__main__":
    main()
