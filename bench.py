"""Benchmark of the B200 paged-KV decode path (tiny-vLLM Llama-3.2-1B geometry).

Workload: decode_sweep — 256 rows with attended lengths L ~ U[512, 8192]
(seed 4), 16 layers, 32 Q / 8 KV heads, head_dim 64, BF16 N(0, 1) K/V in
16-token pages scattered over a pool sized to fit.  With N GPUs the 256 rows
are sharded by request (strong scaling: the job is the same at every N; each
GPU owns its rows, its page pool and its tables; no collective on the data
path).  One step = one decode step of the hot path over all 16 layers, replayed
as one CUDA graph: the plan, then per layer the fused RoPE(q, k) + paged append
of the new token and the fused GQA decode attention.  `weak_scaling` (N > 1)
gives every GPU the whole 256-row workload instead.

Metric: paged-decode KV GB/s = K+V bytes attended (sum_L * 2 KiB per layer) per
second, whole job; also decode tok/s and the fraction of measured HBM peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference algorithm's CPU restatement (the
reference has no CPU implementation of this path) on all host cores, on a
bounded sample of the same workload, and prints the same JSON line shape.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

import workloads as W  # noqa: E402

METRIC = "paged-decode KV GB/s"
UNIT = "GB/s"
PEAKS_FILE = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM_GBS = 6650.0
TRAFFIC_FILE = ROOT / "profiles" / "paged_decode_kernel.decode_sweep.json"


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class L2Flush:
    """Evicts L2 (126 MB) between timed launches: 256 MB written, then 256 MB of
    another buffer read, both outside the timed interval.  The read leaves L2
    holding clean lines of an unrelated buffer, so the next launch finds
    neither its own data in L2 nor dirty lines whose write-back to DRAM would
    be charged to it."""

    NOTE = "flushed between timed launches (256 MB written, then 256 MB of another buffer read)"

    def __init__(self, dev, nbytes=256 << 20):
        import torch
        self.w = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.r = torch.ones(nbytes // 4, dtype=torch.int32, device=dev)

    def __call__(self, i):
        self.w.fill_(i & 0xFF)
        return self.r.sum()


def hbm_peak():
    try:
        peaks = json.loads(PEAKS_FILE.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes(lens: np.ndarray) -> dict:
    """Bytes one decode-attention launch must move (one layer)."""
    lens = lens.astype(np.int64)
    kv = int(lens.sum()) * W.KV_DIM * 2 * 2          # K and V, 1 KiB each per token
    qo = int(lens.size) * W.Q_DIM * 2 * 2             # q in, out
    tables = int(((lens + 15) // 16).sum()) * 4
    return {"kv": kv, "q_out": qo, "tables": tables, "total": kv + qo + tables}


def config_block(world, global_rows, layers=16):
    return {
        "workload": "decode_sweep",
        "global_rows": global_rows,
        "rows_per_gpu": f"{global_rows} / {world}, sharded by request (greedy longest-first by sum L)",
        "seq_len": "L ~ U[512, 8192] (seed 4)",
        "layers": layers,
        "q_heads": 32,
        "kv_heads": 8,
        "head_dim": 64,
        "page_tokens": 16,
        "parallelism": f"request-sharded x{world} (no collective)",
        "step": "one CUDA-graph replay: plan + 16 x (RoPE/append, decode attention)",
        "l2": "inputs larger than L2 (>=2.2 GB of K+V per layer launch at 1 GPU; "
              ">=0.28 GB per launch at 8 GPUs)",
    }


# --------------------------------------------------------------- CPU legs ---
def cpu_sample_case(rows: int, seed: int = 4):
    lens = W.sweep_lengths(seed)[:rows]
    return W.decode_random(seed + 7, lens, slack_pages=0)


def time_cpu(rows: int, budget_s: float, threads: int = 0):
    """Times the oracle (reference semantics, OpenMP) on the first `rows` rows
    of the workload, one layer, repeated until `budget_s` elapsed."""
    import oracle
    case = cpu_sample_case(rows)
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    cores = threads if threads > 0 else len(os.sched_getaffinity(0))
    t0 = time.perf_counter()
    reps = 0
    while True:
        oracle.decode_attention(case.q, case.k_pool, case.v_pool, 0, case.tables, case.lens,
                                threads=cores)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    kv = algorithmic_bytes(case.lens)["kv"]
    gbs = kv * reps / el / 1e9
    return {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": (f"{rows} rows of decode_sweep (sum L = {int(case.lens.sum())}), 1 layer, "
                       f"{reps} repetitions in {el:.1f} s; oracle/tvp_oracle.c (reference "
                       "rounding points, FP32), OpenMP")}, el


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    rows = 32
    samples, step_ms = [], []
    for _ in range(args.warmup):
        time_cpu(rows, 0.5)
    for _ in range(args.steps):
        cb, el = time_cpu(rows, args.cpu_seconds / max(args.steps, 1))
        samples.append(cb["value"])
        step_ms.append(el * 1e3)
    value = statistics.median(samples)
    cb["value"] = round(value, 3)
    # Each timed step is a bounded sample of the workload (32 rows, 1 layer,
    # repeated for its share of --cpu-seconds); ms_per_step is its wall time.
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.median(step_ms), 1),
        "ms_per_step_basis": "wall time of one timed step: a bounded sample (32 rows of "
                             "decode_sweep, 1 layer, repeated), not a full decode step",
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config_block(world, 256), "cpu_baseline": cb,
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- clocks ---
class ClockSampler:
    """SM clock, maximum SM clock and clock-event reasons of one GPU, sampled
    while the timed region runs: every 5 ms through NVML (the library
    nvidia-smi reads these fields from), else by `nvidia-smi -lms 100`.  The
    GPU is found by the CUDA device's UUID, so CUDA_VISIBLE_DEVICES cannot
    point the sampler at another GPU."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        import torch
        self.device = torch.device(device)
        self.rows = []  # (sm MHz, max sm MHz, [active reasons])
        self.source = None
        self._stop = threading.Event()
        self.thread = self.proc = None

    def _nvml(self):
        import pynvml as nv
        import torch
        nv.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        h = nv.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        bits = [(name, getattr(nv, attr)) for name, attr in self.REASONS]

        def sample():
            r = reasons(h)
            self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), max_mhz,
                              [name for name, b in bits if r & b]))
        return sample

    def start(self):
        try:
            sample = self._nvml()
            sample()  # fails here, not in the thread, when NVML cannot read the GPU
            self.rows.clear()

            def loop():
                while True:
                    sample()
                    if self._stop.wait(0.005):
                        return
            self.source = "nvml, 5 ms"
            self.thread = threading.Thread(target=loop, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.rows.clear()
        try:
            import torch
            idx = torch.cuda._get_nvml_device_index(self.device)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(idx), "-lms", "100"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi, 100 ms"
            self.thread = threading.Thread(target=self._read_smi, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read_smi(self):
        names = [n for n, _ in self.REASONS]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                self.rows.append((float(parts[1]), float(parts[2]),
                                  [n for n, f in zip(names, parts[5:9]) if f.lower() == "active"]))
            except ValueError:
                continue

    def stop(self):
        self._stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        rows = list(self.rows)
        if not rows:
            return None
        return {"sm_mhz": statistics.median(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted({n for r in rows for n in r[2]}),
                "samples": len(rows), "source": self.source}


# ------------------------------------------------------------- our arm ---
def shard_case(global_case, world, rank, seed=4):
    """Rank `rank`'s share of the global decode_sweep: its rows (greedy
    longest-first by sum of L, vllm_b200.sharding) with their own page pool and
    block tables, as a GPU that owns those requests holds them.  One rank gets
    the global case itself."""
    from vllm_b200 import sharding
    if world == 1:
        return global_case, np.arange(global_case.batch)
    rows = sharding.shard_by_request(global_case.lens, world)[rank]
    lens = global_case.lens[rows]
    rng = np.random.default_rng(seed + 1000 + 7919 * (rank + 1))
    need = int(sum(W.pages_for(int(L)) for L in lens))
    num_pages = need + 64
    tables = W.scattered_tables(rng, lens, num_pages)
    return W.DecodeCase(lens=lens, tables=tables, num_pages=num_pages,
                        num_layers=global_case.num_layers), rows


class DecodeStep:
    """One GPU's decode step over its rows: the plan, then per layer the fused
    RoPE + paged append of the new token (K1) and the decode attention (K2).
    Pools and inputs are seeded and live in HBM."""

    def __init__(self, case, dev, seed):
        import torch
        from vllm_b200 import ops
        self.ops, self.dev, self.case = ops, dev, case
        B, P, layers = case.batch, case.num_pages, case.num_layers
        self.layers = layers
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        shape = (layers, P, 16, W.KV_DIM)
        self.k_pool = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        self.v_pool = torch.empty(shape, dtype=torch.bfloat16, device=dev)
        for l in range(layers):
            self.k_pool[l].normal_(generator=gen)
            self.v_pool[l].normal_(generator=gen)
        self.tables = torch.from_numpy(case.tables).to(dev)
        self.seq_lens = torch.from_numpy(case.lens).to(dev)
        self.positions = self.seq_lens - 1
        self.q_all = torch.randn((layers, B, W.Q_DIM), generator=gen, device=dev).to(torch.bfloat16)
        self.k_new = torch.randn((layers, B, W.KV_DIM), generator=gen, device=dev).to(torch.bfloat16)
        self.v_new = torch.randn((layers, B, W.KV_DIM), generator=gen, device=dev).to(torch.bfloat16)
        self.out = torch.empty((layers, B, W.Q_DIM), dtype=torch.bfloat16, device=dev)
        self.err = ops.new_error_word(dev)
        self.ws = ops.DecodeWorkspace(B, dev)
        self.stride = case.tables.shape[1]

    def __call__(self, stream, q=None, k=None, v=None, events=None, after_layer=None,
                 before_layer=None):
        ops = self.ops
        q = self.q_all if q is None else q
        k = self.k_new if k is None else k
        v = self.v_new if v is None else v
        ops.decode_plan(self.seq_lens, self.stride, self.ws, error=self.err, stream=stream)
        for l in range(self.layers):
            if before_layer is not None:
                before_layer(l)
            ops.rope_append(self.k_pool, self.v_pool, l, self.tables, self.positions, k[l], v[l],
                            q=q[l], writeback_k=False, error=self.err, stream=stream)
            if events is not None:
                events[l][0].record(stream)
            ops.paged_decode_attention(q[l], self.k_pool, self.v_pool, l, self.tables,
                                       self.seq_lens, self.ws, out=self.out[l], error=self.err,
                                       stream=stream)
            if events is not None:
                events[l][1].record(stream)
            if after_layer is not None:
                after_layer(l)

    def check(self):
        import torch
        torch.cuda.synchronize(self.dev)
        assert int(self.err.item()) == 0, f"device error bits {int(self.err.item())}"


def measure_steps(step, args, world, local_rank, clocks=None):
    """Device time of args.steps decode steps, max over ranks: each step is one
    replay of a CUDA graph of the step (its 1 + 2 x layers launches), timed
    with CUDA events on the replay stream between barriers.  Returns
    (ms per step, average K2 launch ms of this rank, clock record)."""
    import torch
    import torch.distributed as dist
    dev = step.dev
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step(stream)
    step.check()
    # the dominant kernel's live launch time: events around every K2 launch of
    # args.steps eager steps (outside the graph, so each event brackets one launch)
    ev = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(step.layers)]
          for _ in range(args.steps)]
    for s in range(args.steps):
        step(stream, events=ev[s])
    step.check()
    attn_ms = statistics.mean(e[0].elapsed_time(e[1]) for s in ev for e in s)

    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        step(side)  # warm the side stream once outside capture
    stream.wait_stream(side)
    torch.cuda.synchronize(dev)
    with torch.cuda.graph(graph, capture_error_mode="thread_local"):
        step(torch.cuda.current_stream(dev))
    for _ in range(args.warmup):
        graph.replay()
    step.check()

    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    if clocks is not None:
        clocks.start()
    t0.record(stream)
    for _ in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clock_info = clocks.stop() if clocks is not None else None
    step.check()
    ms_total = t0.elapsed_time(t1)
    if world > 1:
        t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    del graph
    return ms_total / args.steps, attn_ms, clock_info


def measure_e2e(step, args, world, local_rank):
    """The same steps through the C-ABI with host buffers: every step copies
    its q, k, v rows in from pinned host memory and its attention rows out,
    inside the timed region.  Layer l's inputs arrive on an H2D stream and
    layer l waits only for them; layer l's output leaves on a D2H stream as
    soon as the layer is done, as in a serving loop.  Returns (ms per step, max
    over ranks; H2D bytes; D2H bytes)."""
    import torch
    import torch.distributed as dist
    dev = step.dev
    stream = torch.cuda.current_stream(dev)
    layers = step.layers
    q_h = step.q_all.cpu().pin_memory()
    k_h = step.k_new.cpu().pin_memory()
    v_h = step.v_new.cpu().pin_memory()
    out_h = torch.empty(step.out.shape, dtype=step.out.dtype).pin_memory()
    q_d, k_d, v_d = (torch.empty_like(step.q_all), torch.empty_like(step.k_new),
                     torch.empty_like(step.v_new))
    h2d_stream = torch.cuda.Stream(dev)
    d2h_stream = torch.cuda.Stream(dev)
    step_done = torch.cuda.Event()
    step_done.record(stream)

    def e2e_step():
        h2d_stream.wait_event(step_done)  # the previous step no longer reads q_d, k_d, v_d
        arrived = []
        with torch.cuda.stream(h2d_stream):
            for l in range(layers):
                q_d[l].copy_(q_h[l], non_blocking=True)
                k_d[l].copy_(k_h[l], non_blocking=True)
                v_d[l].copy_(v_h[l], non_blocking=True)
                arrived.append(torch.cuda.Event())
                arrived[-1].record(h2d_stream)

        def before(l):
            stream.wait_event(arrived[l])

        def after(l):
            done = torch.cuda.Event()
            done.record(stream)
            d2h_stream.wait_event(done)
            with torch.cuda.stream(d2h_stream):
                out_h[l].copy_(step.out[l], non_blocking=True)

        step(stream, q=q_d, k=k_d, v=v_d, before_layer=before, after_layer=after)
        sent = torch.cuda.Event()
        sent.record(d2h_stream)
        stream.wait_event(sent)
        step_done.record(stream)

    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step.check()
    h2d = (q_h.numel() + k_h.numel() + v_h.numel()) * 2
    d2h = out_h.numel() * 2
    return ms / args.steps, h2d, d2h


def gather_rank_stats(dev, world, values):
    """[world][len(values)] of every rank's values (one all_gather)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    if world == 1:
        return [list(values)]
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def run_ours(args, rank, world, local_rank):
    import torch

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    global_case = W.decode_sweep(seed=4, batch=args.rows)
    global_case.num_layers = args.layers
    layers = args.layers
    case, rows = shard_case(global_case, world, rank)
    step = DecodeStep(case, dev, seed=1234 + rank)

    clocks = ClockSampler(dev)
    ms_per_step, attn_ms, clock_info = measure_steps(step, args, world, local_rank, clocks)
    global_kv_step = algorithmic_bytes(global_case.lens)["kv"] * layers
    value = global_kv_step / (ms_per_step / 1e3) / 1e9
    tok_s = global_case.batch / (ms_per_step / 1e3)
    e2e_ms, h2d, d2h = measure_e2e(step, args, world, local_rank)
    e2e_value = global_kv_step / (e2e_ms / 1e3) / 1e9
    nbytes = algorithmic_bytes(case.lens)
    per_rank = gather_rank_stats(dev, world, [case.batch, float(case.lens.sum()),
                                              attn_ms * 1e3, nbytes["total"]])

    weak = None
    if world > 1 and not args.no_extras:
        # every rank with the whole 256-row workload (per-GPU work fixed as N grows)
        step.k_pool = step.v_pool = None
        del step
        wstep = DecodeStep(global_case, dev, seed=1234 + rank)
        wms, _, _ = measure_steps(wstep, args, world, local_rank)
        wbytes = algorithmic_bytes(global_case.lens)["kv"] * layers * world
        weak = {"value": round(wbytes / (wms / 1e3) / 1e9, 2), "unit": UNIT,
                "ms_per_step": round(wms, 4), "rows_per_gpu": global_case.batch,
                "global_rows": global_case.batch * world, "scaling": "weak"}
        wstep.k_pool = wstep.v_pool = None
        del wstep
        torch.cuda.empty_cache()

    # KV-head-sharded long_context (every rank takes part; after the timed runs)
    head_sharded = None
    if world > 1 and W.KV_HEADS % world == 0 and not args.no_extras:
        head_sharded = bench_head_sharded(dev, rank, world, local_rank)

    if rank != 0:
        return
    peak, peak_kind = hbm_peak()
    achieved = nbytes["total"] / (attn_ms / 1e3) / 1e9
    traffic = None
    try:
        prof = json.loads(TRAFFIC_FILE.read_text())
        traffic = int(prof["dram_bytes_per_kv_byte"] * nbytes["kv"])
    except Exception:
        traffic = None
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) BF16 K/V/q, seeded lengths and page scatter)",
        "config": config_block(world, global_case.batch, layers),
        "decode_tok_s": round(tok_s, 1),
        "hbm_peak_frac": round(value / world / peak, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "tvp::paged_decode_kernel<7,2,true,true>",
                     "algorithmic_bytes_per_launch": nbytes["total"],
                     "avg_launch_ms": round(attn_ms, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "rank": 0},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "scope": "rank 0's copies; value over all ranks' bytes, max-over-ranks time"},
        "gpu_launches": args.steps * (1 + 2 * layers),
        "clocks": clock_info,
        "per_rank": [{"rank": r, "rows": int(v[0]), "sum_L": int(v[1]),
                      "k2_us_per_launch": round(v[2], 2),
                      "k2_GBps": round(v[3] / (v[2] / 1e6) / 1e9, 1)}
                     for r, v in enumerate(per_rank)],
    }
    if weak is not None:
        line["weak_scaling"] = weak
    if world == 1 and not args.no_extras:
        line.update(extras(args, dev, case, step.k_pool, step.v_pool, step.q_all, step.out,
                           step.tables, step.seq_lens, step.ws))
    if head_sharded is not None:
        line["long_context_head_sharded"] = head_sharded
    if world == 1 and not args.no_cpu_baseline:
        cb, _ = time_cpu(32, args.cpu_seconds)
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)


def extras(args, dev, case, k_pool, v_pool, q_all, out, tables, seq_lens, ws):
    """Spot parity at full size, the long-context workload and the reference's
    gather+cuBLAS path on decode_small (when its build is present)."""
    import torch
    import oracle
    from vllm_b200 import ops
    res = {}
    # parity spot check: 3 rows of layer 5 against exact attention
    rows = [0, int(np.argmax(case.lens)), int(np.argmin(case.lens))]
    layer = 5
    torch.cuda.synchronize(dev)
    ops.decode_plan(seq_lens, case.tables.shape[1], ws)
    ops.paged_decode_attention(q_all[layer], k_pool, v_pool, layer, tables, seq_lens, ws,
                               out=out[layer])
    torch.cuda.synchronize(dev)
    worst = 0.0
    for r in rows:
        L = int(case.lens[r])
        pages = case.tables[r, :(L + 15) // 16]
        kp = k_pool[layer][torch.from_numpy(pages).to(dev).long()]
        vpp = v_pool[layer][torch.from_numpy(pages).to(dev).long()]
        h = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
        kp_h, vp_h = h(kp)[None], h(vpp)[None]
        tab = np.arange(pages.size, dtype=np.int32)[None]
        exact = oracle.decode_attention_f64(h(q_all[layer][r:r + 1]), kp_h, vp_h, 0, tab,
                                            np.array([L], np.int32))
        got = W.bf16_to_f32(h(out[layer][r:r + 1])).astype(np.float64)
        worst = max(worst, float(np.abs(got - exact).max()))
    res["parity_spot_check"] = {"rows": rows, "layer": layer, "max_abs_err_vs_exact": worst,
                                "tolerance": "1e-2 abs + 2e-2 rel"}
    res["long_context"] = bench_long_context(dev)
    res["long_context_head_shards"] = bench_long_context_heads(dev)
    res["prefill"] = bench_prefill(dev)
    res["decode_small"] = bench_decode_small(dev)
    res["decode_projections"] = bench_projections(dev)
    res["e2e_llama"] = bench_e2e_llama()
    return res


def bench_e2e_llama():
    """The e2e workload (Llama-3.2-1B geometry, seeded random weights, 4 requests
    x 128 prompt + 128 greedy tokens, the reference's scheduler): tokens/s of the
    unmodified engine and of the engine with this path dropped in (best of 3
    runs each, the first of which also builds the decode step's graph; same
    B200, separate processes)."""
    libs = [ROOT / "oracle" / "_ref" / f"libtvp_e2e_{n}.so" for n in ("ref", "tvp")]
    if not all(p.exists() for p in libs):
        return {"note": "end-to-end engines not built (make -C oracle e2e)"}
    out = {"workload": "e2e: Llama-3.2-1B geometry, random N(0,0.02) weights, B=4, 128+128 tokens"}
    for name, args in (("reference", ["--engine", "ref"]),
                       ("ours_compat", ["--engine", "tvp", "--mode", "compat"]),
                       ("ours_fast", ["--engine", "tvp", "--mode", "fast"]),
                       ("ours_batched", ["--engine", "tvp", "--mode", "batched"]),
                       ("ours_native", ["--engine", "tvp", "--mode", "native"])):
        r = subprocess.run([sys.executable, str(ROOT / "tests" / "e2e_runner.py"), *args,
                            "--runs", "3"], capture_output=True, text=True, timeout=900)
        if r.returncode != 0:
            out[name] = {"error": r.stderr[-300:]}
            continue
        d = json.loads(r.stdout.strip().splitlines()[-1])
        out[name] = {"tok_s": round(d["tokens_generated"] / min(d["seconds"]), 1),
                     "seconds": [round(x, 3) for x in d["seconds"]]}
    for name in ("compat", "fast", "batched", "native"):
        try:
            out[f"speedup_{name}"] = round(out[f"ours_{name}"]["tok_s"] / out["reference"]["tok_s"], 2)
        except (KeyError, TypeError, ZeroDivisionError):
            pass
    return out


def bench_long_context(dev, iters=20):
    import torch
    from vllm_b200 import ops
    case = W.long_context(seed=5, batch=16, L=32768, num_layers=1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    shape = (1, case.num_pages, 16, W.KV_DIM)
    kp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    vp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    q = torch.randn((16, W.Q_DIM), generator=gen, device=dev).to(torch.bfloat16)
    tables = torch.from_numpy(case.tables).to(dev)
    lens = torch.from_numpy(case.lens).to(dev)
    ws = ops.DecodeWorkspace(16, dev)
    ops.decode_plan(lens, case.tables.shape[1], ws)
    out = torch.empty_like(q)
    for _ in range(3):
        ops.paged_decode_attention(q, kp, vp, 0, tables, lens, ws, out=out)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(iters)]
    torch.cuda.synchronize(dev)
    for a, b in ev:
        a.record()
        ops.paged_decode_attention(q, kp, vp, 0, tables, lens, ws, out=out)
        b.record()
    torch.cuda.synchronize(dev)
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    nb = algorithmic_bytes(case.lens)
    peak, kind = hbm_peak()
    gbs = nb["total"] / (ms / 1e3) / 1e9
    del kp, vp
    return {"workload": "long_context 16 x 32768, 1 layer, split-K", "us_per_launch": round(ms * 1e3, 2),
            "GBps": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4), "peak_source": kind,
            "inputs": "larger than L2 (1.07 GB per launch)"}


# Pools are freed back to torch's cache between workloads, not to the driver
# (no torch.cuda.empty_cache()): later workloads reuse memory already mapped.


def long_context_pools(dev, kv_heads, seed=99):
    """long_context geometry (16 x 32768, 1 layer) with pools of kv_heads heads."""
    import torch
    case = W.long_context(seed=5, batch=16, L=32768, num_layers=1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    shape = (1, case.num_pages, 16, kv_heads * W.HEAD_DIM)
    kp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    vp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
    q = torch.randn((16, kv_heads * W.GROUP * W.HEAD_DIM), generator=gen, device=dev)
    return case, kp, vp, q.to(torch.bfloat16)


def head_shard_bytes(lens, kv_heads):
    """Algorithmic bytes of one decode launch over kv_heads of the 8 KV heads."""
    nb = algorithmic_bytes(lens)
    kv = nb["kv"] * kv_heads // W.KV_HEADS
    return kv + nb["q_out"] * kv_heads // W.KV_HEADS + nb["tables"], kv


def bench_long_context_heads(dev, iters=20):
    """One GPU's share of KV-head-sharded long_context: the head-shard kernel on
    pools of 4, 2 and 1 KV heads (the 2-, 4- and 8-GPU shards)."""
    import torch
    from vllm_b200 import ops
    peak, kind = hbm_peak()
    res = {"workload": "long_context 16 x 32768, 1 layer, pools of kv_heads of the 8 heads",
           "peak_source": kind, "l2": L2Flush.NOTE}
    flush = L2Flush(dev)
    for kv_heads in (4, 2, 1):
        case, kp, vp, q = long_context_pools(dev, kv_heads)
        tables = torch.from_numpy(case.tables).to(dev)
        lens = torch.from_numpy(case.lens).to(dev)
        ws = ops.DecodeWorkspace(16, dev, kv_heads=kv_heads)
        ops.decode_plan(lens, case.tables.shape[1], ws)
        out = torch.empty_like(q)
        for _ in range(3):
            ops.paged_decode_attention(q, kp, vp, 0, tables, lens, ws, out=out)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(iters)]
        torch.cuda.synchronize(dev)
        for i, (a, b) in enumerate(ev):
            flush(i)
            a.record()
            ops.paged_decode_attention(q, kp, vp, 0, tables, lens, ws, out=out)
            b.record()
        torch.cuda.synchronize(dev)
        ms = statistics.median(a.elapsed_time(b) for a, b in ev)
        total, _ = head_shard_bytes(case.lens, kv_heads)
        gbs = total / (ms / 1e3) / 1e9
        res[f"kv_heads_{kv_heads}"] = {"us_per_launch": round(ms * 1e3, 2), "GBps": round(gbs, 1),
                                       "frac_of_peak": round(gbs / peak, 4),
                                       "bytes_per_launch": total}
        del kp, vp
    return res


def bench_head_sharded(dev, rank, world, local_rank, iters=20):
    """KV-head-sharded long_context over `world` GPUs: rank r holds 8 / world
    KV heads of every page and every rank ends with the [16, 2048] rows.  Two
    forms: the all-gather fused into the decode kernel (p2p: stores into every
    rank's rows over NVLink, then a bounded wait), and the decode followed by
    an NCCL all-gather.  Per-layer time is the max over ranks of CUDA-event
    time on the launching stream; layers alternate the gather buffers."""
    import torch
    import torch.distributed as dist
    from vllm_b200 import sharding
    kv_heads = W.KV_HEADS // world
    case, kp, vp, q = long_context_pools(dev, kv_heads, seed=99 + rank)
    tables = torch.from_numpy(case.tables).to(dev)
    lens = torch.from_numpy(case.lens).to(dev)
    stream = torch.cuda.current_stream(dev)
    res = {"workload": f"long_context 16 x 32768, 1 layer, {kv_heads} KV head(s) per GPU",
           "all_gather_bytes_per_rank": 16 * kv_heads * W.GROUP * W.HEAD_DIM * 2,
           "l2": L2Flush.NOTE}
    flush = L2Flush(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(iters)]
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)
        for i, (a, b) in enumerate(ev):
            flush(i)
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        ms = statistics.median(a.elapsed_time(b) for a, b in ev)
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    nb = algorithmic_bytes(case.lens)
    for mode in ("p2p", "nccl"):
        try:
            dec = sharding.HeadShardedDecode(16, device=dev, mode=mode)
        except RuntimeError as e:  # raised on every rank alike (the ranks agree first)
            res[mode] = {"error": str(e)[:200]}
            continue
        dec.plan(lens, case.tables.shape[1])
        ms = timed(lambda: dec.attend(q, kp, vp, 0, tables, lens))
        if mode == "nccl":
            res["us_decode_only"] = round(timed(lambda: dec.attend(q, kp, vp, 0, tables, lens,
                                                                   gather=False)) * 1e3, 2)
        res[mode] = {"us_per_layer": round(ms * 1e3, 2),
                     "aggregate_kv_GBps": round(nb["kv"] / (ms / 1e3) / 1e9, 1)}
        dec.close()
    if "error" not in res["p2p"]:
        res["p2p"]["collective"] = "fused into the decode kernel: peer stores over NVLink + flag wait"
    if "error" not in res["nccl"]:
        res["nccl"]["collective"] = "NCCL all_gather_into_tensor + interleave"
    del kp, vp
    return res


def tensor_peak():
    try:
        return float(json.loads(PEAKS_FILE.read_text())["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def bench_prefill(dev, iters=20):
    """K3, paged causal prefill attention: 4 prompts x 1024 tokens (the
    reference's cap) and 1 x 8192 (beyond it), 1 layer, L2 flushed between
    launches; against the reference's contiguous cuBLAS prefill path on the
    1024-token prompts (its per-prompt function, 4 calls)."""
    import ctypes
    import torch
    import oracle
    from vllm_b200 import ops
    peak, kind = tensor_peak()
    flush = L2Flush(dev)
    res = {"roofline": "tensor (bf16 mma); flops = 256 (p + 1) per query head per token at position p",
           "peak_source": f"{kind} bf16_tflops {peak}"}
    ref = oracle.load_reference()
    for name, prompts in (("4x1024", [1024] * 4), ("1x8192", [8192])):
        case = W.decode_random(21, prompts, with_data=False, slack_pages=0)
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        shape = (1, case.num_pages, 16, W.KV_DIM)
        kp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
        vp = torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=gen)
        n = sum(prompts)
        q = torch.randn((n, W.Q_DIM), generator=gen, device=dev).to(torch.bfloat16)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(prompts)]), dtype=torch.int32, device=dev)
        pos0 = torch.zeros(len(prompts), dtype=torch.int32, device=dev)
        tables = torch.from_numpy(case.tables).to(dev)
        out = torch.empty_like(q)
        times = []
        for i in range(iters + 3):
            flush(i)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            ops.paged_prefill_attention(q, kp, vp, 0, tables, cu, pos0, max(prompts), out=out)
            b.record()
            torch.cuda.synchronize(dev)
            if i >= 3:
                times.append(a.elapsed_time(b))
        us = statistics.median(times) * 1e3
        flops = sum(256.0 * (L * (L + 1) / 2) * W.Q_HEADS for L in prompts)
        entry = {"us": round(us, 2), "TFLOPs": round(flops / us / 1e6, 2),
                 "frac_of_peak": round(flops / us / 1e6 / peak, 4)}
        if ref is not None and max(prompts) <= 1024:
            # the reference's prefill attention, one prompt per call, same q/k/v per prompt
            ref_us = 0.0
            ref_out = torch.empty((1024, W.Q_DIM), dtype=torch.bfloat16, device=dev)
            for s, L in enumerate(prompts):
                pages = torch.from_numpy(case.tables[s, :(L + 15) // 16].astype(np.int64)).to(dev)
                kc = kp[0][pages].reshape(-1, W.KV_DIM)[:L].contiguous()
                vc = vp[0][pages].reshape(-1, W.KV_DIM)[:L].contiguous()
                qs = q[int(cu[s]):int(cu[s + 1])].contiguous()
                ms = ctypes.c_float(0.0)
                vptr = lambda t: ctypes.c_void_p(t.data_ptr())
                rc = ref.ref_prefill_attention(vptr(qs), vptr(kc), vptr(vc), L, vptr(ref_out),
                                               iters, 256 << 20, ctypes.byref(ms))
                if rc != 0:
                    ref_us = None
                    break
                ref_us += ms.value * 1e3
            if ref_us:
                entry["reference_cublas_us"] = round(ref_us, 2)
                entry["speedup_vs_reference"] = round(ref_us / us, 2)
        res[name] = entry
        del kp, vp
    return res


def bench_decode_small(dev, iters=50):
    """decode_small (4 rows, L = 17..256): our fused launch vs the reference's
    gather + cuBLAS + softmax sequence, both with L2 flushed between launches."""
    import ctypes
    import torch
    import oracle
    from vllm_b200 import ops
    case = W.decode_small()
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)
    k, v, q = to(case.k_pool), to(case.v_pool), to(case.q)
    tables = torch.from_numpy(case.tables).to(dev)
    lens = torch.from_numpy(case.lens).to(dev)
    ws = ops.DecodeWorkspace(4, dev)
    out = torch.empty_like(q)
    flush = L2Flush(dev)
    times = []
    for i in range(iters + 3):
        flush(i)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ops.decode_plan(lens, case.tables.shape[1], ws)
        ops.paged_decode_attention(q, k, v, 0, tables, lens, ws, out=out)
        b.record()
        torch.cuda.synchronize(dev)
        if i >= 3:
            times.append(a.elapsed_time(b))
    ours_us = statistics.median(times) * 1e3
    res = {"workload": "decode_small 4 rows L={17,64,129,256}, 1 layer, L2 flushed",
           "ours_us_plan_plus_attention": round(ours_us, 2)}
    ref = oracle.load_reference()
    if ref is None:
        res["reference_gather_cublas_us"] = None
        res["note"] = "reference build (oracle/_ref) not present"
        return res
    ref_out = torch.empty_like(q)
    tab = np.ascontiguousarray(case.tables, np.int32)
    ln = np.ascontiguousarray(case.lens, np.int32)
    ms = ctypes.c_float(0.0)
    rc = ref.ref_paged_decode(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                              ctypes.c_void_p(v.data_ptr()), case.num_pages, 0,
                              tab.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), tab.shape[1],
                              ln.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), 4,
                              ctypes.c_void_p(ref_out.data_ptr()), iters, 256 << 20,
                              ctypes.byref(ms))
    if rc != 0:
        res["reference_gather_cublas_us"] = None
        res["note"] = f"reference path returned {rc}"
        return res
    ref_us = ms.value * 1e3
    res["reference_gather_cublas_us"] = round(ref_us, 2)
    res["speedup_vs_reference"] = round(ref_us / ours_us, 2)
    kv = algorithmic_bytes(case.lens)["kv"]
    res["reference_kv_GBps"] = round(kv / (ref_us / 1e6) / 1e9, 3)
    res["ours_kv_GBps"] = round(kv / (ours_us / 1e6) / 1e9, 3)
    return res


def bench_projections(dev, iters=20):
    """K5 (tvp_decode_projections): one decode layer's projections of the
    Llama-3.2-1B geometry over 4 rows (Q+K+V, O, gate+up, down: 121.6 MB of
    BF16 weights, 4 launches) and its LM head (128256 x 2048, 525 MB, FP32
    logits), each launch timed alone with L2 flushed before it; against torch's
    cuBLAS BF16 GEMMs of the same shapes (the batched engine's 7 projection
    GEMMs and its LM head GEMM).  Roofline: HBM, bytes = the weights."""
    import torch
    from vllm_b200 import ops
    peak, kind = hbm_peak()
    g = torch.Generator(device=dev).manual_seed(3)
    H, I, KV, VOC, B = 2048, 8192, 512, 128256, 4

    def w(n, k):
        return (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    x = torch.randn(B, H, generator=g, device=dev).to(torch.bfloat16)
    xi = torch.randn(B, I, generator=g, device=dev).to(torch.bfloat16)
    wq, wk, wv, wo, wg, wu, wd = w(H, H), w(KV, H), w(KV, H), w(H, H), w(I, H), w(I, H), w(H, I)
    emb = w(VOC, H)
    o = lambda n, dt=torch.bfloat16: torch.empty(B, n, dtype=dt, device=dev)
    oq, ok, ov, oo, og, ou, od, ol = o(H), o(KV), o(KV), o(H), o(I), o(I), o(H), o(VOC, torch.float32)
    flush = L2Flush(dev)

    def timed(fn):
        # Every iteration is enqueued before one synchronisation, so the host's
        # launch overhead never leaves the GPU idle between the events (the
        # 256 MB flush before each launch keeps the host ahead).
        ev = []
        for i in range(iters + 3):
            flush(i)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            ev.append((a, b))
        torch.cuda.synchronize(dev)
        return statistics.median(a.elapsed_time(b) for a, b in ev[3:]) * 1e3  # us

    layer = {
        "qkv": (lambda: ops.decode_projections(x, [wq, wk, wv], outs=[oq, ok, ov]), [wq, wk, wv]),
        "o": (lambda: ops.decode_projections(x, [wo], outs=[oo]), [wo]),
        "gate_up": (lambda: ops.decode_projections(x, [wg, wu], outs=[og, ou]), [wg, wu]),
        "down": (lambda: ops.decode_projections(xi, [wd], outs=[od]), [wd]),
    }
    cublas = {
        "qkv": lambda: (torch.mm(x, wq.t(), out=oq), torch.mm(x, wk.t(), out=ok),
                        torch.mm(x, wv.t(), out=ov)),
        "o": lambda: torch.mm(x, wo.t(), out=oo),
        "gate_up": lambda: (torch.mm(x, wg.t(), out=og), torch.mm(x, wu.t(), out=ou)),
        "down": lambda: torch.mm(xi, wd.t(), out=od),
    }
    res = {"workload": "Llama-3.2-1B decode projections, 4 rows, BF16 weights, L2 flushed",
           "roofline": "hbm; bytes = weights read", "peak_source": kind}
    tot_ours = tot_lib = tot_bytes = 0.0
    for name, (fn, ws) in layer.items():
        nbytes = sum(t.numel() * 2 for t in ws)
        us, lib_us = timed(fn), timed(cublas[name])
        tot_ours += us
        tot_lib += lib_us
        tot_bytes += nbytes
        res[name] = {"us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
                     "frac_of_peak": round(nbytes / us / 1e3 / peak, 4),
                     "cublas_us": round(lib_us, 2)}
    res["layer"] = {"us": round(tot_ours, 2), "bytes": int(tot_bytes),
                    "GBps": round(tot_bytes / tot_ours / 1e3, 1),
                    "frac_of_peak": round(tot_bytes / tot_ours / 1e3 / peak, 4),
                    "cublas_us": round(tot_lib, 2),
                    "speedup_vs_cublas": round(tot_lib / tot_ours, 2)}
    nb = emb.numel() * 2
    us = timed(lambda: ops.decode_projections(x, [emb], outs=[ol], epilogue="f32"))
    olb = o(VOC)
    lib_us = timed(lambda: torch.mm(x, emb.t(), out=olb))
    res["lm_head"] = {"us": round(us, 2), "GBps": round(nb / us / 1e3, 1),
                      "frac_of_peak": round(nb / us / 1e3 / peak, 4),
                      "cublas_bf16_out_us": round(lib_us, 2)}
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rows", type=int, default=256, help="decode rows per GPU (256)")
    ap.add_argument("--layers", type=int, default=16, help="layers per step (16)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--only", choices=["long_context", "long_context_heads", "decode_small",
                                       "prefill", "e2e", "projections"],
                    help="run one single-GPU sub-measurement alone and print its JSON (profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = env_int("WORLD_SIZE", 1)
    rank = env_int("RANK", 0)
    local_rank = env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.only:
        import torch
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        fn = {"long_context": bench_long_context, "long_context_heads": bench_long_context_heads,
              "decode_small": bench_decode_small, "prefill": bench_prefill,
              "e2e": lambda _dev: bench_e2e_llama(), "projections": bench_projections}[args.only]
        print(json.dumps({args.only: fn(dev)}), flush=True)
        return
    import torch
    import torch.distributed as dist
    if world > 1:
        import datetime
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
