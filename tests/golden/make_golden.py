"""Generates the golden vectors of the paged-KV path by running the REFERENCE's
own kernels (its sources compiled for sm_100a into oracle/_ref/libtvp_ref.so)
on a CUDA device, on seeded inputs from tests/workloads.py.

  rope.npz            ropeKernel (src/model/RoPe.cu) on 4096 consecutive K rows
                      (SHA-256 of all + 15 full rows), single rows at far
                      positions, and q-width (2048) rows.
  prefill_append.npz  rope(k) + storePagedKV for the prefill_append workload:
                      block tables, SHA-256 of both pools, request 0's RoPE'd K.
  decode_small.npz    gather + cuBLAS + softmax decode attention
                      (src/model/paged_transformer.cu:85-94) on decode_small.
  attention_pattern.npz  the same path on the closed-form inputs of the
                      reference's tests/paged_attention_test.cu.

Usage (on a GPU machine): python tests/golden/make_golden.py --out DIR
"""
from __future__ import annotations

import argparse
import ctypes
import hashlib
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path[:0] = [str(HERE.parent), str(HERE.parents[1])]

import oracle  # noqa: E402
import workloads as W  # noqa: E402

ROPE_ROWS = [0, 1, 2, 3, 15, 16, 17, 31, 32, 100, 1000, 2047, 2048, 2049, 4095]
FAR_POSITIONS = [8191, 8192, 16383, 32767]
Q_POSITIONS = [0, 5, 1000, 4095]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def host(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def i32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def rope_golden(ref):
    rng = np.random.default_rng(101)
    x = W.normal_bf16(rng, (4096, 512))
    d = dev(x)
    assert ref.ref_rope(vp(d), 4096, 512, 0) == 0
    out = host(d)
    far_in = W.normal_bf16(rng, (len(FAR_POSITIONS), 512))
    far = []
    for i, p in enumerate(FAR_POSITIONS):
        r = dev(far_in[i:i + 1])
        assert ref.ref_rope(vp(r), 1, 512, p) == 0
        far.append(host(r)[0])
    q_in = W.normal_bf16(rng, (len(Q_POSITIONS), 2048))
    qs = []
    for i, p in enumerate(Q_POSITIONS):
        r = dev(q_in[i:i + 1])
        assert ref.ref_rope(vp(r), 1, 2048, p) == 0
        qs.append(host(r)[0])
    return dict(seed=101, input_sha=sha(x), output_sha=sha(out), rows=np.array(ROPE_ROWS),
                row_values=out[ROPE_ROWS], far_positions=np.array(FAR_POSITIONS),
                far_input=far_in, far_values=np.stack(far), q_positions=np.array(Q_POSITIONS),
                q_input=q_in, q_values=np.stack(qs))


def prefill_golden(ref):
    case = W.prefill_append()
    R, T, P = case.k.shape[0], case.tokens, case.num_pages
    free = list(case.free_list)
    k_pool = torch.zeros((1, P, 16, 512), dtype=torch.bfloat16, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    tables, roped0 = [], None
    for r in range(R):
        table = np.array([free.pop() for _ in range(T // 16)], np.int32)
        tables.append(table)
        k = dev(case.k[r])
        v = dev(case.v[r])
        assert ref.ref_rope(vp(k), T, 512, 0) == 0
        assert ref.ref_store_paged_kv(vp(k_pool), vp(v_pool), P, 0, i32p(table), table.size, 0,
                                      vp(k), vp(v), T) == 0
        if r == 0:
            roped0 = host(k)
    return dict(seed=2, k_input_sha=sha(case.k), tables=np.stack(tables),
                k_pool_sha=sha(host(k_pool)), v_pool_sha=sha(host(v_pool)), roped_k0=roped0)


def decode_golden(ref, case):
    k = dev(case.k_pool)
    v = dev(case.v_pool)
    q = dev(case.q)
    out = torch.empty_like(q)
    tables = np.ascontiguousarray(case.tables, np.int32)
    lens = np.ascontiguousarray(case.lens, np.int32)
    rc = ref.ref_paged_decode(vp(q), vp(k), vp(v), case.num_pages, 0, i32p(tables), tables.shape[1],
                              i32p(lens), case.batch, vp(out), 0, 0, None)
    assert rc == 0
    return dict(lens=lens, tables=tables, q_sha=sha(case.q), k_sha=sha(case.k_pool),
                v_sha=sha(case.v_pool), out=host(out))


def pattern_case():
    lengths, q, k, v = W.reference_attention_pattern()
    tables = W.scattered_tables(np.random.default_rng(7), lengths, 8)
    k_pool = np.zeros((1, 8, 16, 512), np.uint16)
    v_pool = np.zeros((1, 8, 16, 512), np.uint16)
    for row, L in enumerate(lengths):
        oracle.store_paged(k_pool, v_pool, 0, tables[row], 0, k[row, :L], v[row, :L])
    return W.DecodeCase(lens=np.array(lengths, np.int32), tables=tables, num_pages=8,
                        num_layers=1, q=q, k_pool=k_pool, v_pool=v_pool)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    ref = oracle.load_reference()
    if ref is None:
        raise SystemExit("oracle/_ref/libtvp_ref.so is not built (make -C oracle ref)")
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out / "rope.npz", **rope_golden(ref))
    np.savez_compressed(out / "prefill_append.npz", **prefill_golden(ref))
    np.savez_compressed(out / "decode_small.npz", **decode_golden(ref, W.decode_small()))
    np.savez_compressed(out / "attention_pattern.npz", **decode_golden(ref, pattern_case()))
    print("golden vectors written to", out)


if __name__ == "__main__":
    main()
