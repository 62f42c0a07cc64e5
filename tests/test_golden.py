"""Golden vectors: outputs of the REFERENCE's own kernels (its sources built for
sm_100a, run on a B200 by tests/golden/make_golden.py) on seeded inputs.

CPU tests pin the oracle to them (page placement and allocation bit-exact,
RoPE within one BF16 ulp of the device libm, attention within the unpinned
cuBLAS GEMV order); GPU tests pin the CUDA path (RoPE and pages bit-exact,
attention within the path's tolerance)."""
import hashlib
from pathlib import Path

import numpy as np
import pytest

import oracle
import workloads as W
from oracle import allocator as OA

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


def ulps(a, b):
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


def rope_input():
    g = load("rope")
    x = W.normal_bf16(np.random.default_rng(int(g["seed"])), (4096, 512))
    assert sha(x) == str(g["input_sha"]), "seeded generator no longer reproduces the fixture input"
    return g, x


def pattern_case():
    lengths, q, k, v = W.reference_attention_pattern()
    tables = W.scattered_tables(np.random.default_rng(7), lengths, 8)
    k_pool = np.zeros((1, 8, 16, 512), np.uint16)
    v_pool = np.zeros((1, 8, 16, 512), np.uint16)
    for row, L in enumerate(lengths):
        oracle.store_paged(k_pool, v_pool, 0, tables[row], 0, k[row, :L], v[row, :L])
    return W.DecodeCase(lens=np.array(lengths, np.int32), tables=tables, num_pages=8,
                        num_layers=1, q=q, k_pool=k_pool, v_pool=v_pool)


def checked_case(name):
    g = load(name)
    case = W.decode_small() if name == "decode_small" else pattern_case()
    assert sha(case.q) == str(g["q_sha"]) and sha(case.k_pool) == str(g["k_sha"])
    assert sha(case.v_pool) == str(g["v_sha"])
    assert np.array_equal(case.tables, g["tables"]) and np.array_equal(case.lens, g["lens"])
    return g, case


# ------------------------------------------------------------------ CPU ---
def test_oracle_rope_against_reference_kernel():
    g, x = rope_input()
    rows = g["rows"]
    got = oracle.rope(x[rows], positions=rows.astype(np.int32))
    ok, stats = oracle.rope_close(got, g["row_values"], x[rows])  # positions <= 4095
    assert ok, stats
    # positions 8191..32767: pos * theta amplifies a last-bit difference of powf,
    # so more elements differ, all still within one ulp at the input scale
    far = np.concatenate([oracle.rope(g["far_input"][i:i + 1], position_offset=int(p))
                          for i, p in enumerate(g["far_positions"])])
    ok, stats = oracle.rope_close(far, g["far_values"], g["far_input"], max_mismatch_frac=0.05)
    assert ok, stats
    qs = np.concatenate([oracle.rope(g["q_input"][i:i + 1], position_offset=int(p))
                         for i, p in enumerate(g["q_positions"])])
    ok, stats = oracle.rope_close(qs, g["q_values"], g["q_input"], max_mismatch_frac=0.01)
    assert ok, stats


def test_oracle_prefill_pages_and_allocation_against_reference():
    g = load("prefill_append")
    case = W.prefill_append()
    assert sha(case.k) == str(g["k_input_sha"])
    # allocation: the reference LIFO on the shuffled free list
    ocache = OA.OracleCache(case.num_pages)
    ocache.free_blocks = list(case.free_list)
    tables = []
    for r in range(case.k.shape[0]):
        s = OA.OracleSequence()
        OA.reserve_sequence_blocks(ocache, s, case.tokens)
        tables.append(s.block_table)
    assert np.array_equal(np.array(tables, np.int32), g["tables"])
    # V pages (no RoPE): placement bit-exact
    kp = np.zeros((1, case.num_pages, 16, 512), np.uint16)
    vp = np.zeros_like(kp)
    for r in range(case.k.shape[0]):
        oracle.store_paged(kp, vp, 0, g["tables"][r], 0, case.k[r], case.v[r])
    assert sha(vp) == str(g["v_pool_sha"])
    # K pages: RoPE through the libm restatement, checked on request 0
    ok, stats = oracle.rope_close(oracle.rope(case.k[0], position_offset=0), g["roped_k0"],
                                  case.k[0])
    assert ok, stats


@pytest.mark.parametrize("name", ["decode_small", "attention_pattern"])
def test_oracle_attention_against_reference_gather_cublas(name):
    g, case = checked_case(name)
    got = oracle.decode_attention(case.q, case.k_pool, case.v_pool, 0, case.tables, case.lens)
    a, e = W.bf16_to_f32(got), W.bf16_to_f32(g["out"])
    err = np.abs(a - e)
    assert (err <= 4e-3 + 1e-2 * np.abs(e)).all(), err.max()
    # most outputs agree to the bit: only the GEMV summation order is unpinned
    assert (got == g["out"]).mean() > 0.9


# ------------------------------------------------------------------ GPU ---
@pytest.mark.gpu
def test_cuda_rope_bit_exact_against_reference_kernel():
    import torch
    from gpu_util import dev_bf16, dev_i32, host_bf16
    from vllm_b200 import ops
    g, x = rope_input()
    T = x.shape[0]
    k = dev_bf16(x)
    kp = torch.zeros((1, T // 16, 16, 512), dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    ops.rope_append(kp, vp, 0, dev_i32(np.arange(T // 16)[None]), dev_i32(np.arange(T)), k,
                    dev_bf16(x), token_seq=torch.zeros(T, dtype=torch.int32, device="cuda"))
    assert sha(host_bf16(k)) == str(g["output_sha"])
    for i, p in enumerate(g["far_positions"]):
        kk = dev_bf16(g["far_input"][i:i + 1])
        kpp = torch.zeros((1, int(p) // 16 + 1, 16, 512), dtype=torch.bfloat16, device="cuda")
        ops.rope_append(kpp, torch.zeros_like(kpp), 0,
                        dev_i32(np.arange(int(p) // 16 + 1)[None]), dev_i32([int(p)]), kk,
                        dev_bf16(g["far_input"][i:i + 1]), token_seq=dev_i32([0]))
        assert np.array_equal(host_bf16(kk), g["far_values"][i:i + 1])


@pytest.mark.gpu
def test_cuda_prefill_pages_bit_exact_against_reference():
    import torch
    from gpu_util import dev_bf16, dev_i32, host_bf16
    from vllm_b200 import ops
    g = load("prefill_append")
    case = W.prefill_append()
    kp = torch.zeros((1, case.num_pages, 16, 512), dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    T = case.tokens
    for r in range(case.k.shape[0]):
        k = dev_bf16(case.k[r])
        ops.rope_append(kp, vp, 0, dev_i32(g["tables"][r:r + 1]), dev_i32(np.arange(T)), k,
                        dev_bf16(case.v[r]), token_seq=torch.zeros(T, dtype=torch.int32, device="cuda"))
        if r == 0:
            assert np.array_equal(host_bf16(k), g["roped_k0"])
    assert sha(host_bf16(kp)) == str(g["k_pool_sha"])
    assert sha(host_bf16(vp)) == str(g["v_pool_sha"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["decode_small", "attention_pattern"])
def test_cuda_attention_against_reference_gather_cublas(name):
    from gpu_util import assert_close_bf16, run_decode
    from vllm_b200 import _native as N
    g, case = checked_case(name)
    expect = W.bf16_to_f32(g["out"])
    fast, err = run_decode(case)
    assert err == 0
    assert_close_bf16(fast, expect, 1e-2, 2e-2, "FAST vs reference")
    compat, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    assert_close_bf16(compat, expect, 4e-3, 1e-2, "COMPAT vs reference")
    assert (compat == g["out"]).mean() > 0.9
