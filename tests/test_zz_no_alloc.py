"""tvp_paged_decode_attention_noalloc: decode attention for callers that cannot
call cudaMalloc (device memory owned by a host framework's pool, a fixed memory
budget, or a thread that must not take cudaMalloc's device-wide
synchronisation).  Its workspace is a fixed 4 MiB device array inside the
library, so the call allocates nothing.

Checked through the C-ABI against the workspace-taking entry point
(tvp_paged_decode_attention, FAST mode) on two calls in a row, within the
tolerance the other decode tests use (1e-2 abs + 2e-2 rel).  This file is
collected last so that a run stopping at its first failure has already run
every other test; it needs nothing from them."""
import ctypes

import numpy as np
import pytest
import torch

import workloads as W
from gpu_util import assert_close_bf16, dev_bf16, dev_i32, f32, host_bf16, run_decode
from vllm_b200 import _native as N
from vllm_b200 import ops

pytestmark = pytest.mark.gpu


def _noalloc(q, k_pool, v_pool, tables, lens, out, err, num_ctas=0):
    lib = N.load()
    num_layers, num_pages = k_pool.shape[0], k_pool.shape[1]
    kv_heads = k_pool.shape[3] // 64
    return lib.tvp_paged_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k_pool.data_ptr()),
        ctypes.c_void_p(v_pool.data_ptr()), num_pages, num_layers, 0, kv_heads, 4 * kv_heads,
        ctypes.c_void_p(tables.data_ptr()), tables.shape[1], ctypes.c_void_p(lens.data_ptr()),
        lens.numel(), 0.125, num_ctas, ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("kv_heads,lens", [(8, [700, 33, 1500, 16, 4096, 129, 1]),
                                           (8, [17, 64, 129, 256]),
                                           (4, [900, 17, 2500, 64, 1])])
def test_noalloc_matches_workspace_entry_point_on_two_calls(kv_heads, lens):
    case = W.decode_random(123 + len(lens), lens, kv_heads=kv_heads)
    expected, err_bits = run_decode(case)  # tvp_decode_plan + tvp_paged_decode_attention
    assert err_bits == 0
    q, k, v = dev_bf16(case.q), dev_bf16(case.k_pool), dev_bf16(case.v_pool)
    tables, seq_lens = dev_i32(case.tables), dev_i32(case.lens)
    err = ops.new_error_word("cuda")
    for call in range(2):
        out = torch.full_like(q, float("nan"))  # every output element must be written
        rc = _noalloc(q, k, v, tables, seq_lens, out, err)
        torch.cuda.synchronize()
        assert rc == N.TVP_OK, f"call {call}: {N.load().tvp_strerror(rc)}"
        assert int(err.item()) == 0
        assert_close_bf16(host_bf16(out), f32(expected), 1e-2, 2e-2, f"no-alloc call {call}")


def test_noalloc_rejects_a_batch_beyond_its_fixed_workspace():
    q = torch.zeros((1, 2048), dtype=torch.bfloat16, device="cuda")
    pool = torch.zeros((1, 1, 16, 512), dtype=torch.bfloat16, device="cuda")
    tables = torch.zeros((1, 1), dtype=torch.int32, device="cuda")
    err = ops.new_error_word("cuda")
    lib = N.load()
    huge = 200_000  # needs ~9 MB of workspace, more than the 4 MiB array
    rc = lib.tvp_paged_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(pool.data_ptr()),
        ctypes.c_void_p(pool.data_ptr()), 1, 1, 0, 8, 32, ctypes.c_void_p(tables.data_ptr()), 1,
        ctypes.c_void_p(tables.data_ptr()), huge, 0.125, 0, ctypes.c_void_p(q.data_ptr()),
        ctypes.c_void_p(err.data_ptr()), None)
    assert rc == N.TVP_ERR_WORKSPACE
    assert lib.tvp_decode_workspace_bytes(huge, 8, 0) > 4 << 20


def test_rejected_call_enqueues_nothing():
    """A call refused by an argument check (here: no output buffer) returns
    before the plan is enqueued: the error word stays clear and the next valid
    call still matches the workspace entry point."""
    case = W.decode_random(140, [300, 45, 1000])
    expected, _ = run_decode(case)
    q, k, v = dev_bf16(case.q), dev_bf16(case.k_pool), dev_bf16(case.v_pool)
    tables, seq_lens = dev_i32(case.tables), dev_i32(case.lens)
    err = ops.new_error_word("cuda")
    lib = N.load()
    rc = lib.tvp_paged_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), k.shape[1], k.shape[0], 0, 8, 32,
        ctypes.c_void_p(tables.data_ptr()), tables.shape[1], ctypes.c_void_p(seq_lens.data_ptr()),
        seq_lens.numel(), 0.125, 0, None, ctypes.c_void_p(err.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == N.TVP_ERR_INVALID_ARGUMENT
    assert int(err.item()) == 0
    out = torch.full_like(q, float("nan"))
    assert _noalloc(q, k, v, tables, seq_lens, out, err) == N.TVP_OK
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert_close_bf16(host_bf16(out), f32(expected), 1e-2, 2e-2, "no-alloc after a rejected call")
