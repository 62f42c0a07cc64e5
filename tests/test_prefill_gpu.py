"""K3 parity on the GPU: paged causal prefill attention against the oracle
(the reference's prefill semantics per query token) and against the
reference's own contiguous prefill path (computeAttentionScores, causalMask,
softmaxRows, attentionScoresTimesV, built from its sources).  Tolerance as for
the FAST decode: max-abs 1e-2 + rel 2e-2."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import workloads as W
from gpu_util import assert_close_bf16, dev_bf16, dev_i32, f32, host_bf16
from vllm_b200 import _native as N
from vllm_b200 import ops

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2e-2


def make_case(seed, prompts, context=None, kv_heads=8, num_layers=1, slack_pages=3):
    """Pools and tables holding context + prompt tokens of every sequence, and
    the prompt's queries."""
    context = list(context) if context is not None else [0] * len(prompts)
    total = [c + n for c, n in zip(context, prompts)]
    case = W.decode_random(seed, total, kv_heads=kv_heads, num_layers=num_layers,
                           slack_pages=slack_pages)
    q = W.normal_bf16(np.random.default_rng(seed + 1), (sum(prompts), kv_heads * 256))
    cu_q = np.concatenate([[0], np.cumsum(prompts)]).astype(np.int32)
    return case, q, cu_q, np.asarray(context, np.int32)


def run_prefill(case, q, cu_q, q_pos0, layer=0, tables=None):
    err = ops.new_error_word("cuda")
    out = ops.paged_prefill_attention(
        dev_bf16(q), dev_bf16(case.k_pool), dev_bf16(case.v_pool), layer,
        dev_i32(case.tables if tables is None else tables), dev_i32(cu_q), dev_i32(q_pos0),
        int(np.diff(cu_q).max()), error=err)
    torch.cuda.synchronize()
    return host_bf16(out), int(err.item())


def expected(case, q, cu_q, q_pos0, layer=0):
    return f32(oracle.prefill_attention(q, case.k_pool, case.v_pool, layer, case.tables, cu_q,
                                        q_pos0))


@pytest.mark.parametrize("prompts", [[1], [16], [17], [1, 17, 128, 300], [15, 16, 33, 64]])
def test_prompts_match_oracle(prompts):
    case, q, cu_q, pos0 = make_case(11, prompts)
    out, err = run_prefill(case, q, cu_q, pos0)
    assert err == 0
    assert_close_bf16(out, expected(case, q, cu_q, pos0), ATOL, RTOL, f"{prompts}")


def test_chunked_prefill_after_cached_context():
    """Chunks that start after L0 cached tokens attend the cache too."""
    case, q, cu_q, pos0 = make_case(12, [200, 1, 64, 16], context=[1000, 16, 0, 33])
    out, err = run_prefill(case, q, cu_q, pos0)
    assert err == 0
    assert_close_bf16(out, expected(case, q, cu_q, pos0), ATOL, RTOL, "chunked")


def test_prompt_beyond_the_reference_cap():
    """The reference's prefill stops at 1024 tokens (softmaxRows, causalMask)."""
    case, q, cu_q, pos0 = make_case(13, [2048])
    out, err = run_prefill(case, q, cu_q, pos0)
    assert err == 0
    assert_close_bf16(out, expected(case, q, cu_q, pos0), ATOL, RTOL, "2048-token prompt")


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_head_shard_pools(kv_heads):
    case, q, cu_q, pos0 = make_case(14, [100, 37], context=[20, 0], kv_heads=kv_heads)
    out, err = run_prefill(case, q, cu_q, pos0)
    assert err == 0
    assert out.shape == (137, kv_heads * 256)
    assert_close_bf16(out, expected(case, q, cu_q, pos0), ATOL, RTOL, f"kv_heads={kv_heads}")


def test_second_layer_of_the_pool():
    case, q, cu_q, pos0 = make_case(15, [50, 90], num_layers=2)
    out, err = run_prefill(case, q, cu_q, pos0, layer=1)
    assert err == 0
    assert_close_bf16(out, expected(case, q, cu_q, pos0, layer=1), ATOL, RTOL, "layer 1")


def test_stale_nan_slots_are_ignored():
    """Slots of the last page past the last position hold NaN: no effect."""
    case, q, cu_q, pos0 = make_case(16, [21, 40])
    want = expected(case, q, cu_q, pos0)
    k, v = case.k_pool.copy(), case.v_pool.copy()
    for s, n in enumerate([21, 40]):
        last_page = case.tables[s, (n - 1) // 16]
        k[0, last_page, n % 16 or 16:] = 0x7FC0
        v[0, last_page, n % 16 or 16:] = 0x7FC0
    poisoned = W.DecodeCase(lens=case.lens, tables=case.tables, num_pages=case.num_pages,
                            num_layers=1, q=case.q, k_pool=k, v_pool=v)
    out, err = run_prefill(poisoned, q, cu_q, pos0)
    assert err == 0
    assert_close_bf16(out, want, ATOL, RTOL, "NaN in stale slots")


def test_bad_page_is_reported_not_faulted():
    case, q, cu_q, pos0 = make_case(17, [70])
    tables = case.tables.copy()
    tables[0, 2] = case.num_pages + 3
    out, err = run_prefill(case, q, cu_q, pos0, tables=tables)
    assert err & N.TVP_DEVERR_BAD_PAGE
    assert np.isfinite(f32(out)).all()


def test_matches_the_reference_contiguous_prefill(ref_lib):
    """The reference's own prefill attention over the same K/V (gathered from
    the pages into its contiguous [n][512] buffers) and the same q."""
    n = 300
    case, q, cu_q, pos0 = make_case(18, [n])
    pages = case.tables[0, :(n + 15) // 16]
    k = case.k_pool[0, pages].reshape(-1, 512)[:n]
    v = case.v_pool[0, pages].reshape(-1, 512)[:n]
    dq, dk, dv = dev_bf16(q), dev_bf16(np.ascontiguousarray(k)), dev_bf16(np.ascontiguousarray(v))
    ref_out = torch.empty_like(dq)
    vp = lambda t: ctypes.c_void_p(t.data_ptr())
    assert ref_lib.ref_prefill_attention(vp(dq), vp(dk), vp(dv), n, vp(ref_out), 0, 0, None) == 0
    ref = f32(host_bf16(ref_out))
    out, err = run_prefill(case, q, cu_q, pos0)
    assert err == 0
    assert_close_bf16(out, ref, ATOL, RTOL, "vs reference contiguous path")
    # and the oracle restates that path
    assert_close_bf16(host_bf16(ref_out), expected(case, q, cu_q, pos0), 4e-3, 1e-2,
                      "oracle vs reference")
