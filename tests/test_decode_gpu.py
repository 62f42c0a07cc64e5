"""K2 parity on the GPU: the fused paged decode attention against the oracle
(CPU restatement of the reference), the reference's own gather+cuBLAS path
(built from its sources) and exact-arithmetic attention.

Tolerance of the FAST path (BF16 probabilities into P.V, FP32 everywhere else):
max-abs 1e-2 + rel 2e-2 against the reference semantics, the bar stated for
this path.  COMPAT keeps the reference's rounding points and is held to a
single BF16 ulp on at most a small fraction of outputs."""
import numpy as np
import pytest
import torch

import oracle
import workloads as W
from gpu_util import assert_close_bf16, dev_bf16, dev_i32, f32, host_bf16, run_decode
from vllm_b200 import _native as N
from vllm_b200 import ops

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2e-2


def oracle_out(case, layer=0):
    return oracle.decode_attention(case.q, case.k_pool, case.v_pool, layer, case.tables, case.lens)


def exact_out(case, layer=0):
    return oracle.decode_attention_f64(case.q, case.k_pool, case.v_pool, layer, case.tables,
                                       case.lens)


def test_decode_small_fast_matches_oracle_and_exact():
    case = W.decode_small()
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, f32(oracle_out(case)), ATOL, RTOL, "vs reference semantics")
    m = assert_close_bf16(out, exact_out(case), ATOL, RTOL, "vs exact")
    assert m < 8e-3


def test_decode_small_compat_matches_oracle_to_an_ulp():
    case = W.decode_small()
    out, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    ref = oracle_out(case)
    a, e = f32(out), f32(ref)
    diff = np.abs(a - e)
    # one BF16 ulp of the expected value (floor 1e-3 near zero)
    assert (diff <= np.maximum(np.abs(e) * 2.0 ** -7, 1e-3)).all()
    assert (diff > 0).mean() < 0.05


def test_reference_test_pattern_within_reference_tolerance():
    """tests/paged_attention_test.cu of the reference: lengths {16, 17, 33},
    closed-form q/k/v, output max-abs <= 5e-3 against the contiguous path."""
    lengths, q, k, v = W.reference_attention_pattern()
    rng = np.random.default_rng(7)
    num_pages = 8
    tables = W.scattered_tables(rng, lengths, num_pages)
    k_pool = np.zeros((1, num_pages, 16, 512), np.uint16)
    v_pool = np.zeros((1, num_pages, 16, 512), np.uint16)
    for row, L in enumerate(lengths):
        oracle.store_paged(k_pool, v_pool, 0, tables[row], 0, k[row, :L], v[row, :L])
    case = W.DecodeCase(lens=np.array(lengths, np.int32), tables=tables, num_pages=num_pages,
                        num_layers=1, q=q, k_pool=k_pool, v_pool=v_pool)
    out, err = run_decode(case)
    assert err == 0
    exact = exact_out(case)
    assert np.abs(f32(out) - exact).max() <= 5e-3
    compat, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    assert np.abs(f32(compat) - exact).max() <= 5e-3


@pytest.mark.parametrize("lens", [
    [1], [2], [15, 16, 17], [31, 32, 33], [255, 256, 257], [1000, 3, 1, 48],
    [0, 5, 0, 40],
])
def test_edge_lengths(lens):
    case = W.decode_random(11 + len(lens), lens)
    out, err = run_decode(case)
    assert err == 0
    exact = exact_out(case)
    assert_close_bf16(out, exact, ATOL, RTOL, f"lens={lens}")
    for b, L in enumerate(lens):
        if L == 0:
            assert (out[b] == 0).all()


@pytest.mark.parametrize("num_ctas", [1, 3, 7, 148, 300, 1000])
def test_split_k_partition_invariance(num_ctas):
    """The output does not depend on how the flattened page range is cut
    (1000 CTAs > 407 pages: only as many CTAs as pages take work)."""
    case = W.decode_random(21, [700, 33, 1500, 16, 4096, 129])
    out, err = run_decode(case, num_ctas=num_ctas)
    assert err == 0
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, f"ctas={num_ctas}")


def test_page_permutation_gives_identical_bits():
    """Moving every page to another physical slot changes no output bit."""
    case = W.decode_random(31, [300, 17, 900, 64])
    out1, _ = run_decode(case)
    rng = np.random.default_rng(5)
    perm = rng.permutation(case.num_pages)
    k2 = np.empty_like(case.k_pool)
    v2 = np.empty_like(case.v_pool)
    k2[:, perm] = case.k_pool
    v2[:, perm] = case.v_pool
    tables2 = np.where(case.tables >= 0, perm[np.maximum(case.tables, 0)], -1).astype(np.int32)
    case2 = W.DecodeCase(lens=case.lens, tables=tables2, num_pages=case.num_pages, num_layers=1,
                         q=case.q, k_pool=k2, v_pool=v2)
    out2, _ = run_decode(case2)
    assert np.array_equal(out1, out2)


def racing_last_arrivers_case(seed, kv_heads=8):
    """8 ranges of 32 pages: sequence 0 fills ranges 0 and 1 and 31 pages of
    range 2 (whose last page starts sequence 1), so its three pieces finish at
    about the same time and its last arriver is sometimes a range's last piece
    (merged through shared memory) and sometimes not (merged in the loop)."""
    return W.decode_random(seed, [95 * 16, 16, 160 * 16], kv_heads=kv_heads)


def test_merge_is_identical_whichever_piece_arrives_last():
    case = racing_last_arrivers_case(90)
    ref, err = run_decode(case, num_ctas=8)
    assert err == 0
    assert_close_bf16(ref, exact_out(case), ATOL, RTOL)
    for _ in range(30):
        out, err = run_decode(case, num_ctas=8)
        assert err == 0
        assert np.array_equal(out, ref)


def test_attention_right_after_append_sees_the_new_token():
    """The decode attention starts while the append before it in the stream
    is still running (programmatic dependent launch).  The new token is built
    to dominate every head's attention (old keys near zero, its key along the
    query) with value +5, and its slot holds -5 before each append: an
    attention that copied the last page too early would return about -5."""
    rng = np.random.default_rng(77)
    lens = np.array([130, 17, 1, 500, 16, 33], np.int32)
    case = W.decode_random(78, lens.tolist())
    k_pool = (dev_bf16(case.k_pool).float() * 0.01).to(torch.bfloat16)
    v_pool = dev_bf16(case.v_pool)
    tables = dev_i32(case.tables)
    lens_d = dev_i32(lens)
    pos = dev_i32(lens - 1)
    B = len(lens)
    ws = ops.DecodeWorkspace(B, "cuda")
    err = ops.new_error_word("cuda")
    ops.decode_plan(lens_d, case.tables.shape[1], ws, error=err)
    q = dev_bf16(W.normal_bf16(rng, (B, 2048)))
    # each KV head's new key: 64 x the mean of its 4 query heads, not rotated
    # (scores of 24 and more against ~0 for up to 499 old keys)
    k_new = (q.float().view(B, 8, 4, 64).mean(dim=2) * 64).reshape(B, 512).to(torch.bfloat16)
    v_new = torch.full((B, 512), 5.0, dtype=torch.bfloat16, device="cuda")
    rows = torch.arange(B, device="cuda")
    page = tables.long()[rows, (pos // 16).long()]
    slot = (pos % 16).long()
    out = torch.empty_like(q)
    for it in range(20):
        v_pool[0, page, slot] = -5.0  # stale contents of the new token's slot
        k_pool[0, page, slot] = k_new
        ops.rope_append(k_pool, v_pool, 0, tables, pos, k_new.clone(), v_new, rope_k=False,
                        writeback_k=False, error=err)
        ops.paged_decode_attention(q, k_pool, v_pool, 0, tables, lens_d, ws, out=out, error=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        o = out.float()
        assert (o > 4.5).all(), f"iteration {it}: min {o.min().item():.3f} (stale slot read?)"
    exact = oracle.decode_attention_f64(host_bf16(q), host_bf16(k_pool), host_bf16(v_pool), 0,
                                        case.tables, lens)
    assert_close_bf16(host_bf16(out), exact, ATOL, RTOL, "after append")


def test_stale_slots_past_the_length_never_leak():
    """NaN/Inf bit patterns in unused slots of a row's last page are ignored."""
    case = W.decode_random(41, [17, 40, 1, 250])
    for b, L in enumerate(case.lens):
        last = case.tables[b, (L - 1) // 16]
        slot0 = L % 16
        if slot0:
            case.k_pool[0, last, slot0:] = 0x7FC0  # NaN
            case.v_pool[0, last, slot0:] = 0x7F80  # +Inf
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, "stale slots")


def test_layer_offset_selects_the_right_slice():
    case = W.decode_random(51, [64, 200], num_layers=3)
    for layer in range(3):
        out, err = run_decode(case, layer=layer)
        assert err == 0
        assert_close_bf16(out, exact_out(case, layer), ATOL, RTOL, f"layer {layer}")


def test_bad_page_id_is_reported_not_faulted():
    case = W.decode_random(61, [40, 40])
    case.tables[1, 1] = case.num_pages + 5  # out of range
    out, err = run_decode(case)
    assert err & N.TVP_DEVERR_BAD_PAGE
    # the healthy row is unaffected
    exact = exact_out(W.DecodeCase(lens=case.lens[:1], tables=case.tables[:1],
                                   num_pages=case.num_pages, num_layers=1, q=case.q[:1],
                                   k_pool=case.k_pool, v_pool=case.v_pool))
    assert_close_bf16(out[:1], exact, ATOL, RTOL, "healthy row")


def test_plan_mismatch_is_reported():
    case = W.decode_random(71, [64, 64, 64])
    ws = ops.DecodeWorkspace(4, "cuda")
    lens2 = dev_i32(case.lens[:2])
    ops.decode_plan(lens2, case.tables.shape[1], ws)
    ws.batch = 3  # pretend: the plan was made for 2 rows
    err = ops.new_error_word("cuda")
    ops.paged_decode_attention(dev_bf16(case.q), dev_bf16(case.k_pool), dev_bf16(case.v_pool), 0,
                               dev_i32(case.tables), dev_i32(case.lens), ws, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) & N.TVP_DEVERR_BAD_PLAN


@pytest.mark.parametrize("kv_heads", [8, 1])
def test_batch_beyond_one_plan_block(kv_heads):
    """3000 ragged rows (empty, one-page and multi-page rows, a few long ones):
    the plan's prefix scan runs over three 1024-row blocks with a carry, most
    CTAs hold many whole sequences and the split-K slots and counters are
    indexed far past the first block."""
    rng = np.random.default_rng(5)
    lens = rng.integers(0, 120, size=3000).astype(np.int32)
    lens[rng.choice(3000, 6, replace=False)] = [5000, 3000, 2048, 1025, 16, 17]
    lens[::97] = 0
    case = W.decode_random(23, lens, kv_heads=kv_heads)
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, f"3000 rows, kv_heads={kv_heads}")
    assert (out[lens == 0] == 0).all()


def test_long_context_rows():
    case = W.decode_random(81, [32768, 20000, 5])
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, "long context")


def test_sweep_sample_rows():
    lens = W.sweep_lengths(4, batch=48)
    case = W.decode_random(91, lens)
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, "sweep sample")
    # COMPAT on the same rows (up to 8192 tokens: two 4096-token chunks)
    compat, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    assert_close_bf16(compat, exact_out(case), ATOL, RTOL, "sweep sample compat")


@pytest.mark.parametrize("lens", [[32768, 20000, 5], [4096, 4097, 8191, 8192, 12289, 1]])
def test_compat_rows_beyond_one_chunk_match_oracle_to_an_ulp(lens):
    """COMPAT sums rows longer than its 4096-token shared-memory chunk chunk by
    chunk, in the reference's pairwise-tree order over the whole row: against
    the oracle (the same tree over the whole row, computed on the CPU) it stays
    within one BF16 ulp on a small fraction of outputs, as on short rows."""
    case = W.decode_random(95 + len(lens), lens)
    out, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    a, e = f32(out), f32(oracle_out(case))
    diff = np.abs(a - e)
    assert (diff <= np.maximum(np.abs(e) * 2.0 ** -7, 1e-3)).all()
    assert (diff > 0).mean() < 0.05
    assert_close_bf16(out, exact_out(case), ATOL, RTOL, "compat long rows vs exact")


def test_fast_path_agrees_with_reference_gather_cublas(ref_lib):
    """The reference's own decode (gather + cuBLAS + softmax), built from its
    sources, on the single-layer decode workload."""
    import ctypes
    case = W.decode_small()
    k = dev_bf16(case.k_pool)
    v = dev_bf16(case.v_pool)
    q = dev_bf16(case.q)
    ref_out = torch.empty_like(q)
    tables = np.ascontiguousarray(case.tables, np.int32)
    lens = np.ascontiguousarray(case.lens, np.int32)
    rc = ref_lib.ref_paged_decode(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
        case.num_pages, 0, tables.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), tables.shape[1],
        lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), case.batch,
        ctypes.c_void_p(ref_out.data_ptr()), 0, 0, None)
    assert rc == 0
    ref_bits = host_bf16(ref_out)
    ours, err = run_decode(case)
    assert err == 0
    assert_close_bf16(ours, f32(ref_bits), ATOL, RTOL, "FAST vs reference gather+cuBLAS")
    # the oracle (CPU restatement) agrees with the reference to within its unpinned GEMV order
    assert_close_bf16(oracle_out(case), f32(ref_bits), 4e-3, 1e-2, "oracle vs reference")
    compat, _ = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert_close_bf16(compat, f32(ref_bits), 4e-3, 1e-2, "COMPAT vs reference")
