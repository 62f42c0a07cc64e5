"""Parity of the KV-head-shard decode kernel (pools of 1, 2 or 4 KV heads) on
the GPU: against the oracle (the reference's decode semantics on the same
heads), across grids, page orders and lengths, and as the sharded deployment
of the model's 8 heads (each rank's heads, all-gathered, against the 8-head
oracle).  Tolerance as for the 8-head kernel: max-abs 1e-2 + rel 2e-2."""
import numpy as np
import pytest
import torch

import oracle
import workloads as W
from gpu_util import assert_close_bf16, dev_bf16, dev_i32, f32, host_bf16, run_decode
from vllm_b200 import _native as N
from vllm_b200 import ops, sharding

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2e-2


def oracle_out(case, layer=0):
    return oracle.decode_attention(case.q, case.k_pool, case.v_pool, layer, case.tables, case.lens)


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_random_lengths_match_oracle(kv_heads):
    rng = np.random.default_rng(40 + kv_heads)
    lens = rng.integers(1, 3000, size=24).astype(np.int32)
    case = W.decode_random(41 + kv_heads, lens, kv_heads=kv_heads, num_layers=2)
    for layer in (0, 1):
        out, err = run_decode(case, layer=layer)
        assert err == 0
        assert out.shape == (24, kv_heads * 256)
        assert_close_bf16(out, f32(oracle_out(case, layer)), ATOL, RTOL,
                          f"kv_heads={kv_heads} layer={layer}")


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
@pytest.mark.parametrize("lens", [
    [1], [2], [15, 16, 17], [31, 32, 33], [255, 256, 257], [1000, 3, 1, 48], [0, 5, 0, 40],
    [129] * 3 + [0] + [7] * 5,
])
def test_edge_lengths(kv_heads, lens):
    case = W.decode_random(50 + len(lens), lens, kv_heads=kv_heads)
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, f32(oracle_out(case)), ATOL, RTOL, f"{lens}")
    zero_rows = np.asarray(lens) == 0
    assert (out[zero_rows] == 0).all()


@pytest.mark.parametrize("kv_heads", [1, 4])
@pytest.mark.parametrize("ctas", [1, 3, 7, 148, 300, 1000])
def test_any_grid_gives_the_same_attention(kv_heads, ctas):
    """Split-K ranges of every size, pieces that start and end anywhere in a stage."""
    lens = [700, 33, 1, 4096, 250, 17, 1600]
    case = W.decode_random(60, lens, kv_heads=kv_heads)
    out, err = run_decode(case, num_ctas=ctas)
    assert err == 0
    assert_close_bf16(out, f32(oracle_out(case)), ATOL, RTOL, f"ctas={ctas}")


def test_page_permutation_is_bit_exact():
    """The arithmetic follows logical positions only: moving pages to other
    physical slots (tables permuted alike) changes no output bit."""
    case = W.decode_random(70, [900, 40, 2000, 129], kv_heads=2, slack_pages=20)
    out, err = run_decode(case)
    assert err == 0
    rng = np.random.default_rng(71)
    perm = rng.permutation(case.num_pages)
    inv = np.argsort(perm)
    moved = W.DecodeCase(lens=case.lens, tables=np.where(case.tables >= 0, inv[case.tables], -1)
                         .astype(np.int32), num_pages=case.num_pages, num_layers=1, q=case.q,
                         k_pool=case.k_pool[:, perm], v_pool=case.v_pool[:, perm])
    out2, err2 = run_decode(moved)
    assert err2 == 0
    assert np.array_equal(out, out2)


@pytest.mark.parametrize("kv_heads", [1, 2, 4])
def test_merge_is_identical_whichever_piece_arrives_last(kv_heads):
    """Sequence 0 spans ranges 0, 1 and most of 2 of 8 (32 pages each): its
    last arriver is sometimes a range's last piece (merged through shared
    memory) and sometimes not (merged in the page loop); the bits must not
    depend on which."""
    case = W.decode_random(91 + kv_heads, [95 * 16, 16, 160 * 16], kv_heads=kv_heads)
    ref, err = run_decode(case, num_ctas=8)
    assert err == 0
    assert_close_bf16(ref, f32(oracle_out(case)), ATOL, RTOL)
    for _ in range(30):
        out, err = run_decode(case, num_ctas=8)
        assert err == 0
        assert np.array_equal(out, ref)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharded_ranks_reassemble_the_8_head_attention(world):
    """The KV-head-sharded deployment, ranks emulated one after another on one
    GPU: rank r runs its heads' slice of the pools and q, and the interleaved
    slices equal the 8-head oracle (and the 8-head kernel within tolerance)."""
    lens = [3000, 129, 17, 1024, 640, 2]
    case = W.decode_random(80, lens)
    ref = oracle_out(case)
    full, err = run_decode(case)
    assert err == 0
    slices = []
    for heads in sharding.shard_by_kv_head(world):
        part = W.DecodeCase(lens=case.lens, tables=case.tables, num_pages=case.num_pages,
                            num_layers=1, q=np.ascontiguousarray(sharding.slice_q_heads(case.q, heads)),
                            k_pool=np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads)),
                            v_pool=np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads)))
        out, err = run_decode(part)
        assert err == 0
        slices.append(out)
    joined = sharding.interleave_head_shards(np.stack(slices))
    assert joined.shape == (len(lens), 2048)
    assert_close_bf16(joined, f32(ref), ATOL, RTOL, f"world={world}")
    assert_close_bf16(joined, f32(full), ATOL, RTOL, "vs 8-head kernel")


@pytest.mark.parametrize("kv_heads", [1, 2])
def test_compat_mode_on_head_shards(kv_heads):
    case = W.decode_random(90, [17, 64, 129, 256, 1000], kv_heads=kv_heads)
    out, err = run_decode(case, mode=N.TVP_MODE_COMPAT)
    assert err == 0
    e = f32(oracle_out(case))
    diff = np.abs(f32(out) - e)
    assert (diff <= np.maximum(np.abs(e) * 2.0 ** -7, 1e-3)).all()


def test_bad_page_sets_error_bit_and_stays_finite():
    case = W.decode_random(100, [300, 60], kv_heads=1)
    case.tables = case.tables.copy()
    case.tables[0, 3] = case.num_pages + 5
    out, err = run_decode(case)
    assert err & N.TVP_DEVERR_BAD_PAGE
    assert np.isfinite(f32(out)).all()


def test_plan_for_other_head_count_is_refused_on_device():
    """A workspace planned for 8 heads handed to a 4-head pool: the kernel
    finds the plan header's head count wrong and records BAD_PLAN."""
    case = W.decode_random(110, [100, 200], kv_heads=4)
    ws = ops.DecodeWorkspace(case.batch, "cuda", kv_heads=8)
    lens = dev_i32(case.lens)
    err = ops.new_error_word("cuda")
    ops.decode_plan(lens, case.tables.shape[1], ws, error=err)
    ws.kv_heads = 4  # bypass the host-side check to reach the device-side one
    ops.paged_decode_attention(dev_bf16(case.q), dev_bf16(case.k_pool), dev_bf16(case.v_pool), 0,
                               dev_i32(case.tables), lens, ws, error=err)
    torch.cuda.synchronize()
    assert int(err.item()) & N.TVP_DEVERR_BAD_PLAN


def test_workspace_head_count_checked_on_host():
    case = W.decode_random(111, [100], kv_heads=2)
    ws = ops.DecodeWorkspace(1, "cuda", kv_heads=8)
    lens = dev_i32(case.lens)
    ops.decode_plan(lens, case.tables.shape[1], ws)
    with pytest.raises(ValueError):
        ops.paged_decode_attention(dev_bf16(case.q), dev_bf16(case.k_pool), dev_bf16(case.v_pool),
                                   0, dev_i32(case.tables), lens, ws)


def test_long_context_one_head():
    """long_context on one KV head (the 8-GPU head shard): 16 x 32768 tokens."""
    case = W.decode_random(120, [32768] * 16, kv_heads=1, slack_pages=0)
    out, err = run_decode(case)
    assert err == 0
    assert_close_bf16(out, f32(oracle_out(case)), ATOL, RTOL, "long context, 1 head")
