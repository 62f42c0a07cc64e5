"""Multi-process host logic of the multi-GPU decode path, on CPU (gloo,
world size 2): request sharding covers every row exactly once and balances the
attended tokens; the bench's max-over-ranks timing reduction; KV-head
sharding's slices, all-gather and interleave reassemble the 8-head attention
(per-rank attention from the oracle)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
import workloads as W
from vllm_b200 import sharding


def test_request_shards_partition_and_balance():
    lens = W.sweep_lengths(4)
    for world in (1, 2, 4, 8):
        shards = sharding.shard_by_request(lens, world)
        allrows = np.concatenate(shards)
        assert sorted(allrows.tolist()) == list(range(lens.size))
        assert sharding.imbalance(lens, shards) < 1.0 + lens.max() / (lens.sum() / world)
        assert sharding.imbalance(lens, shards) < 1.01


def test_kv_head_shards():
    assert [list(r) for r in sharding.shard_by_kv_head(8)] == [[i] for i in range(8)]
    assert [list(r) for r in sharding.shard_by_kv_head(2)] == [[0, 1, 2, 3], [4, 5, 6, 7]]
    with pytest.raises(ValueError):
        sharding.shard_by_kv_head(3)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        lens = W.sweep_lengths(4)
        mine = sharding.shard_by_request(lens, world)[rank]
        # every rank derives the same partition on its own: gather and compare
        gathered = [None] * world
        dist.all_gather_object(gathered, mine.tolist())
        # bench timing reduction: max over ranks
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        results[rank] = (gathered, float(t.item()), int(lens[mine].sum()))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_partition_agreement_and_max_timing():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    g0, t0, load0 = results[0]
    g1, t1, load1 = results[1]
    assert g0 == g1
    rows = sorted(g0[0] + g0[1])
    assert rows == list(range(256))
    assert t0 == t1 == 11.0
    assert abs(load0 - load1) <= 8192


def test_head_slices_and_interleave_reassemble_the_oracle():
    """Single process: the oracle on each rank's head slice, interleaved,
    is bit-identical to the oracle on all 8 heads (heads are independent)."""
    case = W.decode_random(80, [300, 17, 129, 64])
    full = oracle.decode_attention(case.q, case.k_pool, case.v_pool, 0, case.tables, case.lens)
    for world in (1, 2, 4, 8):
        parts = []
        for heads in sharding.shard_by_kv_head(world):
            q = np.ascontiguousarray(sharding.slice_q_heads(case.q, heads))
            k = np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads))
            v = np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads))
            parts.append(oracle.decode_attention(q, k, v, 0, case.tables, case.lens))
        assert np.array_equal(sharding.interleave_head_shards(np.stack(parts)), full)


def _head_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        case = W.decode_random(81, [500, 33, 1, 260, 90])
        heads = sharding.shard_by_kv_head(world)[rank]
        q = np.ascontiguousarray(sharding.slice_q_heads(case.q, heads))
        k = np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads))
        v = np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads))
        mine = oracle.decode_attention(q, k, v, 0, case.tables, case.lens)
        local = torch.from_numpy(mine.view(np.int16)).view(torch.bfloat16)
        flat = torch.empty((world * 8, local.shape[1]), dtype=torch.bfloat16)  # room for B <= 8
        rows = sharding.all_gather_head_shards(local, flat)
        results[rank] = rows.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_head_sharded_gather():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_head_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    case = W.decode_random(81, [500, 33, 1, 260, 90])
    full = oracle.decode_attention(case.q, case.k_pool, case.v_pool, 0, case.tables, case.lens)
    assert np.array_equal(results[0], full)
    assert np.array_equal(results[1], full)


def _agree_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    from vllm_b200 import _native as N
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # the agreement step alone: no gather group was created on any rank
        dec = sharding.HeadShardedDecode.__new__(sharding.HeadShardedDecode)
        dec.dist, dec.group, dec.world, dec.rank, dec._h = dist, None, world, rank, None
        dec._agree(N.TVP_OK, "all ok", connected=False)
        try:
            dec._agree(N.TVP_ERR_RUNTIME if rank == 1 else N.TVP_OK, "setup", connected=False)
            results[rank] = "returned"
        except RuntimeError as e:
            results[rank] = str(e)
        dist.barrier()  # both ranks are still in step after the failure
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_gather_setup_failure_is_raised_on_every_rank():
    """A setup step that fails on one rank raises on all ranks, none of them
    left waiting in a collective."""
    from vllm_b200 import _native as N
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    procs = [ctx.Process(target=_agree_worker, args=(r, world, port, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want = f"setup failed on ranks {{1: {N.TVP_ERR_RUNTIME}}}"
    assert results[0] == want and results[1] == want
