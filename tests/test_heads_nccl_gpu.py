"""KV-head-sharded decode over NCCL, one process per GPU (2 to 8 GPUs; skipped
with fewer): every rank holds its KV heads of the same pages, runs the fused
decode on them and all-gathers; each rank's reassembled rows must equal the
8-head oracle within the decode tolerance (max-abs 1e-2 + rel 2e-2), and all
ranks must hold identical rows."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [3000, 129, 17, 1024, 640, 2, 0, 5000]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, results):
    import datetime
    import torch.distributed as dist

    import workloads as W
    from gpu_util import dev_bf16, dev_i32, host_bf16
    from vllm_b200 import ops, sharding

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        case = W.decode_random(80, LENS)
        heads = sharding.shard_by_kv_head(world)[rank]
        dec = sharding.HeadShardedDecode(len(LENS), device="cuda")
        lens = dev_i32(case.lens)
        err = ops.new_error_word("cuda")
        dec.plan(lens, case.tables.shape[1], error=err)
        rows = dec.attend(dev_bf16(np.ascontiguousarray(sharding.slice_q_heads(case.q, heads))),
                          dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads))),
                          dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads))),
                          0, dev_i32(case.tables), lens, error=err)
        torch.cuda.synchronize()
        results[rank] = (host_bf16(rows), int(err.item()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 or more GPUs")
def test_head_sharded_decode_over_nccl():
    import torch.multiprocessing as mp

    import oracle
    import workloads as W
    from gpu_util import assert_close_bf16, f32

    world = 8 if torch.cuda.device_count() >= 8 else (4 if torch.cuda.device_count() >= 4 else 2)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    case = W.decode_random(80, LENS)
    ref = oracle.decode_attention(case.q, case.k_pool, case.v_pool, 0, case.tables, case.lens)
    rows0, err0 = results[0]
    assert err0 == 0
    assert_close_bf16(rows0, f32(ref), 1e-2, 2e-2, f"world={world}")
    for r in range(1, world):
        assert results[r][1] == 0
        assert np.array_equal(results[r][0], rows0)
