"""KV-head-sharded decode, one process per GPU (2 to 8 GPUs; skipped with
fewer): every rank holds its KV heads of the same pages and gets the model's
[B, 2048] attention rows, either through the all-gather fused into the decode
kernel (mode p2p: stores into every rank's rows over NVLink, then a bounded
wait) or through an NCCL all-gather (mode nccl).  Three layers in a row, so the
p2p mode alternates its two row buffers.  Each rank's rows must equal the
8-head oracle within the decode tolerance (max-abs 1e-2 + rel 2e-2), and all
ranks must hold identical rows."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [3000, 129, 17, 1024, 640, 2, 0, 5000]
LAYERS = 3


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _layer_q(layer):
    import workloads as W
    return W.normal_bf16(np.random.default_rng(1000 + layer), (len(LENS), W.Q_DIM))


def _rank_main(rank, world, port, mode, results):
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
        case = W.decode_random(80, LENS, num_layers=LAYERS)
        heads = sharding.shard_by_kv_head(world)[rank]
        dec = sharding.HeadShardedDecode(len(LENS), device="cuda", mode=mode)
        lens = dev_i32(case.lens)
        tables = dev_i32(case.tables)
        kp = dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads)))
        vp = dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads)))
        err = ops.new_error_word("cuda")
        dec.plan(lens, case.tables.shape[1], error=err)
        outs = []
        for layer in range(LAYERS):
            q = dev_bf16(np.ascontiguousarray(sharding.slice_q_heads(_layer_q(layer), heads)))
            rows = dec.attend(q, kp, vp, layer, tables, lens, error=err)
            outs.append(host_bf16(rows))
        torch.cuda.synchronize()
        results[rank] = (outs, int(err.item()))
        dec.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 or more GPUs")
@pytest.mark.parametrize("mode", ["p2p", "nccl"])
def test_head_sharded_decode_multi_gpu(mode):
    import torch.multiprocessing as mp

    import oracle
    import workloads as W
    from gpu_util import assert_close_bf16, f32

    world = 8 if torch.cuda.device_count() >= 8 else (4 if torch.cuda.device_count() >= 4 else 2)
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    case = W.decode_random(80, LENS, num_layers=LAYERS)
    outs0, err0 = results[0]
    assert err0 == 0
    for layer in range(LAYERS):
        ref = oracle.decode_attention(_layer_q(layer), case.k_pool, case.v_pool, layer, case.tables,
                                      case.lens)
        assert_close_bf16(outs0[layer], f32(ref), 1e-2, 2e-2, f"{mode} world={world} layer={layer}")
    for r in range(1, world):
        outs, err = results[r]
        assert err == 0
        for layer in range(LAYERS):
            assert np.array_equal(outs[layer], outs0[layer])
