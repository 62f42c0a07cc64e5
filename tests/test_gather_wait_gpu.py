"""The wait at the end of the fused KV-head-shard gather gives up instead of
hanging.  Two processes share one GPU: rank 1 connects and then launches
nothing, so rank 0's flag never reaches the count of both ranks' signals.
Rank 0's gather launch must end after its bound (2 s) with TVP_DEVERR_TIMEOUT
set, the rows of its own heads must be right (the gather's stores reached its
own buffer), and the context must stay usable.  Only one kernel waits, on a
flag nothing else will set; no two waiting kernels share the GPU."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LENS = [700, 33, 1, 260]


def _rank(rank, q_out, q_in, mine_done, other_done, results):
    import workloads as W
    from gpu_util import dev_bf16, dev_i32, f32, host_bf16
    from vllm_b200 import _native as N
    from vllm_b200 import ops, sharding

    torch.cuda.set_device(0)
    lib = N.load()
    h = ctypes.c_void_p()
    N.check(lib.tvp_head_gather_create(2, rank, 4, len(LENS), ctypes.byref(h)))
    mine = (ctypes.c_char * N.TVP_IPC_HANDLE_BYTES)()
    N.check(lib.tvp_head_gather_export(h, mine))
    q_out.put(bytes(mine))
    other = q_in.get(timeout=60)
    blob = bytes(mine) + other if rank == 0 else other + bytes(mine)
    N.check(lib.tvp_head_gather_connect(h, blob))
    if rank == 1:
        # teardown: close the peer's buffer, then free ours once the peer closed it
        N.check(lib.tvp_head_gather_disconnect(h))
        mine_done.set()
        assert other_done.wait(120)
        N.check(lib.tvp_head_gather_destroy(h))
        results[1] = "ok"
        return
    try:
        case = W.decode_random(5, LENS)
        heads = sharding.shard_by_kv_head(2)[0]
        q = dev_bf16(np.ascontiguousarray(sharding.slice_q_heads(case.q, heads)))
        kp = dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads)))
        vp = dev_bf16(np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads)))
        tables, lens = dev_i32(case.tables), dev_i32(case.lens)
        ws = ops.DecodeWorkspace(len(LENS), "cuda", kv_heads=4)
        err = ops.new_error_word("cuda")
        ops.decode_plan(lens, case.tables.shape[1], ws, error=err)
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        N.check(lib.tvp_paged_decode_attention_gather(
            P(q), P(kp), P(vp), case.num_pages, 1, 0, 4, 16, P(tables), case.tables.shape[1],
            P(lens), len(LENS), 0.125, ws.num_ctas, P(ws.buffer), ws.nbytes, h, 0, P(err), stream))
        torch.cuda.synchronize()
        bits = int(err.item())
        rows_ptr = ctypes.c_void_p()
        N.check(lib.tvp_head_gather_rows(h, 0, ctypes.byref(rows_ptr)))
        from vllm_b200.cache import _CudaArray
        rows = torch.as_tensor(_CudaArray(rows_ptr.value, (len(LENS), 2048), "<u2"), device="cuda")
        own = rows.cpu().numpy()[:, :1024].copy()
        # the context is still usable: a plain decode runs clean afterwards
        err2 = ops.new_error_word("cuda")
        out = ops.paged_decode_attention(q, kp, vp, 0, tables, lens, ws, error=err2)
        torch.cuda.synchronize()
        results[0] = (bits, own, host_bf16(out), int(err2.item()))
    finally:
        N.check(lib.tvp_head_gather_disconnect(h))
        mine_done.set()
        assert other_done.wait(120)
        N.check(lib.tvp_head_gather_destroy(h))


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_gather_wait_times_out_when_a_rank_never_signals():
    import torch.multiprocessing as mp

    import oracle
    import workloads as W
    from gpu_util import assert_close_bf16, f32
    from vllm_b200 import _native as N
    from vllm_b200 import sharding

    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    a, b = ctx.Queue(), ctx.Queue()
    d0, d1 = ctx.Event(), ctx.Event()
    procs = [ctx.Process(target=_rank, args=(0, a, b, d0, d1, results)),
             ctx.Process(target=_rank, args=(1, b, a, d1, d0, results))]
    for p in procs:
        p.start()
    for p in procs:
        p.join(180)
        assert p.exitcode == 0
    bits, own, plain, bits2 = results[0]
    assert results[1] == "ok"
    assert bits & N.TVP_DEVERR_TIMEOUT
    assert bits2 == 0
    case = W.decode_random(5, LENS)
    heads = sharding.shard_by_kv_head(2)[0]
    ref = oracle.decode_attention(np.ascontiguousarray(sharding.slice_q_heads(case.q, heads)),
                                  np.ascontiguousarray(sharding.slice_kv_heads(case.k_pool, heads)),
                                  np.ascontiguousarray(sharding.slice_kv_heads(case.v_pool, heads)),
                                  0, case.tables, case.lens)
    assert_close_bf16(own, f32(ref), 1e-2, 2e-2, "own heads through the gather")
    assert_close_bf16(plain, f32(ref), 1e-2, 2e-2, "plain decode after the timeout")
