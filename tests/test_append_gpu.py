"""K1 parity on the GPU: fused RoPE + paged append against the reference's own
ropeKernel/storePagedKV (built from its sources; bit-exact), the CPU oracle
(page placement exact, RoPE within one BF16 ulp) and the reference's
paged_kvcache_test flow through the native host API."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import workloads as W
from gpu_util import assert_close_bf16, dev_bf16, dev_i32, f32, host_bf16
from vllm_b200 import _native as N
from vllm_b200 import cache as C
from vllm_b200 import ops

pytestmark = pytest.mark.gpu


def vp(t):
    return ctypes.c_void_p(t.data_ptr())


def i32p(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def test_prefill_append_bit_exact_vs_reference(ref_lib):
    """prefill_append: 4 requests x 256 tokens, shuffled 256-page pool, layers 0 and 1."""
    case = W.prefill_append()
    R, T = case.k.shape[0], case.tokens
    num_layers = 2
    cache = C.allocatePagedKVCache(case.num_pages, num_layers=num_layers, max_seq_len=1024)
    cache.free_blocks = list(case.free_list)
    ocache_free = list(case.free_list)
    seqs = [C.SequenceKVState() for _ in range(R)]
    k_pool, v_pool = cache.pools()
    k_pool.zero_()
    v_pool.zero_()
    ref_k = torch.zeros_like(k_pool)
    ref_v = torch.zeros_like(v_pool)
    for layer in range(num_layers):
        for r in range(R):
            k = dev_bf16(case.k[r])
            v = dev_bf16(case.v[r])
            q = dev_bf16(case.q[r])
            if layer == 0:
                expect_table = [ocache_free.pop() for _ in range(T // 16)]
            C.storePagedKV(cache, seqs[r], layer, k, v, T, apply_rope=True, rope_q=q)
            torch.cuda.synchronize()
            table = np.array(seqs[r].block_table, np.int32)
            if layer == 0:
                assert list(table) == expect_table  # allocator parity on the shuffled pool
            # reference: rope(q), rope(k), storePagedKV (src/model/paged_transformer.cu:34-36)
            rk = dev_bf16(case.k[r])
            rq = dev_bf16(case.q[r])
            assert ref_lib.ref_rope(vp(rq), T, 2048, 0) == 0
            assert ref_lib.ref_rope(vp(rk), T, 512, 0) == 0
            assert ref_lib.ref_store_paged_kv(vp(ref_k), vp(ref_v), case.num_pages, layer,
                                              i32p(table), table.size, 0, vp(rk), vp(v), T) == 0
            assert torch.equal(k.view(torch.int16), rk.view(torch.int16)), "RoPE(K) bits"
            assert torch.equal(q.view(torch.int16), rq.view(torch.int16)), "RoPE(q) bits"
    torch.cuda.synchronize()
    assert torch.equal(k_pool.view(torch.int16), ref_k.view(torch.int16)), "K pages"
    assert torch.equal(v_pool.view(torch.int16), ref_v.view(torch.int16)), "V pages"


def test_rope_every_position_up_to_32k_bit_exact(ref_lib):
    rng = np.random.default_rng(12)
    T = 32768
    x = W.normal_bf16(rng, (T, 512))
    xr = dev_bf16(x)
    assert ref_lib.ref_rope(vp(xr), T, 512, 0) == 0
    pages = T // 16
    k_pool = torch.zeros((1, pages, 16, 512), dtype=torch.bfloat16, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    table = dev_i32(np.arange(pages, dtype=np.int32)[None, :])
    k = dev_bf16(x)
    v = dev_bf16(x)
    tok_seq = torch.zeros(T, dtype=torch.int32, device="cuda")
    ops.rope_append(k_pool, v_pool, 0, table, dev_i32(np.arange(T)), k, v, token_seq=tok_seq)
    torch.cuda.synchronize()
    assert torch.equal(k.view(torch.int16), xr.view(torch.int16))
    assert torch.equal(k_pool.view(T, 512).view(torch.int16), xr.view(torch.int16))
    # q heads (2048 wide) over the first 8192 positions
    xq = W.normal_bf16(rng, (8192, 2048))
    qr = dev_bf16(xq)
    assert ref_lib.ref_rope(vp(qr), 8192, 2048, 0) == 0
    q = dev_bf16(xq)
    ops.rope_append(k_pool, v_pool, 0, table, dev_i32(np.arange(8192)), k[:8192].contiguous(),
                    v[:8192].contiguous(), q=q, token_seq=tok_seq[:8192].contiguous(),
                    rope_k=False, writeback_k=False)
    torch.cuda.synchronize()
    assert torch.equal(q.view(torch.int16), qr.view(torch.int16))


def test_decode_append_matches_reference_batch(ref_lib):
    """ropeBatch(q), ropeBatch(k) + storePagedKVBatch as one launch (decode form)."""
    rng = np.random.default_rng(13)
    positions = np.array([16, 63, 128, 255], np.int32)
    q = W.normal_bf16(rng, (4, 2048))
    k = W.normal_bf16(rng, (4, 512))
    v = W.normal_bf16(rng, (4, 512))
    tables = W.scattered_tables(rng, positions + 1, 64)
    rq, rk = dev_bf16(q), dev_bf16(k)
    dpos = dev_i32(positions)
    assert ref_lib.ref_rope_batch(vp(rq), 4, 2048, vp(dpos)) == 0
    assert ref_lib.ref_rope_batch(vp(rk), 4, 512, vp(dpos)) == 0
    k_pool = torch.zeros((1, 64, 16, 512), dtype=torch.bfloat16, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    qd, kd, vd = dev_bf16(q), dev_bf16(k), dev_bf16(v)
    ops.rope_append(k_pool, v_pool, 0, dev_i32(tables), dpos, kd, vd, q=qd)
    torch.cuda.synchronize()
    assert torch.equal(qd.view(torch.int16), rq.view(torch.int16))
    assert torch.equal(kd.view(torch.int16), rk.view(torch.int16))
    kp = host_bf16(k_pool)
    vpool = host_bf16(v_pool)
    rk_h = host_bf16(rk)
    for b, pos in enumerate(positions):
        phys = tables[b, pos // 16]
        assert np.array_equal(kp[0, phys, pos % 16], rk_h[b])
        assert np.array_equal(vpool[0, phys, pos % 16], v[b])


def test_append_against_cpu_oracle():
    """Page placement exact (payload with NaN/Inf bit patterns, no RoPE); RoPE
    within one BF16 ulp of the libm restatement."""
    rng = np.random.default_rng(14)
    T, pages = 100, 12
    k = rng.integers(0, 65536, size=(T, 512), dtype=np.uint16)
    v = rng.integers(0, 65536, size=(T, 512), dtype=np.uint16)
    table = rng.permutation(pages).astype(np.int32)[None, :8]
    start = 7
    pos = np.arange(start, start + T, dtype=np.int32)
    kp = torch.zeros((2, pages, 16, 512), dtype=torch.bfloat16, device="cuda")
    vpd = torch.zeros_like(kp)
    ops.rope_append(kp, vpd, 1, dev_i32(table), dev_i32(pos), dev_bf16(k), dev_bf16(v),
                    token_seq=torch.zeros(T, dtype=torch.int32, device="cuda"), rope_k=False)
    ok = np.zeros((2, pages, 16, 512), np.uint16)
    ov = np.zeros_like(ok)
    oracle.store_paged(ok, ov, 1, table[0], start, k, v)
    assert np.array_equal(host_bf16(kp), ok)
    assert np.array_equal(host_bf16(vpd), ov)
    # RoPE values vs the CPU restatement
    kn = W.normal_bf16(rng, (T, 512))
    kd = dev_bf16(kn)
    ops.rope_append(kp, vpd, 0, dev_i32(table), dev_i32(pos), kd, dev_bf16(kn),
                    token_seq=torch.zeros(T, dtype=torch.int32, device="cuda"))
    ours = host_bf16(kd)
    cpu = oracle.rope(kn, positions=pos)
    ok, stats = oracle.rope_close(ours, cpu, kn)
    assert ok, stats


def _cache_values(layer, positions, is_v):
    """Vectorised workloads.reference_cache_value over positions x 512 channels."""
    pos = np.asarray(positions, np.int64)[:, None]
    d = np.arange(512, dtype=np.int64)[None, :]
    if is_v:
        n = (layer * 11 + pos * 7 + d % 23) % 103 - 51
    else:
        n = (layer * 13 + pos * 3 + d % 17) % 101 - 50
    return W.bf16_bits((n / 8.0).astype(np.float32))


def test_value_formula_vectorisation_matches_reference_formula():
    for layer, t, d, is_v in [(0, 0, 0, False), (3, 17, 100, True), (15, 33, 511, False)]:
        a = _cache_values(layer, [t], is_v)[0, d]
        b = W.bf16_bits(np.float32(W.reference_cache_value(layer, t, d, is_v)))
        assert a == b


def test_reference_kvcache_test_flow_on_device():
    """tests/paged_kvcache_test.cu:25-97: deterministic payload through
    storePagedKV for prompt lengths {1,15,16,17,31,32,33}, 3 passes x 16 layers,
    every stored value checked at its page offset."""
    for prompt in (1, 15, 16, 17, 31, 32, 33):
        cache = C.allocatePagedKVCache(9)
        for b in range(9):
            assert C.allocatePhysicalBlock(cache) == b
        for b in (8, 2, 5):
            C.freePhysicalBlock(cache, b)
        seq = C.SequenceKVState()
        for p in range(3):
            count = prompt if p == 0 else 1
            start = seq.current_seq_len
            for layer in range(16):
                positions = range(start, start + count)
                C.storePagedKV(cache, seq, layer, dev_bf16(_cache_values(layer, positions, False)),
                               dev_bf16(_cache_values(layer, positions, True)), count)
                assert seq.current_seq_len == start
            seq.current_seq_len = start + count
            assert seq.block_table == [5, 2, 8][:len(seq.block_table)]
            k_pool, v_pool = cache.pools()
            kp, vpp = host_bf16(k_pool), host_bf16(v_pool)
            L = seq.current_seq_len
            tab = np.array(seq.block_table)
            t = np.arange(L)
            for layer in range(16):
                assert np.array_equal(kp[layer, tab[t // 16], t % 16], _cache_values(layer, t, False))
                assert np.array_equal(vpp[layer, tab[t // 16], t % 16], _cache_values(layer, t, True))
        C.freeSequenceBlocks(cache, seq)
        assert len(cache.free_blocks) == 3
        cache.close()


def test_bad_token_rows_are_reported_and_skipped():
    kp = torch.zeros((1, 4, 16, 512), dtype=torch.bfloat16, device="cuda")
    vpd = torch.zeros_like(kp)
    table = dev_i32(np.array([[0, 1], [2, -1]], np.int32))
    k = torch.ones((3, 512), dtype=torch.bfloat16, device="cuda")
    v = torch.ones_like(k)
    err = ops.new_error_word("cuda")
    # token 0 -> row 1, position 20: table entry -1 (no page); token 1 -> row 5 (no such row)
    ops.rope_append(kp, vpd, 0, table, dev_i32([20, 3, 17]), k, v,
                    token_seq=dev_i32([1, 5, 0]), rope_k=False, error=err)
    torch.cuda.synchronize()
    bits = int(err.item())
    assert bits & N.TVP_DEVERR_BAD_PAGE and bits & N.TVP_DEVERR_BAD_TOKEN
    h = host_bf16(kp)
    assert (h[0, 1, 1] == 0x3F80).all()     # the valid token landed (row 0, pos 17)
    assert (h[0, 2] == 0).all() and (h[0, 0] == 0).all()


def test_host_api_prefill_then_batched_decode_matches_oracle():
    """storePagedKV (fused RoPE) per request, then one decode step through
    preparePagedBatch / storePagedKVBatch / pagedDecodeAttention."""
    rng = np.random.default_rng(15)
    prompts = [40, 17, 129]
    cache = C.allocatePagedKVCache(64, num_layers=2)
    seqs = [C.SequenceKVState() for _ in prompts]
    for layer in range(2):
        for s, n in zip(seqs, prompts):
            C.storePagedKV(cache, s, layer, dev_bf16(W.normal_bf16(rng, (n, 512))),
                           dev_bf16(W.normal_bf16(rng, (n, 512))), n, apply_rope=True)
    for s, n in zip(seqs, prompts):
        s.current_seq_len = n
    md = C.PagedBatchMetadata(max_batch=4, max_pages_per_seq=64)
    C.preparePagedBatch(cache, seqs, md)
    q = dev_bf16(W.normal_bf16(rng, (3, 2048)))
    k = dev_bf16(W.normal_bf16(rng, (3, 512)))
    v = dev_bf16(W.normal_bf16(rng, (3, 512)))
    layer = 1
    C.storePagedKVBatch(cache, md, layer, q, k, v)
    out = torch.empty_like(q)
    C.pagedDecodeAttention(cache, md, layer, q, out)
    torch.cuda.synchronize()
    assert md.error_bits() == 0
    k_pool, v_pool = cache.pools()
    tables = np.full((3, 64), -1, np.int32)
    for i, s in enumerate(seqs):
        tables[i, :len(s.block_table)] = s.block_table
    lens = np.array([n + 1 for n in prompts], np.int32)
    exact = oracle.decode_attention_f64(host_bf16(q), host_bf16(k_pool), host_bf16(v_pool),
                                        layer, tables, lens)
    assert_close_bf16(host_bf16(out), exact, 1e-2, 2e-2, "host API decode")
    compat = torch.empty_like(q)
    C.pagedDecodeAttention(cache, md, layer, q, compat, mode=N.TVP_MODE_COMPAT)
    torch.cuda.synchronize()
    ref = oracle.decode_attention(host_bf16(q), host_bf16(k_pool), host_bf16(v_pool), layer,
                                  tables, lens)
    assert_close_bf16(host_bf16(compat), f32(ref), 4e-3, 1e-2, "host API compat")
    # the store did not advance lengths; the caller does (reference contract)
    assert [s.current_seq_len for s in seqs] == prompts
