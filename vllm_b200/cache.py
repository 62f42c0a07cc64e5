"""Reference-named host API of the paged KV cache, over the C-ABI handles.

Same names, argument meaning and error behaviour as the reference's
include/paged_kvcache.cuh:21-28 and include/paged_attention.cuh:17-27:
ValueError where the reference throws std::invalid_argument, RuntimeError
(``TvpError`` / ``TvpNoFreeBlocks``) where it throws std::runtime_error.
The allocator itself is the native C++ one (vllm_b200/csrc/tvp_host.cpp).
"""
from __future__ import annotations

import ctypes
from ctypes import c_int, c_int32, c_void_p

import torch

from . import _native as N
from .ops import _stream


class _CudaArray:
    """__cuda_array_interface__ view of a raw device allocation (no ownership)."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": typestr, "version": 3, "strides": None}


class PagedKVCache:
    """PagedKVCache (include/paged_kvcache.cuh:8-14): K/V pools + LIFO free list."""

    def __init__(self, handle, num_layers: int, device_storage: bool):
        self._h = handle
        self.num_layers = num_layers
        self.device_storage = device_storage

    @property
    def handle(self):
        return self._h

    @property
    def num_blocks(self) -> int:
        n = c_int(0)
        N.check(N.load().tvp_cache_pools(self._h, None, None, ctypes.byref(n)))
        return n.value

    @property
    def free_blocks(self) -> list[int]:
        lib = N.load()
        n = lib.tvp_cache_free_count(self._h)
        buf = (c_int32 * max(n, 1))()
        lib.tvp_cache_free_list(self._h, buf, n)
        return list(buf[:n])

    @free_blocks.setter
    def free_blocks(self, blocks) -> None:
        arr = (c_int32 * max(len(blocks), 1))(*blocks)
        N.check(N.load().tvp_cache_set_free_list(self._h, arr, len(blocks)), "set free list")

    def pools(self):
        """(k_blocks, v_blocks) as torch views [num_layers, num_blocks, 16, 512] (no copy)."""
        if not self.device_storage:
            raise ValueError("cache has no device storage")
        k, v, n = c_void_p(), c_void_p(), c_int(0)
        N.check(N.load().tvp_cache_pools(self._h, ctypes.byref(k), ctypes.byref(v), ctypes.byref(n)))
        shape = (self.num_layers, n.value, N.PAGE_TOKENS, N.KV_HEADS * N.HEAD_DIM)
        kt = torch.as_tensor(_CudaArray(k.value, shape, "<u2"), device="cuda").view(torch.bfloat16)
        vt = torch.as_tensor(_CudaArray(v.value, shape, "<u2"), device="cuda").view(torch.bfloat16)
        return kt, vt

    def close(self) -> None:
        if self._h:
            N.load().tvp_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class SequenceKVState:
    """SequenceKVState (include/paged_kvcache.cuh:16-19)."""

    def __init__(self):
        h = c_void_p()
        N.check(N.load().tvp_seq_create(ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    @property
    def current_seq_len(self) -> int:
        return N.load().tvp_seq_length(self._h)

    @current_seq_len.setter
    def current_seq_len(self, value: int) -> None:
        N.check(N.load().tvp_seq_set_length(self._h, int(value)))

    @property
    def block_table(self) -> list[int]:
        lib = N.load()
        n = lib.tvp_seq_block_table(self._h, None, 0)
        buf = (c_int32 * max(n, 1))()
        lib.tvp_seq_block_table(self._h, buf, n)
        return list(buf[:n])

    def __del__(self):
        try:
            if self._h:
                N.load().tvp_seq_destroy(self._h)
                self._h = None
        except Exception:
            pass


def allocatePagedKVCache(num_blocks: int, num_layers: int = 16, max_seq_len: int = 1024,
                         device_storage: bool = True) -> PagedKVCache:
    """src/model/paged_kvcache.cu:37-62; device_storage=False builds the allocator only."""
    h = c_void_p()
    N.check(N.load().tvp_cache_create(num_blocks, num_layers, N.KV_HEADS, max_seq_len,
                                      int(device_storage), ctypes.byref(h)), "allocatePagedKVCache")
    return PagedKVCache(h, num_layers, device_storage)


def freePagedKVCache(cache: PagedKVCache) -> None:
    cache.close()


def allocatePhysicalBlock(cache: PagedKVCache) -> int:
    out = c_int(0)
    N.check(N.load().tvp_allocate_physical_block(cache.handle, ctypes.byref(out)),
            "allocatePhysicalBlock")
    return out.value


def freePhysicalBlock(cache: PagedKVCache, block: int) -> None:
    N.check(N.load().tvp_free_physical_block(cache.handle, int(block)), "freePhysicalBlock")


def freeSequenceBlocks(cache: PagedKVCache, seq: SequenceKVState) -> None:
    N.check(N.load().tvp_free_sequence_blocks(cache.handle, seq.handle), "freeSequenceBlocks")


def reserveSequenceBlocks(cache: PagedKVCache, seq: SequenceKVState, total_seq_len: int) -> None:
    N.check(N.load().tvp_reserve_sequence_blocks(cache.handle, seq.handle, int(total_seq_len)),
            "reserveSequenceBlocks")


def storePagedKV(cache: PagedKVCache, seq: SequenceKVState, layer: int, k, v, num_tokens: int,
                 apply_rope: bool = False, rope_q=None, stream=None) -> None:
    """storePagedKV (src/model/paged_kvcache.cu:119-139); with apply_rope the
    fused kernel also rotates k in place (and q when given)."""
    for t, name in ((k, "k"), (v, "v")):
        if t is not None and (not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous()):
            raise ValueError(f"{name} must be a contiguous bf16 CUDA tensor")
    kp = c_void_p(k.data_ptr()) if k is not None else None
    vp = c_void_p(v.data_ptr()) if v is not None else None
    qp = c_void_p(rope_q.data_ptr()) if rope_q is not None else None
    N.check(N.load().tvp_store_paged_kv(cache.handle, seq.handle, layer, kp, vp, int(num_tokens),
                                        int(apply_rope), qp, _stream(stream)), "storePagedKV")


class PagedBatchMetadata:
    """PagedBatchMetadata (include/paged_attention.cuh:6-15) with persistent
    device tables and the decode plan workspace."""

    def __init__(self, max_batch: int = 4, max_pages_per_seq: int = 64):
        h = c_void_p()
        N.check(N.load().tvp_batch_create(max_batch, max_pages_per_seq, ctypes.byref(h)),
                "PagedBatchMetadata")
        self._h = h

    @property
    def handle(self):
        return self._h

    def device_views(self):
        """(positions, lengths, block_tables) as torch views of the device arrays."""
        pos, lens, tabs, stride = c_void_p(), c_void_p(), c_void_p(), c_int(0)
        b = N.check(N.load().tvp_batch_positions(self._h, ctypes.byref(pos), ctypes.byref(lens),
                                                 ctypes.byref(tabs), ctypes.byref(stride)))
        mk = lambda p, shape: torch.as_tensor(_CudaArray(p.value, shape, "<i4"), device="cuda")
        return mk(pos, (b,)), mk(lens, (b,)), mk(tabs, (b, stride.value))

    def error_bits(self, stream=None) -> int:
        bits = c_int32(0)
        N.check(N.load().tvp_batch_error(self._h, _stream(stream), ctypes.byref(bits)))
        return bits.value

    def close(self):
        if self._h:
            N.load().tvp_batch_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def preparePagedBatch(cache: PagedKVCache, sequences, metadata: PagedBatchMetadata,
                      stream=None) -> None:
    arr = (c_void_p * len(sequences))(*[s.handle for s in sequences])
    N.check(N.load().tvp_prepare_paged_batch(cache.handle, arr, len(sequences), metadata.handle,
                                             _stream(stream)), "preparePagedBatch")


def storePagedKVBatch(cache: PagedKVCache, metadata: PagedBatchMetadata, layer: int, q, k, v,
                      stream=None) -> None:
    """ropeBatch(q), ropeBatch(k), storePagedKVBatch as one launch."""
    ptr = lambda t: c_void_p(t.data_ptr()) if t is not None else None
    N.check(N.load().tvp_store_paged_kv_batch(cache.handle, metadata.handle, layer, ptr(q), ptr(k),
                                              ptr(v), _stream(stream)), "storePagedKVBatch")


def pagedDecodeAttention(cache: PagedKVCache, metadata: PagedBatchMetadata, layer: int, q, out,
                         mode: int = N.TVP_MODE_FAST, stream=None) -> None:
    """computePagedAttentionScores + softmaxRows + pagedAttentionScoresTimesV as one launch."""
    N.check(N.load().tvp_paged_attention(cache.handle, metadata.handle, layer,
                                         c_void_p(q.data_ptr()), c_void_p(out.data_ptr()), mode,
                                         _stream(stream)), "pagedDecodeAttention")
