"""vllm_b200 — B200-native (sm_100a) paged-KV hot path for the tiny-vLLM
Llama-3.2-1B engine: fused RoPE + paged append and fused GQA paged decode
attention with a split-K combine, behind the C-ABI in include/tvp_paged.h.

``vllm_b200.ops``   kernels on torch CUDA tensors
``vllm_b200.cache`` the reference-named PagedKVCache / SequenceKVState /
                    PagedBatchMetadata host API (native allocator)
``vllm_b200.build`` builds ``_lib/libtvp_paged.so`` with nvcc for sm_100a
"""
from . import _native
from ._native import (KV_HEADS, Q_HEADS, HEAD_DIM, PAGE_TOKENS, GQA_GROUP, TVP_MODE_FAST,
                      TVP_MODE_COMPAT, TvpError, TvpNoFreeBlocks, load)

__all__ = ["KV_HEADS", "Q_HEADS", "HEAD_DIM", "PAGE_TOKENS", "GQA_GROUP", "TVP_MODE_FAST",
           "TVP_MODE_COMPAT", "TvpError", "TvpNoFreeBlocks", "load"]
