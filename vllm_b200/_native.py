"""ctypes binding of ``libtvp_paged.so`` (the C-ABI declared in include/tvp_paged.h).

Loading fails loudly when the library is missing: there is no CPU or PyTorch
fallback for any operation of this package.
"""
from __future__ import annotations

import ctypes
import os
import re
from ctypes import POINTER, c_float, c_int, c_int32, c_size_t, c_uint16, c_void_p
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "_lib" / "libtvp_paged.so"
HEADER_PATH = _PKG.parent / "include" / "tvp_paged.h"

TVP_OK = 0
TVP_ERR_INVALID_ARGUMENT = -1
TVP_ERR_RUNTIME = -2
TVP_ERR_NO_FREE_BLOCKS = -3
TVP_ERR_UNSUPPORTED = -4
TVP_ERR_WORKSPACE = -5

TVP_DEVERR_BAD_PAGE = 1
TVP_DEVERR_BAD_LENGTH = 2
TVP_DEVERR_TIMEOUT = 4
TVP_DEVERR_BAD_PLAN = 8
TVP_DEVERR_BAD_TOKEN = 16
TVP_DEVERR_SMEM_ALIGN = 32
TVP_DEVERR_WAIT_FULL = 0x100
TVP_DEVERR_WAIT_EMPTY = 0x200
TVP_DEVERR_WAIT_DRAIN = 0x400
TVP_DEVERR_WAIT_PEERS = 0x800

TVP_MODE_FAST = 0
TVP_MODE_COMPAT = 1

TVP_APPEND_ROPE_K = 1
TVP_APPEND_ROPE_Q = 2
TVP_APPEND_WRITEBACK_K = 4

TVP_IPC_HANDLE_BYTES = 64

HEAD_DIM = 64
PAGE_TOKENS = 16
GQA_GROUP = 4
KV_HEADS = 8
Q_HEADS = 32

_bf16p = POINTER(c_uint16)
_i32p = POINTER(c_int32)

# name -> (restype, argtypes)
_SIGNATURES = {
    "tvp_strerror": (ctypes.c_char_p, [c_int]),
    "tvp_version": (c_int, []),
    "tvp_device_sm_count": (c_int, [POINTER(c_int)]),
    "tvp_rope_append": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_int,
                                c_int, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                c_int, c_int, c_void_p, c_void_p]),
    "tvp_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "tvp_decode_plan": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                c_void_p, c_void_p]),
    "tvp_paged_decode_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                           c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                           c_float, c_int, c_int, c_void_p, c_size_t, c_void_p,
                                           c_void_p, c_void_p]),
    "tvp_paged_decode_attention_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int,
                                                   c_int, c_int, c_int, c_void_p, c_int, c_void_p,
                                                   c_int, c_float, c_int, c_void_p, c_void_p,
                                                   c_void_p]),
    "tvp_paged_prefill_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                            c_int, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                            c_int, c_int, ctypes.c_float, c_void_p, c_void_p,
                                            c_void_p]),
    "tvp_greedy_argmax_workspace_bytes": (c_size_t, [c_int]),
    "tvp_greedy_argmax": (c_int, [c_void_p, c_int, c_int, ctypes.c_longlong, c_void_p, c_void_p,
                                  c_size_t, c_void_p]),
    "tvp_decode_projections": (c_int, [c_void_p, c_int, c_int, c_int, POINTER(c_void_p),
                                       POINTER(c_int), POINTER(c_void_p), c_int, c_void_p]),
    "tvp_decode_projection_residual_rmsnorm": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p,
                                                       c_void_p, c_void_p, c_void_p, c_void_p]),
    "tvp_decode_qkv_rope_append": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                           c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                           c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "tvp_decode_down_norm_qkv": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                         c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                         c_void_p, c_int, c_void_p, c_void_p, c_void_p]),
    "tvp_head_gather_create": (c_int, [c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    "tvp_head_gather_export": (c_int, [c_void_p, c_void_p]),
    "tvp_head_gather_connect": (c_int, [c_void_p, c_void_p]),
    "tvp_head_gather_rows": (c_int, [c_void_p, c_int, POINTER(c_void_p)]),
    "tvp_paged_decode_attention_gather": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                                  c_int, c_int, c_void_p, c_int, c_void_p, c_int,
                                                  ctypes.c_float, c_int, c_void_p, c_size_t,
                                                  c_void_p, c_int, c_void_p, c_void_p]),
    "tvp_head_gather_disconnect": (c_int, [c_void_p]),
    "tvp_head_gather_destroy": (c_int, [c_void_p]),
    "tvp_cache_create": (c_int, [c_int, c_int, c_int, c_int, c_int, POINTER(c_void_p)]),
    "tvp_cache_destroy": (None, [c_void_p]),
    "tvp_cache_pools": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int)]),
    "tvp_cache_free_count": (c_int, [c_void_p]),
    "tvp_cache_free_list": (c_int, [c_void_p, _i32p, c_int]),
    "tvp_cache_set_free_list": (c_int, [c_void_p, _i32p, c_int]),
    "tvp_allocate_physical_block": (c_int, [c_void_p, POINTER(c_int)]),
    "tvp_free_physical_block": (c_int, [c_void_p, c_int]),
    "tvp_seq_create": (c_int, [POINTER(c_void_p)]),
    "tvp_seq_destroy": (None, [c_void_p]),
    "tvp_seq_length": (c_int, [c_void_p]),
    "tvp_seq_set_length": (c_int, [c_void_p, c_int]),
    "tvp_seq_block_table": (c_int, [c_void_p, _i32p, c_int]),
    "tvp_reserve_sequence_blocks": (c_int, [c_void_p, c_void_p, c_int]),
    "tvp_free_sequence_blocks": (c_int, [c_void_p, c_void_p]),
    "tvp_store_paged_kv": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int,
                                   c_void_p, c_void_p]),
    "tvp_batch_create": (c_int, [c_int, c_int, POINTER(c_void_p)]),
    "tvp_batch_destroy": (None, [c_void_p]),
    "tvp_prepare_paged_batch": (c_int, [c_void_p, POINTER(c_void_p), c_int, c_void_p, c_void_p]),
    "tvp_batch_positions": (c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p),
                                    POINTER(c_void_p), POINTER(c_int)]),
    "tvp_store_paged_kv_batch": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_void_p,
                                         c_void_p]),
    "tvp_paged_attention": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int,
                                    c_void_p]),
    "tvp_batch_error": (c_int, [c_void_p, c_void_p, _i32p]),
}

_lib = None


class TvpError(RuntimeError):
    """A C-ABI call returned a runtime failure (reference: std::runtime_error)."""


class TvpNoFreeBlocks(TvpError):
    """The page pool is exhausted (reference: runtime_error from allocatePhysicalBlock)."""


def declared_symbols() -> list[str]:
    """Function names declared in include/tvp_paged.h."""
    text = HEADER_PATH.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tvp_[a-z0-9_]+)\s*\(", text)))


def load() -> ctypes.CDLL:
    """Loads the native library (once) and declares every C-ABI signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m vllm_b200.build` "
            "(the paged-KV path has no CPU fallback)")
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int, what: str = "") -> int:
    """Maps a C-ABI return code onto the reference's exception types."""
    if rc >= 0:
        return rc
    msg = load().tvp_strerror(rc).decode()
    if what:
        msg = f"{what}: {msg}"
    if rc == TVP_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == TVP_ERR_NO_FREE_BLOCKS:
        raise TvpNoFreeBlocks(msg)
    raise TvpError(msg)
