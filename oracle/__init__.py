"""TEST INFRASTRUCTURE ONLY — the oracle (checker) of the paged-KV path.

Loads the plain-C restatement of the reference (``tvp_oracle.c`` ->
``_build/liboracle.so``) and, when it was built, the reference's own hot-path
sources compiled for sm_100a (``_ref/libtvp_ref.so``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference legs
import this package; the product (``vllm_b200``) never does.

Arrays are numpy: BF16 is carried as raw ``uint16`` bits, pools are
``[num_layers, num_pages, 16, 512]`` (the reference layout), tables ``int32``.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from ctypes import POINTER, c_double, c_float, c_int, c_int32, c_size_t, c_uint16, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libtvp_ref.so"

_lib = None
_ref = None


def build(with_reference: bool = True) -> None:
    """Runs oracle/Makefile: the C restatement always, the reference build when
    the reference tree is present.  Only the Makefile knows where that tree is
    (its REF variable; the environment variable TVP_REFERENCE_DIR overrides it);
    its ``has-ref`` target answers whether the sources are there."""
    make = shutil.which("make")
    if make is None:
        raise RuntimeError("make not found")
    extra = [f"REF={os.environ['TVP_REFERENCE_DIR']}"] if os.environ.get("TVP_REFERENCE_DIR") else []
    subprocess.run([make, "-C", str(HERE), *extra], check=True)
    if not with_reference:
        return
    present = subprocess.run([make, "-s", "-C", str(HERE), "has-ref", *extra],
                             capture_output=True).returncode == 0
    if present:
        subprocess.run([make, "-C", str(HERE), "ref", "e2e", *extra], check=True)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build(with_reference=False)
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    u16p, i32p, f32p, f64p = POINTER(c_uint16), POINTER(c_int32), POINTER(c_float), POINTER(c_double)
    lib.orc_rope.argtypes = [u16p, c_int, c_int, i32p, c_int]
    lib.orc_rope.restype = None
    lib.orc_llama3_theta.argtypes = [c_int]
    lib.orc_llama3_theta.restype = c_float
    lib.orc_store_paged.argtypes = [u16p, u16p, c_int, c_int, c_int, i32p, c_int, c_int, c_int,
                                    u16p, u16p]
    lib.orc_store_paged.restype = c_int
    lib.orc_decode_attention.argtypes = [u16p, u16p, u16p, c_int, c_int, c_int, i32p, c_int, i32p,
                                         c_int, c_float, u16p, c_int]
    lib.orc_decode_attention.restype = c_int
    lib.orc_decode_attention_f64.argtypes = [u16p, u16p, u16p, c_int, c_int, c_int, i32p, c_int,
                                             i32p, c_int, c_double, f64p, c_int]
    lib.orc_decode_attention_f64.restype = c_int
    lib.orc_page_offset.argtypes = [c_int, c_int, c_int, c_int, c_int]
    lib.orc_page_offset.restype = c_size_t
    lib.orc_f32_to_bf16_array.argtypes = [f32p, u16p, c_size_t]
    lib.orc_f32_to_bf16_array.restype = None
    lib.orc_max_threads.argtypes = []
    lib.orc_max_threads.restype = c_int
    _lib = lib
    return lib


def load_reference():
    """The reference's own sources built for sm_100a, or None when not built."""
    global _ref
    if _ref is not None:
        return _ref
    if not REF_LIB_PATH.exists():
        return None
    lib = ctypes.CDLL(os.fspath(REF_LIB_PATH))
    lib.ref_rope.argtypes = [c_void_p, c_int, c_int, c_int]
    lib.ref_rope.restype = c_int
    lib.ref_rope_batch.argtypes = [c_void_p, c_int, c_int, c_void_p]
    lib.ref_rope_batch.restype = c_int
    lib.ref_store_paged_kv.argtypes = [c_void_p, c_void_p, c_int, c_int, POINTER(c_int32), c_int,
                                       c_int, c_void_p, c_void_p, c_int]
    lib.ref_store_paged_kv.restype = c_int
    lib.ref_paged_decode.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_int, POINTER(c_int32),
                                     c_int, POINTER(c_int32), c_int, c_void_p, c_int, c_size_t,
                                     POINTER(c_float)]
    lib.ref_paged_decode.restype = c_int
    lib.ref_prefill_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                          c_size_t, POINTER(c_float)]
    lib.ref_prefill_attention.restype = c_int
    _ref = lib
    return lib


# ---------------------------------------------------------------- helpers ---
def _p(a: np.ndarray, ctype):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(POINTER(ctype))


def f32_to_bf16(a) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even (restated in tvp_oracle.c)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    load().orc_f32_to_bf16_array(_p(a, c_float), _p(out, c_uint16), a.size)
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return (a.astype(np.uint32) << 16).view(np.float32)


def llama3_theta(pair: int) -> float:
    return float(load().orc_llama3_theta(pair))


def rope(x: np.ndarray, positions=None, position_offset: int = 0) -> np.ndarray:
    """RoPE of x [tokens, proj_dim] (bf16 bits); returns a new array."""
    out = np.ascontiguousarray(x, dtype=np.uint16).copy()
    tokens, dim = out.shape
    pos = None
    if positions is not None:
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        assert pos.shape == (tokens,)
    load().orc_rope(_p(out, c_uint16), tokens, dim, _p(pos, c_int32) if pos is not None else None,
                    position_offset)
    return out


def store_paged(k_pool: np.ndarray, v_pool: np.ndarray, layer: int, table, start: int,
                k: np.ndarray, v: np.ndarray) -> None:
    """storePagedKV into numpy pools [L, P, 16, kv_dim] (in place)."""
    num_pages, kv_dim = k_pool.shape[1], k_pool.shape[3]
    t = np.ascontiguousarray(table, dtype=np.int32)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    rc = load().orc_store_paged(_p(k_pool, c_uint16), _p(v_pool, c_uint16), num_pages, layer,
                                kv_dim, _p(t, c_int32), t.size, start, k.shape[0],
                                _p(k, c_uint16), _p(v, c_uint16))
    if rc != 0:
        raise ValueError("page table entry out of range")


def decode_attention(q, k_pool, v_pool, layer, tables, lens, scale=0.125, threads=0) -> np.ndarray:
    """Reference-semantics decode attention; returns bf16 bits [batch, 2048]."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    batch = lens.size
    kv_heads = k_pool.shape[3] // 64
    out = np.empty((batch, kv_heads * 4 * 64), dtype=np.uint16)
    rc = load().orc_decode_attention(_p(q, c_uint16), _p(k_pool, c_uint16), _p(v_pool, c_uint16),
                                     k_pool.shape[1], layer, kv_heads, _p(tables, c_int32),
                                     tables.shape[1], _p(lens, c_int32), batch, scale,
                                     _p(out, c_uint16), threads)
    if rc != 0:
        raise ValueError("page table entry out of range")
    return out


def decode_attention_f64(q, k_pool, v_pool, layer, tables, lens, scale=0.125, threads=0) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint16)
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    batch = lens.size
    kv_heads = k_pool.shape[3] // 64
    out = np.empty((batch, kv_heads * 4 * 64), dtype=np.float64)
    rc = load().orc_decode_attention_f64(_p(q, c_uint16), _p(k_pool, c_uint16),
                                         _p(v_pool, c_uint16), k_pool.shape[1], layer, kv_heads,
                                         _p(tables, c_int32), tables.shape[1], _p(lens, c_int32),
                                         batch, scale, _p(out, c_double), threads)
    if rc != 0:
        raise ValueError("page table entry out of range")
    return out


def prefill_attention(q, k_pool, v_pool, layer, tables, cu_q, q_pos0, scale=0.125, threads=0):
    """Reference-semantics causal prefill attention over the pages; bf16 bits
    [num_tokens, q_heads*64].  Query token t of sequence s, at position p,
    attends keys 0..p: the reference's prefill row (src/model/paged_transformer.cu:37-40:
    BF16 scores, causal mask, softmaxRows, FP32 P.V) has -inf past p, whose
    exp is exactly 0 in its pairwise sum, so it equals decode attention with
    length p + 1 (src/model/paged_attention.cu:133-161)."""
    cu_q = np.asarray(cu_q, dtype=np.int64)
    q_pos0 = np.asarray(q_pos0, dtype=np.int64)
    n = int(cu_q[-1])
    rows = np.empty(n, dtype=np.int64)
    lens = np.empty(n, dtype=np.int32)
    for s in range(len(q_pos0)):
        a, b = int(cu_q[s]), int(cu_q[s + 1])
        rows[a:b] = s
        lens[a:b] = q_pos0[s] + np.arange(b - a) + 1
    tab = np.ascontiguousarray(np.asarray(tables, dtype=np.int32)[rows])
    return decode_attention(q, k_pool, v_pool, layer, tab, lens, scale=scale, threads=threads)


def greedy_argmax(logits) -> np.ndarray:
    """Greedy token per row of FP32 logits [rows][vocab], as the reference's
    CPU scan restated in tests/argmax_test.cu:41-45 and implemented on the GPU
    by src/model/argmax.cu:16-45: each logit rounded to BF16; the running
    maximum starts at logit 0 and moves only on a strictly larger value, so
    ties keep the lowest index, NaNs never win, -0 equals +0, and a NaN logit
    0 keeps token 0."""
    x = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
    b = bf16_to_f32(f32_to_bf16(x))
    out = np.zeros(x.shape[0], np.int32)
    for r in range(x.shape[0]):
        if np.isnan(b[r, 0]):
            continue
        # NaNs -> -inf cannot win: logit 0 is a number at or above -inf and
        # comes first, so np.argmax's first-occurrence rule returns it then
        out[r] = int(np.argmax(np.where(np.isnan(b[r]), -np.inf, b[r])))
    return out


def max_threads() -> int:
    return int(load().orc_max_threads())


def rope_close(got: np.ndarray, expect: np.ndarray, rope_input: np.ndarray,
               max_mismatch_frac: float = 0.005) -> tuple[bool, dict]:
    """Compares RoPE outputs (bf16 bits) of two implementations whose FP32
    sin/cos/pow may differ in the last bit.  An element may differ by one BF16
    ulp at the scale of its input pair, |x| + |y| (the rotation's magnitude),
    which allows multi-ulp bit differences only for outputs near a zero
    crossing; at most `max_mismatch_frac` of elements may differ at all."""
    got = np.ascontiguousarray(got, np.uint16)
    expect = np.ascontiguousarray(expect, np.uint16)
    x = bf16_to_f32(rope_input).astype(np.float64)
    cols = np.arange(x.shape[-1])
    partner = (cols // 64) * 64 + (cols % 64 + 32) % 64
    mag = np.abs(x) + np.abs(x[..., partner])
    err = np.abs(bf16_to_f32(got).astype(np.float64) - bf16_to_f32(expect).astype(np.float64))
    within = err <= mag * 2.0 ** -7 + 1e-6
    frac = float((got != expect).mean())
    ok = bool(within.all()) and frac <= max_mismatch_frac
    return ok, {"max_abs_err": float(err.max()) if err.size else 0.0, "mismatch_frac": frac,
                "outside": int((~within).sum())}
