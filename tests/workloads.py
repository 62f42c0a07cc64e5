"""Seeded synthetic workloads of the paged-KV path (tests, golden generator, bench).

The reference measures no public dataset for this path; every input here is
seeded synthetic data with the shapes of the five workload configurations:

  decode_small   single-layer decode attention, Llama-3.2-1B geometry (32 Q / 8 KV
                 heads, head_dim 64), 4 rows with L = {17, 64, 129, 256}, block
                 tables a seeded permutation of a 128-page pool, BF16 N(0, 1).
  prefill_append 4 requests x 256 prompt tokens through RoPE + paged append, pages
                 from a shuffled 256-page pool.
  e2e            Llama-3.2-1B decode, batch 4, 128 prompt + 128 generated tokens.
  decode_sweep   256 rows, L ~ U[512, 8192], 16 layers, scattered 16-token pages.
  long_context   16 rows x L = 32768, split-K.

BF16 values are N(0, 1) float32 draws (numpy PCG64) rounded to nearest even.
"""
from __future__ import annotations

import dataclasses

import numpy as np

HEAD_DIM = 64
PAGE = 16
KV_HEADS = 8
GROUP = 4
Q_HEADS = KV_HEADS * GROUP  # 32
KV_DIM = KV_HEADS * HEAD_DIM  # 512
Q_DIM = Q_HEADS * HEAD_DIM    # 2048


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even, NaN kept NaN (numpy only)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def normal_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    return bf16_bits(rng.standard_normal(shape, dtype=np.float32))


def pages_for(L: int) -> int:
    return (L + PAGE - 1) // PAGE


@dataclasses.dataclass
class DecodeCase:
    """One decode-attention input set: pools [layers, P, 16, 512] (bf16 bits),
    tables [B, stride] int32 (-1 padded), lens [B] int32, q [B, 2048]."""
    lens: np.ndarray
    tables: np.ndarray
    num_pages: int
    num_layers: int
    q: np.ndarray | None = None
    k_pool: np.ndarray | None = None
    v_pool: np.ndarray | None = None

    @property
    def batch(self) -> int:
        return int(self.lens.size)

    @property
    def kv_bytes_per_layer(self) -> int:
        return int(self.lens.astype(np.int64).sum()) * KV_DIM * 2 * 2


def scattered_tables(rng: np.random.Generator, lens, num_pages: int, stride: int | None = None):
    """Block tables drawn in order from a seeded permutation of the pool."""
    lens = np.asarray(lens, dtype=np.int32)
    need = [pages_for(int(L)) for L in lens]
    if sum(need) > num_pages:
        raise ValueError("pool too small")
    stride = stride or max(max(need), 1)
    perm = rng.permutation(num_pages).astype(np.int32)
    tables = np.full((lens.size, stride), -1, dtype=np.int32)
    cur = 0
    for b, n in enumerate(need):
        tables[b, :n] = perm[cur:cur + n]
        cur += n
    return tables


def decode_small(seed: int = 1, with_data: bool = True) -> DecodeCase:
    """Single-layer decode, L = {17, 64, 129, 256}, 128-page pool."""
    rng = np.random.default_rng(seed)
    lens = np.array([17, 64, 129, 256], dtype=np.int32)
    tables = scattered_tables(rng, lens, 128)
    case = DecodeCase(lens=lens, tables=tables, num_pages=128, num_layers=1)
    if with_data:
        case.q = normal_bf16(rng, (4, Q_DIM))
        case.k_pool = normal_bf16(rng, (1, 128, PAGE, KV_DIM))
        case.v_pool = normal_bf16(rng, (1, 128, PAGE, KV_DIM))
    return case


def decode_random(seed: int, lens, num_pages: int | None = None, num_layers: int = 1,
                  slack_pages: int = 3, with_data: bool = True, kv_heads: int = KV_HEADS) -> DecodeCase:
    """Random decode case; kv_heads < 8 gives the pools and q of one KV-head shard."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, dtype=np.int32)
    need = sum(pages_for(int(L)) for L in lens)
    num_pages = num_pages or need + slack_pages
    tables = scattered_tables(rng, lens, num_pages)
    case = DecodeCase(lens=lens, tables=tables, num_pages=num_pages, num_layers=num_layers)
    if with_data:
        case.q = normal_bf16(rng, (lens.size, kv_heads * GROUP * HEAD_DIM))
        case.k_pool = normal_bf16(rng, (num_layers, num_pages, PAGE, kv_heads * HEAD_DIM))
        case.v_pool = normal_bf16(rng, (num_layers, num_pages, PAGE, kv_heads * HEAD_DIM))
    return case


def sweep_lengths(seed: int = 4, batch: int = 256, lo: int = 512, hi: int = 8192) -> np.ndarray:
    """decode_sweep lengths: L ~ U[lo, hi] inclusive, seeded."""
    return np.random.default_rng(seed).integers(lo, hi + 1, size=batch).astype(np.int32)


def decode_sweep(seed: int = 4, batch: int = 256) -> DecodeCase:
    """decode_sweep geometry only (16 layers; pools are filled on the device)."""
    rng = np.random.default_rng(seed + 1000)
    lens = sweep_lengths(seed, batch)
    need = int(sum(pages_for(int(L)) for L in lens))
    num_pages = need + 64
    tables = scattered_tables(rng, lens, num_pages)
    return DecodeCase(lens=lens, tables=tables, num_pages=num_pages, num_layers=16)


def long_context(seed: int = 5, batch: int = 16, L: int = 32768, num_layers: int = 1) -> DecodeCase:
    """long_context geometry only (pools are filled on the device)."""
    rng = np.random.default_rng(seed)
    lens = np.full(batch, L, dtype=np.int32)
    num_pages = batch * pages_for(L)
    tables = scattered_tables(rng, lens, num_pages)
    return DecodeCase(lens=lens, tables=tables, num_pages=num_pages, num_layers=num_layers)


@dataclasses.dataclass
class PrefillCase:
    """prefill_append: k, v [R, T, 512] pre-RoPE, q [R, T, 2048], free-list order."""
    k: np.ndarray
    v: np.ndarray
    q: np.ndarray
    free_list: np.ndarray  # bottom..top of the LIFO stack (top is handed out first)
    num_pages: int
    tokens: int


def prefill_append(seed: int = 2, requests: int = 4, tokens: int = 256,
                   num_pages: int = 256) -> PrefillCase:
    rng = np.random.default_rng(seed)
    k = normal_bf16(rng, (requests, tokens, KV_DIM))
    v = normal_bf16(rng, (requests, tokens, KV_DIM))
    q = normal_bf16(rng, (requests, tokens, Q_DIM))
    free_list = rng.permutation(num_pages).astype(np.int32)
    return PrefillCase(k=k, v=v, q=q, free_list=free_list, num_pages=num_pages, tokens=tokens)


def reference_attention_pattern():
    """The closed-form q, k, v of the reference's paged_attention_test
    (tests/paged_attention_test.cu:64-79): 3 rows, lengths {16, 17, 33},
    k/v [3][33][512], q [3][2048] (fp32 values, exact in bf16)."""
    lengths = [16, 17, 33]
    q = np.zeros((3, Q_DIM), dtype=np.float32)
    k = np.zeros((3, 33, KV_DIM), dtype=np.float32)
    v = np.zeros((3, 33, KV_DIM), dtype=np.float32)
    d2 = np.arange(Q_DIM)
    d = np.arange(KV_DIM)
    for row in range(3):
        q[row] = (((d2 * 3 + row) % 11) - 5) / 16.0
        for t in range(33):
            k[row, t] = (((t * 3 + d + row * 7) % 19) - 9) / 16.0
            v[row, t] = (((t + d * 5 + row * 11) % 23) - 11) / 16.0
    return lengths, bf16_bits(q), bf16_bits(k), bf16_bits(v)


def reference_cache_value(layer: int, position: int, d: int, is_v: bool) -> float:
    """Deterministic page payload of the reference's paged_kvcache_test
    (tests/paged_kvcache_test.cu:19-23)."""
    if is_v:
        n = (layer * 11 + position * 7 + d % 23) % 103 - 51
    else:
        n = (layer * 13 + position * 3 + d % 17) % 101 - 50
    return n / 8.0
