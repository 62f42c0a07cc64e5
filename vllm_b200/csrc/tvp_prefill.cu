// K3 — paged causal prefill attention, reading K and V from the pages, on the
// 5th-generation tensor cores (tcgen05, accumulators in Tensor Memory).
//
// Replaces the reference's prefill attention (src/model/paged_transformer.cu:37-40):
// computeAttentionScores (32 cuBLAS GEMMs over the contiguous K,
// src/model/attention.cu:10-51), causalMask (src/model/causalMask.cu:7-38),
// softmaxRows (src/model/softmax.cu:47-72, capped at 1024 columns) and
// attentionScoresTimesV (32 GEMMs, src/model/attention.cu:144-192).  Here the
// query tokens of each sequence attend, causally, the keys 0..position already
// in that sequence's pages (the prompt just appended by K1, plus any earlier
// context: chunked prefill), with no length cap and no score matrix in HBM.
//
// Queries are varlen: sequence s owns query tokens [cu_q[s], cu_q[s + 1]) at
// positions q_pos0[s], q_pos0[s] + 1, ...  A CTA takes one (32-token tile,
// sequence, KV head); its 128 MMA rows are the tile's (token, query head)
// pairs of the GQA group, row 4 t + h, so every K/V byte serves 4 heads.
// Keys go in chunks of 4 pages (64 keys).  A CTA has 12 warps:
//   * warp 0 streams each chunk's K and V boxes (the decode kernels' tensor
//     maps, 128-byte swizzle) into a 4-stage ring with TMA; page slots past
//     the tile's last position are filled with zeros by an out-of-range box;
//   * warp 1 allocates Tensor Memory and one of its threads issues the MMAs:
//     S = Q K^T (M 128, N 64, K 64: Q and K both K-major in shared memory,
//     S in TMEM) and O += P V (M 128, N 64, K 64: P K-major, V MN-major as it
//     lands from TMA, O in TMEM), each followed by tcgen05.commit to an
//     mbarrier;
//   * two softmax sides of four warps, warps 4-7 and 8-11, one thread per row
//     (TMEM lane quarter = warp % 4).  Side s takes the chunks c with
//     c % 2 == s: it reads S buffer s from TMEM, rounds the scores to BF16
//     where the reference rounds them, masks causally, keeps its own online
//     base-2 softmax (running max, normaliser, lazy rescale of its own
//     accumulator O_s when the max grows by more than kLazyMargin) and writes
//     P as BF16 into P buffer s, a 128-byte-swizzled A tile of the P V MMA.
//     At the end the two sides merge their (max, sum, O) per row.
// One thread per row and chunk was a chain of 64 exponentials with only two
// softmax warps per SM sub-partition; two sides double the rows in flight
// per sub-partition without exchanging anything per chunk.  The producer and
// MMA warpgroup hands registers to the two softmax warpgroups (setmaxnreg).
// The MMA thread issues S(0), S(1), then per chunk c: [wait P(c)] P V(c) into
// O_{c % 2}, S(c + 2).  S(c)'s commit covers every earlier MMA, P V(c - 2)
// included, so when side c % 2 sees S(c) it may overwrite P buffer c % 2 and
// rescale O_{c % 2}.  The order is checked by a host model
// (tests/test_pipeline_protocol.py).  ~112 KiB of pipeline state and 256 TMEM
// columns per CTA let two CTAs share an SM.
#include "tvp_tile.cuh"
#include "tvp_umma.cuh"

namespace tvp {

namespace {

constexpr int kTcTokens = 32;                       // query tokens per CTA
constexpr int kTcRows = kTcTokens * kGroup;         // 128 MMA rows
constexpr int kTcChunkPages = 4;                    // pages per key chunk
constexpr int kTcChunk = kTcChunkPages * kPage;     // 64 keys
constexpr int kTcStages = 4;
constexpr int kTcKvBytes = kTcChunkPages * kTileBytes;  // 8 KiB of K (or of V) per stage
constexpr int kTcStageBytes = 2 * kTcKvBytes;           // K, then V
constexpr int kTcQBytes = kTcRows * 128;                // 64 BF16 per row
constexpr int kTcPBytes = kTcRows * 128;                // 64 keys per row
constexpr int kTcThreads = 12 * 32;
// S(even chunks) 0-63, S(odd) 64-127, O of side 0 128-191, O of side 1 192-255
constexpr uint32_t kTcTmemCols = 256;
// Register split: the warpgroup of warps 0-3 (producer, MMA issuer, two idle
// warps) drops to kTcLowRegs, the two softmax warpgroups rise to kTcHighRegs.
// The launch must provide kTcThreads x registers >= the split (checked on the
// host before the first launch: an unsatisfiable increase would never return).
constexpr int kTcLowRegs = 32;
constexpr int kTcHighRegs = 104;
// Of every kExpStride probability pairs, the last takes its 2^x on the FMA pipe
// (exp2_fma_x2) instead of the MUFU; 0 = all on the MUFU.  Measured on the
// 1 x 8192 prompt: none 567 us, a quarter 592 us, half 623 us: the softmax is
// bound by its instruction issue, not by the MUFU, so none is the default.
#ifndef TVP_PREFILL_EXP_STRIDE
#define TVP_PREFILL_EXP_STRIDE 0
#endif
constexpr int kExpStride = TVP_PREFILL_EXP_STRIDE;

// 2^x for two lanes without the MUFU, for x <= 10.  Range reduction
// x = i + f: adding 1.5 * 2^23 rounds x to the integer i, which lands in the
// low mantissa bits of the sum t; f = x - i lies in [-1/2, 1/2].  2^f is a
// cubic fitted (least squares on Chebyshev nodes, reweighted toward minimax)
// to the relative error of 2^f on that interval: 7.5e-5 at most, far below a
// BF16 probability's 2^-9.  i enters the exponent field by an integer add of
// t's bits shifted by 23.  Inputs below -125 (masked keys are -inf) give
// 2^-125, a normal number that adds nothing to a BF16 P.V product.
__device__ __forceinline__ uint64_t exp2_fma_x2(uint64_t x2) {
  float a, b;
  f2_unpack(x2, a, b);
  const uint64_t x = f2_pack(fmaxf(a, -125.f), fmaxf(b, -125.f));
  const uint64_t t = f2_add(x, f2_pack(12582912.f, 12582912.f));
  const uint64_t i = f2_add(t, f2_pack(-12582912.f, -12582912.f));  // round(x), exact
  const uint64_t f = f2_fma(i, f2_pack(-1.f, -1.f), x);              // x - i, exact
  uint64_t y = f2_fma(f, f2_pack(0.055171769f, 0.055171769f), f2_pack(0.24261113f, 0.24261113f));
  y = f2_fma(y, f, f2_pack(0.69326097f, 0.69326097f));
  y = f2_fma(y, f, f2_pack(0.99992806f, 0.99992806f));
  float ya, yb, ta, tb;
  f2_unpack(y, ya, yb);
  f2_unpack(t, ta, tb);
  return f2_pack(__int_as_float(__float_as_int(ya) + (__float_as_int(ta) << 23)),
                 __int_as_float(__float_as_int(yb) + (__float_as_int(tb) << 23)));
}
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kTcQBytes;                // P(even), then P(odd)
constexpr int kOffStages = kOffP + 2 * kTcPBytes;
constexpr int kOffBars = kOffStages + kTcStages * kTcStageBytes;
// q_full, o_full, drain, (unused), s_full[2], p_full[2], kv_full[stages], kv_empty[stages]
constexpr int kBarSFull = 4;
constexpr int kBarPFull = 6;
constexpr int kBarKvFull = 8;
constexpr int kBarKvEmpty = kBarKvFull + kTcStages;
constexpr int kNumBars = kBarKvEmpty + kTcStages;

constexpr size_t prefill_smem_bytes() { return kOffBars + kNumBars * 8 + 16; }

__global__ void __launch_bounds__(kTcThreads, 2)
    paged_prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map) {
  // 128-byte swizzled tiles need 1 KiB alignment.  The dynamic shared window of
  // this kernel (no static shared memory) starts 1 KiB aligned; a launch where
  // it does not reports an error instead of running.
  extern __shared__ __align__(1024) unsigned char smem[];
  const uint32_t sbase = smem_addr(smem);
  if (sbase & 1023u) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_SMEM_ALIGN);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBars);
  auto bar = [&](int i) { return smem_addr(&bars[i]); };
  const uint32_t q_full = bar(0), o_full = bar(1), drain = bar(2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int s = blockIdx.x, g = blockIdx.y;
  const int q_begin = __ldg(p.cu_q + s), q_end = __ldg(p.cu_q + s + 1);
  // Tiles run last-first: under causality the last tiles stream the most pages.
  // The tile is the slowest grid dimension, so the longest tiles of every
  // sequence and head start in the first wave and the short ones fill the tail.
  const int tile = gridDim.z - 1 - blockIdx.z;
  const int tok0 = q_begin + tile * kTcTokens;
  if (tok0 >= q_end) return;  // this sequence has fewer tiles
  const int count = min(kTcTokens, q_end - tok0);
  const int pos0 = __ldg(p.q_pos0 + s) + tile * kTcTokens;  // position of the tile's token 0
  const int pos_last = pos0 + count - 1;
  if (pos0 < 0 || pos_last / kPage >= p.table_stride) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_TOKEN);
    return;
  }
  const int last_page = pos_last / kPage;
  const int n_chunks = pos_last / kTcChunk + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 4);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(kBarSFull + b), 1);
      mbar_init(bar(kBarPFull + b), 4);
    }
    for (int i = 0; i < kTcStages; ++i) {
      mbar_init(bar(kBarKvFull + i), 1);
      mbar_init(bar(kBarKvEmpty + i), 1);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Threads that meet before Tensor Memory is released: warp 1 and both sides.
  constexpr int kEndThreads = 32 + 8 * 32;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTcLowRegs));
    if (warp >= 2) return;  // the rest of this warpgroup only hands its registers over
  }

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      prefetch_tensor_map(&k_map);
      prefetch_tensor_map(&v_map);
    }
    int issued = 0;
    for (int c = 0; c < n_chunks; ++c) {
      const int st = c % kTcStages;
      if (c >= kTcStages) {
        int timed_out = 0;
        if (lane == 0)
          timed_out = !mbar_wait_bounded(bar(kBarKvEmpty + st), ((c / kTcStages) - 1) & 1);
        if (__shfl_sync(0xffffffffu, timed_out, 0)) {
          if (lane == 0) {
            *abort_flag = 1;
            record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_EMPTY);
          }
          break;
        }
      }
      // lanes 0-3: K box of page slot `lane`, lanes 4-7: V box of slot lane - 4
      const int pg = c * kTcChunkPages + (lane & 3);
      const bool real = lane < 8 && pg <= last_page;
      const int phys = real ? __ldg(p.tables + (size_t)s * p.table_stride + pg) : -1;
      const bool ok = real && phys >= 0 && phys < p.num_pages;
      if (real && !ok && lane < 4) record_error(p.err, TVP_DEVERR_BAD_PAGE);
      if (lane == 0) mbar_arrive_expect_tx(bar(kBarKvFull + st), kTcStageBytes);
      __syncwarp();
      if (lane < 8) {
        const uint32_t dst = sbase + kOffStages + st * kTcStageBytes +
                             (lane < 4 ? 0 : kTcKvBytes) + (lane & 3) * kTileBytes;
        // A box wholly outside the pool (rows -16 .. -1) arrives as zeros.
        const int y = ok ? (int)(p.layer_row_base + (long long)phys * kPage) : -kPage;
        tma_load_2d(dst, lane < 4 ? &k_map : &v_map, g * kHeadDim, y, bar(kBarKvFull + st));
      }
      issued = c + 1;
    }
    drain_issued_stages<kTcStages>(bars + kBarKvFull, issued, lane, p.err);
    return;
  }

  if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      constexpr uint32_t kIdS = umma_idesc_bf16_f32(kTcRows, kTcChunk, false, false);
      constexpr uint32_t kIdO = umma_idesc_bf16_f32(kTcRows, kHeadDim, false, true);
      const uint32_t q_tile = sbase + kOffQ;
      auto stage_k = [&](int c) { return sbase + kOffStages + (c % kTcStages) * kTcStageBytes; };
      bool ok = true;
      auto wait = [&](uint32_t b, uint32_t parity) {
        if (ok && !mbar_wait_bounded(b, parity)) {
          record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
          ok = false;
        }
        return ok;
      };
      // S(c) = Q K(c)^T into S buffer c % 2: K = the 64 channels, 16 per MMA.
      auto issue_s = [&](int c) {
        if (!wait(bar(kBarKvFull + c % kTcStages), (c / kTcStages) & 1)) return;
        tc_fence_after_sync();
        const uint32_t k_tile = stage_k(c);
#pragma unroll
        for (int k = 0; k < kHeadDim / 16; ++k)
          umma_bf16(tmem + 64 * (c & 1), umma_desc_sw128(q_tile + 32 * k, 16, 1024),
                    umma_desc_sw128(k_tile + 32 * k, 16, 1024), kIdS, k > 0);
        umma_commit(bar(kBarSFull + (c & 1)));
      };
      wait(q_full, 0);
      issue_s(0);
      if (n_chunks > 1) issue_s(1);
      for (int c = 0; ok && c < n_chunks; ++c) {
        // O_{c % 2} += P(c) V(c): K = the chunk's 64 keys, 16 (one page of V)
        // per MMA; the first chunk of each side overwrites its accumulator.
        if (!wait(bar(kBarPFull + (c & 1)), (c >> 1) & 1)) break;
        tc_fence_after_sync();
        const uint32_t p_tile = sbase + kOffP + (c & 1) * kTcPBytes;
        const uint32_t v_tile = stage_k(c) + kTcKvBytes;
        const uint32_t tmem_o = tmem + 128 + 64 * (c & 1);
#pragma unroll
        for (int kk = 0; kk < kTcChunkPages; ++kk)
          umma_bf16(tmem_o, umma_desc_sw128(p_tile + 32 * kk, 16, 1024),
                    umma_desc_sw128(v_tile + kk * kTileBytes, 0, 1024), kIdO, (c >= 2 || kk > 0));
        umma_commit(bar(kBarKvEmpty + c % kTcStages));
        if (c + 2 < n_chunks) issue_s(c + 2);
      }
      if (ok) umma_commit(o_full);
      if (!ok) *abort_flag = 1;
      // Every MMA issued has completed before Tensor Memory is released.
      umma_commit(drain);
      if (!mbar_wait_bounded(drain, 0))
        record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_DRAIN);
    }
    __syncwarp();
    tc_fence_before_sync();
    named_barrier_sync(1, kEndThreads);
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTcTmemCols);
    return;
  }

  // ------------------------------ softmax sides ----------------------------
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTcHighRegs));
  const int side = (warp - 4) >> 2;  // 0: warps 4-7 (even chunks), 1: warps 8-11 (odd)
  const int quarter = warp & 3;      // TMEM lanes 32 quarter .. + 31
  const int row = quarter * 32 + lane;
  const int t = row >> 2, h = row & 3;
  const bool valid = t < count;
  const int qpos = pos0 + t;
  const int qdim = p.kv_heads * kGroup * kHeadDim;
  const int hq = g * kGroup + h;
  const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
  if (side == 0) {
    // Q row (token t, head hq) into the swizzled A tile of S = Q K^T.
    const uint4* src =
        reinterpret_cast<const uint4*>(p.q + (size_t)(tok0 + t) * qdim + hq * kHeadDim);
#pragma unroll
    for (int cc = 0; cc < 8; ++cc)
      *reinterpret_cast<uint4*>(smem + kOffQ + sw128_offset(row, cc)) =
          valid ? __ldg(src + cc) : make_uint4(0, 0, 0, 0);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(q_full);
  }
  float m = -INFINITY, l = 0.f;  // this side's running max (base-2 units) and normaliser
  bool ok = true;
  constexpr float kLog2e = 1.4426950408889634f;
  // A positive power-of-two scale (the reference's 1/8) commutes with the
  // BF16 rounding of the scores and folds into the exponent's constant:
  // bf16(s 2^k) = 2^k bf16(s), and r 2^k log2(e) is the same product as
  // before, so the bits do not change and a multiply per score is saved.
  const bool pow2 = p.scale_pow2 != 0;
  const float c_log2 = pow2 ? p.scale * kLog2e : kLog2e;
  const uint64_t scale2 = f2_pack(p.scale, p.scale);
  for (int c = side; c < n_chunks; c += 2) {
    bool ready = !*abort_flag && mbar_wait_bounded(bar(kBarSFull + side), (c >> 1) & 1);
    ready = __all_sync(0xffffffffu, ready);
    if (!ready) {
      if (lane == 0 && !*abort_flag) {
        *abort_flag = 1;
        record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
      }
      ok = false;
      break;
    }
    tc_fence_after_sync();
    // Scores rounded to BF16 where the reference rounds them (its score GEMM
    // writes BF16, src/model/attention.cu:10-51), two per conversion, kept as
    // packed BF16 pairs; keys past the row's position masked (only chunks
    // that reach the tile's first position need the test).
    const int key0 = c * kTcChunk;
    const bool diagonal = key0 + kTcChunk - 1 > pos0;
    uint32_t pk[kTcChunk / 2];
    uint32_t mxp[8];  // eight independent running maxima of BF16 pairs
#pragma unroll
    for (int i = 0; i < 8; ++i) mxp[i] = 0xff80ff80u;  // (-inf, -inf)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t sr[32];
      tmem_ld32(tmem + 64 * side + 32 * half + lane_base, sr);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float a = __uint_as_float(sr[j]), b = __uint_as_float(sr[j + 1]);
        if (!pow2) f2_unpack(f2_mul(f2_pack(a, b), scale2), a, b);
        if (diagonal) {
          const int key = key0 + 32 * half + j;
          if (key > qpos) a = -INFINITY;
          if (key + 1 > qpos) b = -INFINITY;
        }
        const uint32_t pr = pack_bf16x2(a, b);
        pk[16 * half + (j >> 1)] = pr;
        mxp[(j >> 1) & 7] = bf16x2_max(mxp[(j >> 1) & 7], pr);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) mxp[i] = bf16x2_max(mxp[i], mxp[i + 4]);
    const uint32_t m2 = bf16x2_max(bf16x2_max(mxp[0], mxp[1]), bf16x2_max(mxp[2], mxp[3]));
    float mx = fmaxf(bf16lo_to_f32(m2), bf16hi_to_f32(m2));
    mx *= c_log2;
    // Lazy running max: rescale only when a score beats the side's max by
    // more than kLazyMargin (probabilities stay below 2^kLazyMargin).
    float alpha = 1.f;
    if (mx > m + kLazyMargin) {
      const float mn = fmaxf(m, mx);
      alpha = m == -INFINITY ? 0.f : fast_exp2(m - mn);
      m = mn;
    }
    if (c >= 2 && __any_sync(0xffffffffu, alpha != 1.f)) {
      // O_side holds this side's earlier chunks: S(c)'s commit, just waited
      // for, covered P V(c - 2), the last MMA into it.
      // 16 columns at a time: the packed scores stay live meanwhile.
#pragma unroll 1
      for (int part = 0; part < 4; ++part) {
        const uint32_t taddr = tmem + 128 + 64 * side + 16 * part + lane_base;
        uint32_t o[16];
        tmem_ld16(taddr, o);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
        tmem_st16(taddr, o);
      }
      tmem_wait_st();
    }
    const float nbase = m == -INFINITY ? 0.f : -m;
    // P row into this side's swizzled A tile of O += P V.  S(c)'s commit also
    // covered P V(c - 2), the last reader of this tile.
    unsigned char* p_tile = smem + kOffP + side * kTcPBytes;
    const uint64_t l2e2 = f2_pack(c_log2, c_log2), nb2 = f2_pack(nbase, nbase);
    uint64_t ls2[4];  // four independent paired sums
#pragma unroll
    for (int i = 0; i < 4; ++i) ls2[i] = f2_pack(0.f, 0.f);
#pragma unroll
    for (int cc = 0; cc < 8; ++cc) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t pr = pk[4 * cc + e];
        const uint64_t arg = f2_fma(f2_pack(bf16lo_to_f32(pr), bf16hi_to_f32(pr)), l2e2, nb2);
        float p0, p1;
        if (kExpStride > 0 && e % (kExpStride > 0 ? kExpStride : 1) == kExpStride - 1) {
          f2_unpack(exp2_fma_x2(arg), p0, p1);
        } else {
          float a0, a1;
          f2_unpack(arg, a0, a1);
          p0 = fast_exp2(a0);
          p1 = fast_exp2(a1);
        }
        ls2[e] = f2_add(ls2[e], f2_pack(p0, p1));
        w[e] = pack_bf16x2(p0, p1);
      }
      *reinterpret_cast<uint4*>(p_tile + sw128_offset(row, cc)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    float la, lb;
    f2_unpack(f2_add(f2_add(ls2[0], ls2[1]), f2_add(ls2[2], ls2[3])), la, lb);
    l = l * alpha + (la + lb);
    // The last page's rows past pos_last hold stale data (possibly NaN): zero
    // them in the V tile before P V reads it (P is 0 there, but 0 x NaN is not).
    if (c == n_chunks - 1 && quarter == 0)
      zero_stale_v_rows(smem + kOffStages + (c % kTcStages) * kTcStageBytes + kTcKvBytes +
                            (last_page - c * kTcChunkPages) * kTileBytes,
                        pos_last % kPage + 1, lane);
    fence_proxy_async_smem();
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(kBarPFull + side));
  }
  bool fin = ok && !*abort_flag && mbar_wait_bounded(o_full, 0);
  fin = __all_sync(0xffffffffu, fin);
  if (!fin && ok && lane == 0 && !*abort_flag) {
    *abort_flag = 1;
    record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
  }
  // Merge the two sides per row: side 1 hands its (max, normaliser) to side 0
  // through the Q tile, whose last reader (an S MMA) completed before o_full.
  float* xchg = reinterpret_cast<float*>(smem + kOffQ);
  if (side == 1) {
    xchg[2 * row] = m;
    xchg[2 * row + 1] = l;
  }
  named_barrier_sync(2, 8 * 32);
  if (side == 0 && fin) {
    const float mb = xchg[2 * row], lb = xchg[2 * row + 1];
    const float mt = fmaxf(m, mb);
    const float wa = m == -INFINITY ? 0.f : fast_exp2(m - mt);
    const float wb = mb == -INFINITY ? 0.f : fast_exp2(mb - mt);
    const float lt = l * wa + lb * wb;
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const bool two = n_chunks > 1;  // side 1 wrote its accumulator
    tc_fence_after_sync();
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t oa[32], ob[32];
      tmem_ld32(tmem + 128 + 32 * half + lane_base, oa);
      if (two) tmem_ld32(tmem + 192 + 32 * half + lane_base, ob);
      tmem_wait_ld();
      if (valid) {
        uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(tok0 + t) * qdim + hq * kHeadDim) +
                     4 * half;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = 8 * cc + 2 * e;
            float x0 = __uint_as_float(oa[d]) * wa, x1 = __uint_as_float(oa[d + 1]) * wa;
            if (two) {
              x0 = fmaf(__uint_as_float(ob[d]), wb, x0);
              x1 = fmaf(__uint_as_float(ob[d + 1]), wb, x1);
            }
            w[e] = pack_bf16x2(x0 * inv, x1 * inv);
          }
          dst[cc] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
  tc_fence_before_sync();
  named_barrier_sync(1, kEndThreads);
}
}  // namespace

cudaError_t launch_paged_prefill(const PrefillParams& p, long long pool_rows, int max_q_len,
                                 int num_seqs, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    // The register split must fit the launch's pool (threads x registers per
    // thread); a warpgroup asking for more than is left would wait forever.
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, paged_prefill_kernel);
    if (e != cudaSuccess) return e;
    if ((long long)fa.numRegs * kTcThreads < 128LL * kTcLowRegs + 256LL * kTcHighRegs)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(paged_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)prefill_smem_bytes());
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  CUtensorMap k_map, v_map;
  if (!pool_tensor_map(p.k_pool, pool_rows, p.kv_heads, &k_map) ||
      !pool_tensor_map(p.v_pool, pool_rows, p.kv_heads, &v_map))
    return cudaErrorInvalidValue;
  const dim3 grid(num_seqs, p.kv_heads, (max_q_len + kTcTokens - 1) / kTcTokens);
  paged_prefill_kernel<<<grid, kTcThreads, prefill_smem_bytes(), stream>>>(p, k_map, v_map);
  return cudaGetLastError();
}

}  // namespace tvp
