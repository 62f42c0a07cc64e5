// Per-tile building blocks of the fused decode attention: one warp attends
// the 4 query heads of one KV head over one 16-token page tile held in shared
// memory (128-byte swizzled rows of 64 BF16 channels, as the tiled TMA writes
// them), and keeps an online-softmax state in mma accumulator layout.
//
// Fragment layouts (mma.m16n8k16, BF16 in, FP32 accumulate):
//   S^T = K Q^T : A = K tile (16 tokens x 16 channels per k-step, row-major,
//                 ldmatrix), B = Q^T (16 channels x 8 query columns, 4 real),
//                 C rows = tokens tr, tr + 8; columns = query heads 2hc, 2hc+1.
//   O^T += V^T P^T : A = V^T (64 channels x 16 tokens, ldmatrix.trans of the V
//                 tile), B = P^T (16 tokens x 8 columns) obtained from the
//                 accumulator layout of S^T with movmatrix.
#pragma once

#include "tvp_params.cuh"

namespace tvp {

constexpr int kTileBytes = kPage * kHeadDim * 2;  // 2048: one KV head of one page
constexpr float kLazyMargin = 8.f;                // base-2 exponent units

// CTA shape shared by the decode kernels: a stage holds 8 (K, V) tile pairs
// (8 K tiles, then 8 V tiles); 16 consumer warps in 2 sets of 8, behind one
// producer warp, or behind a producer warpgroup that hands its registers to
// the consumers (REGSPLIT: the producer warpgroup keeps kProducerRegs per
// thread, the consumer warpgroups take kConsumerRegs; the launch must provide
// threads x registers >= the split, which the host checks before the first
// launch, since an unsatisfiable increase would never return).
constexpr int kPlanMagic = 0x54565031;  // "TVP1"
constexpr int kStageTiles = 8;
constexpr int kStageBytes = 2 * kStageTiles * kTileBytes;  // 32 KiB
constexpr int kProducerRegs = 40;
constexpr int kConsumerRegs = 104;

template <int SETS, bool REGSPLIT>
constexpr int decode_threads() {
  return (SETS * kStageTiles + (REGSPLIT ? 4 : 1)) * 32;
}

// True when a kernel compiled to `regs_per_thread` registers and launched with
// `threads` threads can satisfy the register split.
inline bool regsplit_fits(int regs_per_thread, int threads) {
  return (long long)regs_per_thread * threads >=
         128LL * kProducerRegs + (long long)(threads - 128) * kConsumerRegs;
}

// This lane's place in the fragments and in the tile's rows.
struct TileLane {
  int tr;        // accumulator row (token) of this lane
  int hc;        // accumulator column pair (query heads 2hc, 2hc + 1)
  int mrow;      // row within an 8x8 ldmatrix matrix
  int k_chunk;   // 16-byte chunk offset of this lane's K matrix
  int v_chunk;   // 16-byte chunk offset of this lane's V matrix
  uint32_t k_row;  // byte offset of this lane's K row within a tile
  uint32_t v_row;  // byte offset of this lane's V row within a tile
  __device__ __forceinline__ explicit TileLane(int lane) {
    const int mat = lane >> 3;
    tr = lane >> 2;
    hc = lane & 3;
    mrow = lane & 7;
    k_chunk = mat >> 1;
    v_chunk = mat & 1;
    k_row = (mrow + (mat & 1) * 8) * 128;   // K matrices: tokens 8*(m&1).., chunk 2*k4+(m>>1)
    v_row = (mrow + (mat >> 1) * 8) * 128;  // V matrices: tokens 8*(m>>1).., chunk 2*d+(m&1)
  }
};

// Abort-safe end of a producer: no copy into this CTA's shared memory may be in
// flight when the CTA exits.  A consumer whose wait gave up does not release
// its stage, so the producer's next wait for that slot runs out too and it
// stops issuing (no per-page check of the abort flag on the producer's
// critical path); every slot then has at most one use outstanding: the last
// min(STAGES, issued) stages issued.  Lane 0 waits, each wait bounded, for
// their full barriers (on the normal path these have completed or are about to).
template <int STAGES>
__device__ __forceinline__ void drain_issued_stages(const uint64_t* full_bar, int issued, int lane,
                                                    int32_t* err) {
  if (lane == 0) {
    for (int k = issued > STAGES ? issued - STAGES : 0; k < issued; ++k)
      if (!mbar_wait_bounded(smem_addr(&full_bar[k % STAGES]), (uint32_t)((k / STAGES) & 1))) {
        record_error(err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_DRAIN);
        break;
      }
  }
  __syncwarp();
}

// Online-softmax state of one (KV head, piece) in accumulator layout.
struct HeadState {
  float m0, m1, l0, l1;
  float acc[4][4];
  __device__ __forceinline__ void reset() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int d = 0; d < 4; ++d) acc[d][0] = acc[d][1] = acc[d][2] = acc[d][3] = 0.f;
  }
};

// Q^T operand fragments of the 4 query heads at `q_group` (head j at j * 64).
__device__ __forceinline__ void load_q_frags(const __nv_bfloat16* q_group, const TileLane& tl,
                                             uint32_t qb[4][2]) {
  const __nv_bfloat16* qrow = q_group + tl.tr * kHeadDim + 2 * tl.hc;
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    qb[k4][0] = tl.tr < kGroup ? __ldg(reinterpret_cast<const uint32_t*>(qrow + k4 * 16)) : 0u;
    qb[k4][1] = tl.tr < kGroup ? __ldg(reinterpret_cast<const uint32_t*>(qrow + k4 * 16 + 8)) : 0u;
  }
}

// Rows past the sequence end hold stale data: zero them in the V tile so that
// 0-probability rows cannot inject NaN/Inf into P.V.  Whole 128-byte rows, so
// the swizzle does not matter.
__device__ __forceinline__ void zero_stale_v_rows(unsigned char* vtile, int valid, int lane) {
  for (int idx = lane; idx < (kPage - valid) * 8; idx += 32) {
    const int r = valid + (idx >> 3);
    *reinterpret_cast<uint4*>(vtile + r * 128 + (idx & 7) * 16) = make_uint4(0, 0, 0, 0);
  }
}

// K and V fragments of one tile (shared addresses of its K and V tiles).
__device__ __forceinline__ void load_tile_frags(uint32_t ktile, uint32_t vtile, const TileLane& tl,
                                                uint32_t kf[4][4], uint32_t vf[4][4]) {
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4)
    ldmatrix_x4(ktile + tl.k_row + (((2 * k4 + tl.k_chunk) ^ tl.mrow) << 4), kf[k4][0], kf[k4][1],
                kf[k4][2], kf[k4][3]);
#pragma unroll
  for (int d = 0; d < 4; ++d)
    ldmatrix_x4_trans(vtile + tl.v_row + (((2 * d + tl.v_chunk) ^ tl.mrow) << 4), vf[d][0],
                      vf[d][1], vf[d][2], vf[d][3]);
}

// One tile into the online softmax: scores, (lazy) running max, BF16
// probabilities, P.V accumulation.  `valid` = tokens of the tile inside the
// sequence (rows >= valid are masked).
template <bool LAZY>
__device__ __forceinline__ void attend_tile(HeadState& st, const uint32_t kf[4][4],
                                            const uint32_t vf[4][4], const uint32_t qb[4][2],
                                            int valid, const TileLane& tl, float scale_log2) {
  // S^T = K Q^T, as two independent accumulation chains (channels 0-31, 32-63)
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
#pragma unroll
  for (int k4 = 0; k4 < 2; ++k4) {
    mma_bf16_16816(s0, s1, s2, s3, kf[k4][0], kf[k4][1], kf[k4][2], kf[k4][3], qb[k4][0],
                   qb[k4][1]);
    mma_bf16_16816(t0, t1, t2, t3, kf[k4 + 2][0], kf[k4 + 2][1], kf[k4 + 2][2], kf[k4 + 2][3],
                   qb[k4 + 2][0], qb[k4 + 2][1]);
  }
  float x0 = (s0 + t0) * scale_log2, x1 = (s1 + t1) * scale_log2;
  float x2 = (s2 + t2) * scale_log2, x3 = (s3 + t3) * scale_log2;
  if (valid < kPage) {
    if (tl.tr >= valid) x0 = x1 = -INFINITY;
    if (tl.tr + 8 >= valid) x2 = x3 = -INFINITY;
  }
  float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
  // LAZY keeps the running maximum unless a score beats it by more than
  // kLazyMargin: probabilities stay below 2^kLazyMargin, and the cross-lane max
  // and the rescale run only on a piece's first tile or on a new maximum.
  const bool grow = !LAZY || __any_sync(0xffffffffu, mx0 > st.m0 + kLazyMargin ||
                                                        mx1 > st.m1 + kLazyMargin);
  float al0 = 1.f, al1 = 1.f;
  if (grow) {
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(st.m0, mx0), mn1 = fmaxf(st.m1, mx1);
    al0 = fast_exp2(st.m0 - mn0);
    al1 = fast_exp2(st.m1 - mn1);
    st.m0 = mn0;
    st.m1 = mn1;
  }
  const uint32_t pa = pack_bf16x2(fast_exp2(x0 - st.m0), fast_exp2(x1 - st.m1));
  const uint32_t pb = pack_bf16x2(fast_exp2(x2 - st.m0), fast_exp2(x3 - st.m1));
  st.l0 = st.l0 * al0 + (bf16lo_to_f32(pa) + bf16lo_to_f32(pb));
  st.l1 = st.l1 * al1 + (bf16hi_to_f32(pa) + bf16hi_to_f32(pb));
  if (grow && __any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      st.acc[d][0] *= al0; st.acc[d][1] *= al1; st.acc[d][2] *= al0; st.acc[d][3] *= al1;
    }
  }
  // O^T += V^T P^T
  const uint32_t y0 = movmatrix_trans(pa), y1 = movmatrix_trans(pb);
#pragma unroll
  for (int d = 0; d < 4; ++d)
    mma_bf16_16816(st.acc[d][0], st.acc[d][1], st.acc[d][2], st.acc[d][3], vf[d][0], vf[d][1],
                   vf[d][2], vf[d][3], y0, y1);
}

// Sums the per-lane partial normalisers over the token rows.
__device__ __forceinline__ void reduce_l(HeadState& st) {
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, o);
    st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, o);
  }
}

// Destination of one (sequence, KV head group) output of 4 x 64 channels:
// this rank's rows at `local`, or, for a KV-head-shard gather, element `off`
// of every rank's gathered rows (peers[0 .. world), plain stores over NVLink).
struct OutGroup {
  __device__ __forceinline__ static __nv_bfloat16* peer(__nv_bfloat16* const* peers, int r) {
    return reinterpret_cast<__nv_bfloat16*>(
        __ldg(reinterpret_cast<const unsigned long long*>(peers) + r));
  }
  __nv_bfloat16* local;
  __nv_bfloat16* const* peers;
  size_t off;
  int world;
  __device__ __forceinline__ void store(int i, __nv_bfloat16 v) const {
    if (peers == nullptr) {
      local[i] = v;
      return;
    }
    for (int r = 0; r < world; ++r) peer(peers, r)[off + i] = v;
  }
  __device__ __forceinline__ void store16(int i, uint4 v) const {
    if (peers == nullptr) {
      *reinterpret_cast<uint4*>(local + i) = v;
      return;
    }
    for (int r = 0; r < world; ++r) *reinterpret_cast<uint4*>(peer(peers, r) + off + i) = v;
  }
};

__device__ __forceinline__ OutGroup local_out(__nv_bfloat16* group) {
  return OutGroup{group, nullptr, 0, 1};
}

// Normalised BF16 output of a whole sequence for the 4 query heads of `out`.
__device__ __forceinline__ void write_output(const HeadState& st, const OutGroup& out,
                                             const TileLane& tl) {
  if (tl.hc >= 2) return;  // columns 4-7 are padding
  const int h0 = 2 * tl.hc, h1 = 2 * tl.hc + 1;
  const float inv0 = st.l0 > 0.f ? 1.f / st.l0 : 0.f, inv1 = st.l1 > 0.f ? 1.f / st.l1 : 0.f;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int ch = 16 * d + tl.tr;
    out.store(h0 * kHeadDim + ch, __float2bfloat16_rn(st.acc[d][0] * inv0));
    out.store(h1 * kHeadDim + ch, __float2bfloat16_rn(st.acc[d][1] * inv1));
    out.store(h0 * kHeadDim + ch + 8, __float2bfloat16_rn(st.acc[d][2] * inv0));
    out.store(h1 * kHeadDim + ch + 8, __float2bfloat16_rn(st.acc[d][3] * inv1));
  }
}

// Unnormalised partial (m[4], l[4], O[4][64]) of one piece into `part`.
__device__ __forceinline__ void write_partial(const HeadState& st, float* part,
                                              const TileLane& tl) {
  if (tl.hc >= 2) return;
  const int h0 = 2 * tl.hc, h1 = 2 * tl.hc + 1;
  if (tl.tr == 0) {
    part[h0] = st.m0;
    part[h1] = st.m1;
    part[kGroup + h0] = st.l0;
    part[kGroup + h1] = st.l1;
  }
  float* po = part + 2 * kGroup;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    const int ch = 16 * d + tl.tr;
    po[h0 * kHeadDim + ch] = st.acc[d][0];
    po[h1 * kHeadDim + ch] = st.acc[d][1];
    po[h0 * kHeadDim + ch + 8] = st.acc[d][2];
    po[h1 * kHeadDim + ch + 8] = st.acc[d][3];
  }
}

// Page ranges: the T pages of a step cut into R contiguous ranges
// [floor(rT/R), floor((r+1)T/R)); range_of_page gives the range holding page p.
__device__ __forceinline__ int range_of_page(long long p, long long T, long long R) {
  return (int)(((p + 1) * R - 1) / T);
}
__device__ __forceinline__ int range_start(long long r, long long T, long long R) {
  return (int)(r * T / R);
}
// Partial slot of sequence [first, end) in range r: slot 2r when the sequence
// started at or before the range, 2r + 1 otherwise.
__device__ __forceinline__ int partial_slot(int r, int first, long long T, long long R) {
  return r * 2 + (range_start(r, T, R) < first ? 1 : 0);
}

// Merges the partial pieces of sequence [first, end) for KV head group g from
// the slots of ranges r0..r1 (lane -> query head lane/8 of the group, channels
// (lane%8)*8 .. +7) and writes the normalised output to `out`.
// Phase A: lane j reads m[4], l[4] of pieces j, j + 32, ... (all in flight at
// once); the warp reduces the maxima and the normalisers.  Phase B: each lane
// sums its 8 channels over the pieces, loading piece j + 1 before folding j;
// piece j's weight comes from lane j % 32 by shuffle.  About 1 + n L2 round
// trips at most, n / 2 when loads overlap.
__device__ __forceinline__ const float* partial_of(const float* partials, int groups, int g, int r,
                                                   int r0, int first, long long T, long long R) {
  const int slot = (r == r0) ? partial_slot(r, first, T, R) : r * 2;
  return partials + ((size_t)slot * groups + g) * kPartialFloats;
}

__device__ __forceinline__ float pick(const float4& v, int h) {
  return h == 0 ? v.x : h == 1 ? v.y : h == 2 ? v.z : v.w;
}

// BATCH: pieces whose output partials one lane loads at once in Phase B; each
// kernel takes the largest that fits its register budget without spilling.
template <int BATCH>
__device__ __forceinline__ void combine_partials(const float* partials, int groups, int g,
                                                 int first, int end, long long T, long long R,
                                                 const OutGroup& out, int lane) {
  const int r0 = range_of_page(first, T, R), r1 = range_of_page(end - 1, T, R);
  const int n = r1 - r0 + 1;
  const int h = lane >> 3, d0 = (lane & 7) * 8;
  // Phase A: per-head maximum over all pieces.
  float4 M = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  for (int j = lane; j < n; j += 32) {
    const float4 m = __ldcg(reinterpret_cast<const float4*>(
        partial_of(partials, groups, g, r0 + j, r0, first, T, R)));
    M.x = fmaxf(M.x, m.x); M.y = fmaxf(M.y, m.y); M.z = fmaxf(M.z, m.z); M.w = fmaxf(M.w, m.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    M.x = fmaxf(M.x, __shfl_xor_sync(0xffffffffu, M.x, o));
    M.y = fmaxf(M.y, __shfl_xor_sync(0xffffffffu, M.y, o));
    M.z = fmaxf(M.z, __shfl_xor_sync(0xffffffffu, M.z, o));
    M.w = fmaxf(M.w, __shfl_xor_sync(0xffffffffu, M.w, o));
  }
  float4 ls = make_float4(0.f, 0.f, 0.f, 0.f);  // this lane's share of the normalisers
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  for (int base = 0; base < n; base += 32) {
    // Lane j: weights of piece base + j for the 4 heads (0 past the last piece).
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    if (base + lane < n) {
      const float* part = partial_of(partials, groups, g, r0 + base + lane, r0, first, T, R);
      const float4 m = __ldcg(reinterpret_cast<const float4*>(part));
      const float4 l = __ldcg(reinterpret_cast<const float4*>(part + kGroup));
      w.x = m.x == -INFINITY ? 0.f : exp2f(m.x - M.x);
      w.y = m.y == -INFINITY ? 0.f : exp2f(m.y - M.y);
      w.z = m.z == -INFINITY ? 0.f : exp2f(m.z - M.z);
      w.w = m.w == -INFINITY ? 0.f : exp2f(m.w - M.w);
      ls.x += w.x * l.x; ls.y += w.y * l.y; ls.z += w.z * l.z; ls.w += w.w * l.w;
    }
    // Phase B: this lane's 8 channels over the chunk, BATCH pieces' loads in
    // flight at once; piece j's weight comes from lane j by shuffle.
    const int cnt = min(32, n - base);
    for (int j0 = 0; j0 < cnt; j0 += BATCH) {
      float4 a[BATCH], b[BATCH];
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        a[k] = b[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j0 + k < cnt) {
          const float* src = partial_of(partials, groups, g, r0 + base + j0 + k, r0, first, T, R) +
                             2 * kGroup + h * kHeadDim + d0;
          a[k] = __ldcg(reinterpret_cast<const float4*>(src));
          b[k] = __ldcg(reinterpret_cast<const float4*>(src + 4));
        }
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const int j = min(j0 + k, 31);
        const float4 wj = make_float4(__shfl_sync(0xffffffffu, w.x, j), __shfl_sync(0xffffffffu, w.y, j),
                                      __shfl_sync(0xffffffffu, w.z, j), __shfl_sync(0xffffffffu, w.w, j));
        const float wh = j0 + k < cnt ? pick(wj, h) : 0.f;
        o[0] += wh * a[k].x; o[1] += wh * a[k].y; o[2] += wh * a[k].z; o[3] += wh * a[k].w;
        o[4] += wh * b[k].x; o[5] += wh * b[k].y; o[6] += wh * b[k].z; o[7] += wh * b[k].w;
      }
    }
  }
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) {
    ls.x += __shfl_xor_sync(0xffffffffu, ls.x, k);
    ls.y += __shfl_xor_sync(0xffffffffu, ls.y, k);
    ls.z += __shfl_xor_sync(0xffffffffu, ls.z, k);
    ls.w += __shfl_xor_sync(0xffffffffu, ls.w, k);
  }
  const float lsum = pick(ls, h);
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  uint4 packed;
  packed.x = pack_bf16x2(o[0] * inv, o[1] * inv);
  packed.y = pack_bf16x2(o[2] * inv, o[3] * inv);
  packed.z = pack_bf16x2(o[4] * inv, o[5] * inv);
  packed.w = pack_bf16x2(o[6] * inv, o[7] * inv);
  out.store16(h * kHeadDim + d0, packed);
}

// Publishes a partial piece; true in every lane when it is the last piece of
// its sequence to arrive (a counter per (sequence, KV head group), reset by
// the last arriver for the next launch; no waiting).
__device__ __forceinline__ bool publish_partial(const HeadState& st, float* partials, int* counters,
                                                int groups, int g, int s, int slot, int first,
                                                int end, long long T, long long R,
                                                const TileLane& tl, int lane) {
  write_partial(st, partials + ((size_t)slot * groups + g) * kPartialFloats, tl);
  __threadfence();
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    const int pieces = range_of_page(end - 1, T, R) - range_of_page(first, T, R) + 1;
    const int old = atomicAdd(counters + (size_t)s * groups + g, 1);
    last = (old == pieces - 1);
    if (last) {
      atomicExch(counters + (size_t)s * groups + g, 0);
      __threadfence();
    }
  }
  return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// Publishes a partial piece and, when it is the last of its sequence to arrive,
// merges all of them.
template <int BATCH>
__device__ __forceinline__ void finish_partial(const HeadState& st, float* partials, int* counters,
                                               int groups, int g, int s, int slot, int first,
                                               int end, long long T, long long R,
                                               const OutGroup& out, const TileLane& tl,
                                               int lane) {
  if (publish_partial(st, partials, counters, groups, g, s, slot, first, end, T, R, tl, lane))
    combine_partials<BATCH>(partials, groups, g, first, end, T, R, out, lane);
}

// combine_partials for a warp with shared memory to spare.  The warp copies
// the partials' output rows (1 KiB each, two cp.async instructions of 512
// contiguous bytes per piece) into `stage`, a round of up to `cap` pieces at
// once, so that a round costs one L2 round trip and no registers; the first
// round's copies go out before the maxima's loads (copies whose 32 source and
// 32 destination chunks are both contiguous issue fastest).  Lane L folds the
// piece's floats 8L .. 8L+7; lanes 4-7 of each 8 read their second 16 bytes
// first, so that each 8-lane phase of a 16-byte shared load covers all 32
// banks.
// The piece weights pass through a 32-entry table in `stage` instead of
// shuffles.  The maxima, weights, normalisers and the fold of the rows in
// piece order are combine_partials' own operations: the output is
// bit-identical whichever of the two a sequence's last arriver runs.
// `stage`: 16-byte aligned, 512 + 1024 cap bytes; cap >= 1.
__device__ __forceinline__ void combine_partials_staged(const float* partials, int groups, int g,
                                                        int first, int end, long long T,
                                                        long long R, const OutGroup& out,
                                                        int lane, float* stage, int cap) {
  const int r0 = range_of_page(first, T, R), r1 = range_of_page(end - 1, T, R);
  const int n = r1 - r0 + 1;
  const int h = lane >> 3, d0 = (lane & 7) * 8;
  const int slot0 = partial_slot(r0, first, T, R);
  auto piece = [&](int j) {
    return partials + ((size_t)(j == 0 ? slot0 : 2 * (r0 + j)) * groups + g) * kPartialFloats;
  };
  float4* wtab = reinterpret_cast<float4*>(stage);         // weights of a chunk's 32 pieces
  float* rows = stage + 128;                                 // [cap][256 floats]
  const uint32_t copy_dst = smem_addr(rows) + 16u * lane;  // + 1024 i (piece), + 512
  auto issue = [&](int j0, int cnt) {  // output rows of pieces j0 .. j0 + cnt - 1
    for (int i = 0; i < cnt; ++i) {
      const float* src = piece(j0 + i) + 2 * kGroup + 4 * lane;
      cp_async_16(copy_dst + 1024u * i, src);
      cp_async_16(copy_dst + 1024u * i + 512u, src + 128);
    }
  };
  int lo = 0, hi = min(cap, n);  // pieces [lo, hi) are (being) staged
  issue(0, hi);
  // Maxima over all pieces, loaded directly while the copies are in flight;
  // lane j keeps m, l of piece j for the first 32 pieces' weights.
  float4 m_lane = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  float4 l_lane = make_float4(0.f, 0.f, 0.f, 0.f);
  if (lane < n) {
    m_lane = __ldcg(reinterpret_cast<const float4*>(piece(lane)));
    l_lane = __ldcg(reinterpret_cast<const float4*>(piece(lane) + kGroup));
  }
  float4 M = m_lane;
#pragma unroll 4
  for (int j = lane + 32; j < n; j += 32) {
    const float4 m = __ldcg(reinterpret_cast<const float4*>(piece(j)));
    M.x = fmaxf(M.x, m.x); M.y = fmaxf(M.y, m.y); M.z = fmaxf(M.z, m.z); M.w = fmaxf(M.w, m.w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    M.x = fmaxf(M.x, __shfl_xor_sync(0xffffffffu, M.x, o));
    M.y = fmaxf(M.y, __shfl_xor_sync(0xffffffffu, M.y, o));
    M.z = fmaxf(M.z, __shfl_xor_sync(0xffffffffu, M.z, o));
    M.w = fmaxf(M.w, __shfl_xor_sync(0xffffffffu, M.w, o));
  }
  float4 ls = make_float4(0.f, 0.f, 0.f, 0.f);  // this lane's share of the normalisers
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  const int sw = (lane >> 2) & 1;             // read order of this lane's two halves
  const float* my_x = rows + 8 * lane + 4 * sw;  // read first
  const float* my_y = rows + 8 * lane + 4 - 4 * sw;
  for (int base = 0; base < n; base += 32) {
    // m, l of the next chunk's pieces, in flight while this chunk folds
    float4 m_next = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    float4 l_next = make_float4(0.f, 0.f, 0.f, 0.f);
    if (base + 32 + lane < n) {
      m_next = __ldcg(reinterpret_cast<const float4*>(piece(base + 32 + lane)));
      l_next = __ldcg(reinterpret_cast<const float4*>(piece(base + 32 + lane) + kGroup));
    }
    // Lane j: weights of piece base + j for the 4 heads (0 past the last piece).
    float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
    if (base + lane < n) {
      const float4 m = m_lane, l = l_lane;
      w.x = m.x == -INFINITY ? 0.f : exp2f(m.x - M.x);
      w.y = m.y == -INFINITY ? 0.f : exp2f(m.y - M.y);
      w.z = m.z == -INFINITY ? 0.f : exp2f(m.z - M.z);
      w.w = m.w == -INFINITY ? 0.f : exp2f(m.w - M.w);
      ls.x += w.x * l.x; ls.y += w.y * l.y; ls.z += w.z * l.z; ls.w += w.w * l.w;
    }
    __syncwarp();  // the previous chunk's weights are read
    wtab[lane] = w;
    __syncwarp();
    const float* wcol = reinterpret_cast<const float*>(wtab) + h;  // piece jj's weight at 4 jj
    const int cnt = min(32, n - base);
    int jj = 0;
    while (jj < cnt) {
      const int j = base + jj;
      if (j == hi) {  // the next round, once every lane has read this one
        __syncwarp();
        lo = j;
        hi = min(j + cap, n);
        issue(lo, hi - lo);
      }
      cp_async_wait_all();
      __syncwarp();
      const int stop = min(cnt, hi - base);  // pieces of this chunk in the staged round
#pragma unroll 4
      for (; jj < stop; ++jj) {
        const float wh = wcol[4 * jj];
        const float4 x = *reinterpret_cast<const float4*>(my_x + 256 * (base + jj - lo));
        const float4 y = *reinterpret_cast<const float4*>(my_y + 256 * (base + jj - lo));
        const float4 a = sw ? y : x, b = sw ? x : y;  // channels d0 .. +3, d0 + 4 .. +7
        o[0] += wh * a.x; o[1] += wh * a.y; o[2] += wh * a.z; o[3] += wh * a.w;
        o[4] += wh * b.x; o[5] += wh * b.y; o[6] += wh * b.z; o[7] += wh * b.w;
      }
    }
    m_lane = m_next;
    l_lane = l_next;
  }
#pragma unroll
  for (int k = 16; k > 0; k >>= 1) {
    ls.x += __shfl_xor_sync(0xffffffffu, ls.x, k);
    ls.y += __shfl_xor_sync(0xffffffffu, ls.y, k);
    ls.z += __shfl_xor_sync(0xffffffffu, ls.z, k);
    ls.w += __shfl_xor_sync(0xffffffffu, ls.w, k);
  }
  const float lsum = pick(ls, h);
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  uint4 packed;
  packed.x = pack_bf16x2(o[0] * inv, o[1] * inv);
  packed.y = pack_bf16x2(o[2] * inv, o[3] * inv);
  packed.z = pack_bf16x2(o[4] * inv, o[5] * inv);
  packed.w = pack_bf16x2(o[6] * inv, o[7] * inv);
  out.store16(h * kHeadDim + d0, packed);
}

}  // namespace tvp
