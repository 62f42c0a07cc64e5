// K3 — paged causal prefill attention, reading K and V from the pages.
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
// positions q_pos0[s], q_pos0[s] + 1, ...  A CTA takes one (16-query tile,
// sequence, KV head): a producer warp streams the sequence's pages 0 .. the
// tile's last position (one 2 KiB K box and one V box of this KV head per
// page, the decode kernels' tensor maps and 128-byte swizzle), and 4 consumer
// warps, one per query head of the GQA group, share every page.  Per page a
// warp forms, for each of its 16-query m-tiles (sharing the page's K and V
// fragments), S = Q K^T (16 queries x 16 keys) and O += P V (16 x 64) with
// mma.m16n8k16 (BF16 in, FP32 accumulate), P going from the S accumulators to
// the A operand without a shuffle, and keeps an online base-2 softmax per row
// over BF16-rounded scores, with a lazy running max.
#include "tvp_tile.cuh"

namespace tvp {

namespace {

constexpr int kPrefillStages = 6;
constexpr int kPrefillStage = 2 * kTileBytes;  // K tile, then V tile (4 KiB)
// 16-row m-tiles per warp.  Two (each page's K/V fragments serving 32 queries)
// measured slower on B200 than one: 188 vs 150 us for 4 x 1024 prompts, with
// half the CTAs and two instead of three CTAs per SM.
constexpr int kPrefillMTiles = 1;
constexpr int kQTile = 16 * kPrefillMTiles;    // query tokens per CTA
constexpr int kPrefillThreads = (kGroup + 1) * 32;

constexpr size_t prefill_smem_bytes() {
  return 1024 /* alignment slack */ + (size_t)kPrefillStages * kPrefillStage +
         2 * kPrefillStages * 8 + (kPrefillStages + 4) * 4;
}

// MT: 16-row m-tiles per warp; every K/V fragment loaded from a page serves MT.
template <int MT>
__global__ void __launch_bounds__(kPrefillThreads)
    paged_prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap k_map,
                         const __grid_constant__ CUtensorMap v_map) {
  extern __shared__ unsigned char smem_raw[];
  // 128-byte swizzled tiles need 1 KiB alignment: round the window up.
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t smem_base = smem_addr(smem);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kPrefillStages * kPrefillStage);
  uint64_t* empty_bar = full_bar + kPrefillStages;
  int* stage_ok = reinterpret_cast<int*>(empty_bar + kPrefillStages);
  volatile int* abort_flag = stage_ok + kPrefillStages;

  const int s = blockIdx.y, g = blockIdx.z;
  const int q_begin = __ldg(p.cu_q + s), q_end = __ldg(p.cu_q + s + 1);
  // Tiles run last-first: under causality the last tiles stream the most pages,
  // so starting them first shortens the launch's tail.
  const int tile = gridDim.x - 1 - blockIdx.x;
  const int tok0 = q_begin + tile * kQTile;
  if (tok0 >= q_end) return;  // this sequence has fewer tiles
  const int count = min(kQTile, q_end - tok0);
  const int pos0 = __ldg(p.q_pos0 + s) + tile * kQTile;  // position of the tile's row 0
  const int pos_last = pos0 + count - 1;
  if (pos0 < 0 || pos_last / kPage >= p.table_stride) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_TOKEN);
    return;
  }
  const int n_pages = pos_last / kPage + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPrefillStages; ++i) {
      mbar_init(smem_addr(&full_bar[i]), 1);
      mbar_init(smem_addr(&empty_bar[i]), kGroup);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kGroup) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      prefetch_tensor_map(&k_map);
      prefetch_tensor_map(&v_map);
    }
    int stage = 0, issued = 0;
    uint32_t empty_parity = 1;
    int next_phys = __ldg(p.tables + (size_t)s * p.table_stride);
    for (int j = 0; j < n_pages; ++j) {
      const int phys = next_phys;
      if (j + 1 < n_pages) next_phys = __ldg(p.tables + (size_t)s * p.table_stride + j + 1);
      if (j >= kPrefillStages) {
        int timed_out = 0;
        if (lane == 0) timed_out = !mbar_wait_bounded(smem_addr(&empty_bar[stage]), empty_parity);
        if (__shfl_sync(0xffffffffu, timed_out, 0)) {
          if (lane == 0) {
            *abort_flag = 1;
            record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_EMPTY);
          }
          break;
        }
      }
      const bool ok = phys >= 0 && phys < p.num_pages;
      const uint32_t full = smem_addr(&full_bar[stage]);
      if (lane == 0) {
        stage_ok[stage] = ok ? 1 : 0;
        if (!ok) record_error(p.err, TVP_DEVERR_BAD_PAGE);
        mbar_arrive_expect_tx(full, ok ? (uint32_t)kPrefillStage : 0u);
      }
      __syncwarp();
      if (ok && lane < 2) {
        const int y = (int)(p.layer_row_base + (long long)phys * kPage);
        tma_load_2d(smem_base + stage * kPrefillStage + lane * kTileBytes,
                    lane == 0 ? &k_map : &v_map, g * kHeadDim, y, full);
      }
      issued = j + 1;
      if (++stage == kPrefillStages) {
        stage = 0;
        empty_parity ^= 1u;
      }
    }
    drain_issued_stages<kPrefillStages>(full_bar, issued, lane, p.err);
    return;
  }

  // ------------------------------ consumers -------------------------------
  const int hq = g * kGroup + warp;  // query head of this warp
  const int qdim = p.kv_heads * kGroup * kHeadDim;
  const int r = lane >> 2, c = lane & 3;  // accumulator rows r, r + 8; column pair 2c
  const int mrow = lane & 7, mat = lane >> 3;

  // Per m-tile mt (query rows 16 mt .. 16 mt + 15 of the CTA's tile):
  // Q A-operand fragments, O accumulators, running max and normaliser of rows
  // 16 mt + r (index 0) and 16 mt + r + 8 (index 1).
  uint32_t qa[MT][4][4];
  float o[MT][8][4];
  float m[MT][2], l[MT][2];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int ra = 16 * mt + r, rb = ra + 8;
    const __nv_bfloat16* qr = p.q + (size_t)(tok0 + ra) * qdim + hq * kHeadDim + 2 * c;
    const __nv_bfloat16* qr8 = qr + (size_t)8 * qdim;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      qa[mt][ks][0] = ra < count ? __ldg(reinterpret_cast<const uint32_t*>(qr + ks * 16)) : 0u;
      qa[mt][ks][1] = rb < count ? __ldg(reinterpret_cast<const uint32_t*>(qr8 + ks * 16)) : 0u;
      qa[mt][ks][2] = ra < count ? __ldg(reinterpret_cast<const uint32_t*>(qr + ks * 16 + 8)) : 0u;
      qa[mt][ks][3] = rb < count ? __ldg(reinterpret_cast<const uint32_t*>(qr8 + ks * 16 + 8)) : 0u;
    }
#pragma unroll
    for (int d = 0; d < 8; ++d) o[mt][d][0] = o[mt][d][1] = o[mt][d][2] = o[mt][d][3] = 0.f;
    m[mt][0] = m[mt][1] = -INFINITY;
    l[mt][0] = l[mt][1] = 0.f;
  }

  // ldmatrix row addresses: K (non-transposed, B operand of S = Q K^T):
  // matrix i = keys 8 (i >> 1) .., chunk 2 ks + (i & 1); V (transposed, B
  // operand of O = P V): matrix i = keys 8 (i & 1) .., chunk 2 dp + (i >> 1).
  const int k_key = (mat >> 1) * 8 + mrow, k_chunk = mat & 1;
  const int v_key = (mat & 1) * 8 + mrow, v_chunk = mat >> 1;

  int stage = 0;
  uint32_t parity = 0;
  for (int j = 0; j < n_pages; ++j) {
    bool ready = false;
    if (!*abort_flag) ready = mbar_wait_bounded(smem_addr(&full_bar[stage]), parity);
    ready = __all_sync(0xffffffffu, ready);
    if (!ready && lane == 0 && !*abort_flag) {
      *abort_flag = 1;
      record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
    }
    const bool have = ready && stage_ok[stage];
    const uint32_t kt = smem_base + stage * kPrefillStage, vt = kt + kTileBytes;
    // Rows of the last page past pos_last hold stale data: warp 0 zeroes them in
    // the V tile before any warp reads it (all 4 warps meet at the barrier).
    if (j == n_pages - 1) {
      if (have && warp == 0) {
        zero_stale_v_rows(smem + stage * kPrefillStage + kTileBytes, pos_last % kPage + 1, lane);
        fence_proxy_async_smem();
      }
      named_barrier_sync(1, kGroup * 32);
    }
    uint32_t kb[4][4], vb[4][4];
    if (have) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
        ldmatrix_x4(kt + k_key * 128 + (((2 * ks + k_chunk) ^ (k_key & 7)) << 4), kb[ks][0],
                    kb[ks][1], kb[ks][2], kb[ks][3]);
#pragma unroll
      for (int dp = 0; dp < 4; ++dp)
        ldmatrix_x4_trans(vt + v_key * 128 + (((2 * dp + v_chunk) ^ (v_key & 7)) << 4),
                          vb[dp][0], vb[dp][1], vb[dp][2], vb[dp][3]);
    }
    __syncwarp();
    if (ready && lane == 0) mbar_arrive(smem_addr(&empty_bar[stage]));
    if (have) {
      const int key0 = j * kPage + 2 * c;  // keys key0, key0 + 1, key0 + 8, key0 + 9
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        // S = Q K^T: n-tile 0 = keys 0-7, n-tile 1 = keys 8-15 of the page.
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          mma_bf16_16816(s0[0], s0[1], s0[2], s0[3], qa[mt][ks][0], qa[mt][ks][1], qa[mt][ks][2],
                         qa[mt][ks][3], kb[ks][0], kb[ks][1]);
          mma_bf16_16816(s1[0], s1[1], s1[2], s1[3], qa[mt][ks][0], qa[mt][ks][1], qa[mt][ks][2],
                         qa[mt][ks][3], kb[ks][2], kb[ks][3]);
        }
        float x[8] = {s0[0], s0[1], s1[0], s1[1], s0[2], s0[3], s1[2], s1[3]};
        const int qpos_a = pos0 + 16 * mt + r, qpos_b = qpos_a + 8;
        // Scores are rounded to BF16 where the reference rounds them (its score
        // GEMM writes BF16, src/model/attention.cu:10-51), then taken to base 2.
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int key = key0 + (e & 1) + ((e >> 1) & 1) * 8;
          const int qpos = e < 4 ? qpos_a : qpos_b;
          x[e] = key <= qpos
                     ? __bfloat162float(__float2bfloat16_rn(x[e] * p.scale)) * 1.4426950408889634f
                     : -INFINITY;
        }
        float mx_a = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
        float mx_b = fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7]));
        // Lazy running max (as in the decode kernels): the row maxima are
        // reduced and O rescaled only when a score beats a row's max by more
        // than kLazyMargin, so probabilities stay below 2^kLazyMargin.
        float al_a = 1.f, al_b = 1.f;
        if (__any_sync(0xffffffffu, mx_a > m[mt][0] + kLazyMargin || mx_b > m[mt][1] + kLazyMargin)) {
#pragma unroll
          for (int sh = 1; sh < 4; sh <<= 1) {
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, sh));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, sh));
          }
          const float mn_a = fmaxf(m[mt][0], mx_a), mn_b = fmaxf(m[mt][1], mx_b);
          al_a = m[mt][0] == -INFINITY ? 0.f : fast_exp2(m[mt][0] - mn_a);
          al_b = m[mt][1] == -INFINITY ? 0.f : fast_exp2(m[mt][1] - mn_b);
          m[mt][0] = mn_a;
          m[mt][1] = mn_b;
        }
        // rows that have seen no key yet keep a zero base (no inf - inf)
        const float base_a = m[mt][0] == -INFINITY ? 0.f : m[mt][0];
        const float base_b = m[mt][1] == -INFINITY ? 0.f : m[mt][1];
        // P as the A operand of O += P V (keys 0-7 then 8-15 of the page)
        uint32_t pa[4];
        pa[0] = pack_bf16x2(fast_exp2(x[0] - base_a), fast_exp2(x[1] - base_a));
        pa[1] = pack_bf16x2(fast_exp2(x[4] - base_b), fast_exp2(x[5] - base_b));
        pa[2] = pack_bf16x2(fast_exp2(x[2] - base_a), fast_exp2(x[3] - base_a));
        pa[3] = pack_bf16x2(fast_exp2(x[6] - base_b), fast_exp2(x[7] - base_b));
        l[mt][0] = l[mt][0] * al_a + (bf16lo_to_f32(pa[0]) + bf16hi_to_f32(pa[0]) +
                                      bf16lo_to_f32(pa[2]) + bf16hi_to_f32(pa[2]));
        l[mt][1] = l[mt][1] * al_b + (bf16lo_to_f32(pa[1]) + bf16hi_to_f32(pa[1]) +
                                      bf16lo_to_f32(pa[3]) + bf16hi_to_f32(pa[3]));
        if (__any_sync(0xffffffffu, al_a != 1.f || al_b != 1.f)) {
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            o[mt][d][0] *= al_a; o[mt][d][1] *= al_a; o[mt][d][2] *= al_b; o[mt][d][3] *= al_b;
          }
        }
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {
          mma_bf16_16816(o[mt][2 * dp][0], o[mt][2 * dp][1], o[mt][2 * dp][2], o[mt][2 * dp][3],
                         pa[0], pa[1], pa[2], pa[3], vb[dp][0], vb[dp][1]);
          mma_bf16_16816(o[mt][2 * dp + 1][0], o[mt][2 * dp + 1][1], o[mt][2 * dp + 1][2],
                         o[mt][2 * dp + 1][3], pa[0], pa[1], pa[2], pa[3], vb[dp][2], vb[dp][3]);
        }
      }
    }
    if (++stage == kPrefillStages) {
      stage = 0;
      parity ^= 1u;
    }
  }

  // Normalise and store rows 16 mt + r, + 8 (channels 8 d + 2 c, + 1).
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float la = l[mt][0], lb = l[mt][1];
#pragma unroll
    for (int sh = 1; sh < 4; sh <<= 1) {
      la += __shfl_xor_sync(0xffffffffu, la, sh);
      lb += __shfl_xor_sync(0xffffffffu, lb, sh);
    }
    const float inv_a = la > 0.f ? 1.f / la : 0.f, inv_b = lb > 0.f ? 1.f / lb : 0.f;
    const int ra = 16 * mt + r;
    __nv_bfloat16* out_a = p.out + (size_t)(tok0 + ra) * qdim + hq * kHeadDim + 2 * c;
    __nv_bfloat16* out_b = out_a + (size_t)8 * qdim;
#pragma unroll
    for (int d = 0; d < 8; ++d) {
      if (ra < count)
        *reinterpret_cast<uint32_t*>(out_a + 8 * d) =
            pack_bf16x2(o[mt][d][0] * inv_a, o[mt][d][1] * inv_a);
      if (ra + 8 < count)
        *reinterpret_cast<uint32_t*>(out_b + 8 * d) =
            pack_bf16x2(o[mt][d][2] * inv_b, o[mt][d][3] * inv_b);
    }
  }
}

}  // namespace

cudaError_t launch_paged_prefill(const PrefillParams& p, long long pool_rows, int max_q_len,
                                 int num_seqs, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(paged_prefill_kernel<kPrefillMTiles>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)prefill_smem_bytes());
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  CUtensorMap k_map, v_map;
  if (!pool_tensor_map(p.k_pool, pool_rows, p.kv_heads, &k_map) ||
      !pool_tensor_map(p.v_pool, pool_rows, p.kv_heads, &v_map))
    return cudaErrorInvalidValue;
  const dim3 grid((max_q_len + kQTile - 1) / kQTile, num_seqs, p.kv_heads);
  paged_prefill_kernel<kPrefillMTiles>
      <<<grid, kPrefillThreads, prefill_smem_bytes(), stream>>>(p, k_map, v_map);
  return cudaGetLastError();
}

}  // namespace tvp
