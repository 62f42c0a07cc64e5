// K2 — fused GQA paged decode attention with a split-K (flash-decoding)
// combine, and the per-step plan kernel.
//
// Replaces the reference's decode attention (src/model/paged_transformer.cu:85-94):
// gatherPagedKernel copies every page of K into a contiguous view, 32 cuBLAS
// GEMVs per row compute BF16 scores, 32 softmax launches per row normalise
// them, a second gather copies V and 32 more GEMVs form the output
// (src/model/paged_attention.cu:102-161, src/model/attention.cu:53-142,
// src/model/softmax.cu:6-72).  Here one persistent launch reads every page
// once, in place.
//
// Work split.  The plan kernel turns the attended lengths into page prefix
// sums cu[0..B].  The T = cu[B] pages of the step, laid end to end, are cut
// into C = min(gridDim.x, T) contiguous ranges of floor/ceil(T / C) pages, one
// per CTA, so every CTA streams the same number of pages whatever the length
// mix (CTAs past C have no pages).  A range
// covers whole sequences ("complete pieces", finalised in place) and at most
// two sequence fragments at its ends ("partial pieces"); partials go to the
// workspace and the last CTA to finish a sequence merges them (a counter per
// (sequence, KV head), no waiting).
//
// CTA layout: one producer warp and SETS x 8 consumer warps.  The producer
// streams one page per stage into shared memory with two tiled TMA loads, one
// box {64 channels x 16 tokens x 8 heads} of K and one of V, through 3-D
// tensor maps that view a pool's rows of 512 channels as (channel, token,
// head).  Each box lands as eight head-major 2 KiB tiles, 128-byte swizzled so
// that the consumers' ldmatrix reads of 8 tokens hit 8 different bank groups.
// (One 2-D box per head and page, sixteen TMA instructions per page, left the
// producer issue-bound at ~0.84 of the HBM rate; one bulk copy per 1 KiB token
// row streamed at only ~4.4 TB/s.)
// Consumer warp g of set s owns KV head g on the pages i of each sequence
// piece with i % SETS == s (the sets' states are merged at the piece's end).
// With an odd number of stages consecutive rounds of a stage go to different
// sets, so each set gates its stage waits on the stage's round tag.
// Per page it forms S^T = K_g Q_g^T (16 tokens x 8 query columns, 4 real) and
// O^T += V_g^T P^T with mma.m16n8k16 (BF16 in, FP32 accumulate), running an
// online softmax in base 2 on the accumulator fragments; P^T is turned from
// accumulator layout into operand layout with movmatrix.
#include <cudaTypedefs.h>

#include "tvp_tile.cuh"

namespace tvp {

constexpr int kMergeFields = 2;  // per-lane values exchanged per merge round (see below)
constexpr int kTailBarrier = 1 + kMaxKvHeads;  // all consumer warps (ids 1..8: the set merges)


// ---------------------------------------------------------------------------
// Plan: cu[b] = sum_{i<b} ceil(L_i / 16), cta_start[c] = {s, cu[s], cu[s + 1]}
// for the sequence s holding CTA c's first page, header, counters = 0.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024)
    decode_plan_kernel(const int32_t* __restrict__ lens, int batch, int table_stride,
                       int num_ctas, int groups, int32_t* header, int32_t* cu, int4* cta_start,
                       int32_t* counters, int32_t* err) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < batch; base += 1024) {
    const int i = base + tid;
    int L = i < batch ? lens[i] : 0;
    if (i < batch && (L < 0 || L > table_stride * kPage)) {
      record_error(err, TVP_DEVERR_BAD_LENGTH);
      L = L < 0 ? 0 : table_stride * kPage;
    }
    const int pages = (L + kPage - 1) / kPage;
    int x = pages;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    if (i < batch) cu[i] = carry + (warp > 0 ? warp_sums[warp - 1] : 0) + x - pages;
    __syncthreads();
    if (tid == 0) carry += warp_sums[31];
    __syncthreads();
  }
  // CTA c of C = min(num_ctas, T) starts at page floor(c T / C), which lies in
  // sequence s exactly when ceil(cu[s] C / T) <= c < ceil(cu[s + 1] C / T):
  // every sequence writes its own CTAs (empty sequences none).  cu[] was
  // written by this block before the last barrier of the scan: plain loads.
  const long long T = carry;
  const long long C = T < num_ctas ? T : num_ctas;
  for (int s = tid; s < batch && C > 0; s += blockDim.x) {
    const long long a = cu[s];
    const long long b = s + 1 < batch ? (long long)cu[s + 1] : T;
    for (long long c = (a * C + T - 1) / T; c < (b * C + T - 1) / T; ++c)
      cta_start[c] = make_int4(s, (int)a, (int)b, 0);
  }
  if (tid == 0) {
    cu[batch] = carry;
    header[0] = kPlanMagic;
    header[1] = batch;
    header[2] = num_ctas;
    header[3] = groups;
  }
  for (int i = tid; i < batch * groups; i += blockDim.x) counters[i] = 0;
}

template <int STAGES, int SETS, bool LAZY, bool REGSPLIT = false>
__global__ void __launch_bounds__(decode_threads<SETS, REGSPLIT>(), 1)
    paged_decode_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap k_map,
                        const __grid_constant__ CUtensorMap v_map) {
  // The 128-byte swizzle pattern repeats every 1 KiB: stage tiles must start
  // 1 KiB aligned.  The dynamic shared window of this kernel (no static shared
  // memory) starts 1 KiB aligned; a launch where it does not reports an error
  // instead of running the copies.
  extern __shared__ __align__(1024) unsigned char smem[];
  // The plan's header, the step's page count and this CTA's start record,
  // loaded together (one round trip) before anything depends on them.  The
  // record is read only when the header matches this launch and the CTA
  // takes pages; the workspace holds one record per CTA of the grid.
  const int4 hdr = __ldg(reinterpret_cast<const int4*>(p.header));
  const int total_pages = __ldg(p.cu + p.batch);
  const int4 start = __ldg(p.cta_start + blockIdx.x);
  if (smem_addr(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_SMEM_ALIGN);
    return;
  }
  const bool plan_ok = (hdr.x == kPlanMagic && hdr.y == p.batch && hdr.z == (int)gridDim.x &&
                        hdr.w == kMaxKvHeads);
  if (!plan_ok) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_PLAN);
    return;
  }
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  // Per stage: ((round + 1) << 1) | (page id in range), written by the
  // producer before it issues the round (see stage_tag_wait).
  volatile int* stage_tag = reinterpret_cast<int*>(empty_bar + STAGES);
  volatile int* abort_flag = stage_tag + STAGES;
  // Set-merge scratch (used with two consumer sets only), 16-byte aligned.
  [[maybe_unused]] float* const merge = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem + STAGES * kStageBytes + 2 * STAGES * 8 +
                                   (STAGES + 4) * 4) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kMaxKvHeads);
      stage_tag[s] = 0;
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  // Only min(grid, T) CTAs take pages, so that every range holds at least one
  // page and the pieces of a sequence are exactly the CTAs c0..c1 it spans.
  const long long T = total_pages;
  const long long C = T < (long long)gridDim.x ? T : (long long)gridDim.x;
  const long long c = blockIdx.x;
  const int p_begin = c < C ? (int)(c * T / C) : 0;
  const int p_end = c < C ? (int)((c + 1) * T / C) : 0;
  const uint32_t smem_base = smem_addr(smem);

  // First sequence of the range (the s with cu[s] <= p_begin < cu[s + 1]) and
  // its page span, from the plan.
  const int s0 = p_begin < p_end ? start.x : 0;

  if (warp >= SETS * kMaxKvHeads) {
    // ------------------------------ producer ------------------------------
    if (REGSPLIT) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
      if (warp != SETS * kMaxKvHeads) return;  // the rest of the producer warpgroup idles
    }
    if (lane == 0) {
      prefetch_tensor_map(&k_map);
      prefetch_tensor_map(&v_map);
    }
    // The page walk (sequence s, its first page and end) lives in registers
    // and the next page id is loaded one iteration ahead, so nothing but the
    // empty-slot wait sits between a slot being freed and its refill.
    int s = s0;
    int seq_first = start.y, seq_end = start.z;  // used only when the CTA takes pages
    int next_phys = p_begin < p_end
                        ? __ldg(p.tables + (size_t)s * p.table_stride + (p_begin - seq_first))
                        : 0;
    int stage = 0, round = 0, issued = 0;
    uint32_t empty_parity = 1;  // parity of the previous round of each slot
    // Launched as a programmatic dependent launch: the kernel before this one
    // in the stream (the append of the step's new token) may still be
    // running.  It writes pages and q, never the plan or the block tables, so
    // the walk's first loads above go out now and the wait comes before the
    // first page copy.
    bool waited = false;
    for (int pg = p_begin, kk = 0; pg < p_end; ++pg, ++kk) {
      const int phys = next_phys;
      if (pg + 1 < p_end) {
        while (pg + 1 >= seq_end) {
          ++s;
          seq_first = seq_end;
          seq_end = __ldg(p.cu + s + 1);
        }
        next_phys = __ldg(p.tables + (size_t)s * p.table_stride + (pg + 1 - seq_first));
      }
      if (kk >= STAGES) {
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
      if (!waited) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // the previous grid's page writes, seen by this thread's copies
        asm volatile("fence.proxy.async.global;" ::: "memory");
        waited = true;
      }
      const bool ok = phys >= 0 && phys < p.num_pages;
      const uint32_t full = smem_addr(&full_bar[stage]);
      if (lane == 0) {
        stage_tag[stage] = ((round + 1) << 1) | (ok ? 1 : 0);
        if (!ok) record_error(p.err, TVP_DEVERR_BAD_PAGE);
        mbar_arrive_expect_tx(full, ok ? (uint32_t)kStageBytes : 0u);
      }
      __syncwarp();
      if (ok && lane < 2) {
        // lane 0: the page's K, lane 1: its V, each as one box of all 8 heads
        // (16 KiB, landing as 8 head-major 2 KiB tiles).  One TMA instruction
        // per 2 KiB head tile took ~0.6 us per page to issue, longer than the
        // page takes to stream at the HBM rate; two take ~0.1 us.
        const uint32_t dst = smem_base + stage * kStageBytes + lane * kMaxKvHeads * kTileBytes;
        tma_load_3d(dst, lane == 0 ? &k_map : &v_map, 0,
                    (int)(p.layer_row_base + (long long)phys * kPage), 0, full);
      }
      issued = kk + 1;
      if (++stage == STAGES) {
        stage = 0;
        ++round;
        empty_parity ^= 1u;
      }
    }
    drain_issued_stages<STAGES>(full_bar, issued, lane, p.err);
    return;
  }

  // ------------------------------ consumers -------------------------------
  if (REGSPLIT) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
  // q and the rows' last pages may be the previous grid's output, and this
  // grid's outputs may be inputs it still reads: nothing before the wait.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int set = warp / kMaxKvHeads;
  const int g = warp % kMaxKvHeads;
  const TileLane tl(lane);
  // This warp's K and V tiles within a stage: head g of the 8 K, then 8 V tiles.
  const uint32_t k_off = g * kTileBytes, v_off = (kMaxKvHeads + g) * kTileBytes;
  constexpr int kOutRow = kMaxKvHeads * kGroup * kHeadDim;  // 2048

  // Rows of length 0 attend to nothing: their output is zero.
  if (set == 0) {
    for (int s = blockIdx.x; s < p.batch; s += gridDim.x) {
      if (__ldg(p.cu + s) == __ldg(p.cu + s + 1)) {
        uint4 z = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(p.out + (size_t)s * kOutRow + g * kGroup * kHeadDim + lane * 8) = z;
      }
    }
  }

  int s = s0;
  int first = start.y, end = start.z;  // page span of sequence s
  int pg = p_begin;
  int kbase = 0;
  // Slot and round of this set's current page, advanced incrementally (page
  // kk of the CTA sits in slot kk % STAGES, round kk / STAGES).  With two sets
  // and an odd number of stages, consecutive rounds of a slot go to different
  // sets, so a set's wait is gated on the slot's tag (stage_tag_wait).
  int c_kk = 0, c_stage = 0, c_round = 0;
  HeadState st;
  bool last_partial = false;  // the range ends inside a sequence that started earlier
  while (pg < p_end) {
    while (pg >= end) {  // next non-empty sequence
      ++s;
      first = end;
      end = __ldg(p.cu + s + 1);
    }
    const int piece_end = min(p_end, end);
    const int n = piece_end - pg;
    const bool complete = (pg == first) && (piece_end == end);
    const int L = __ldg(p.seq_lens + s);

    // Q_g^T operand fragments: column n = tr holds query head 4g + tr (tr < 4).
    uint32_t qb[4][2];
    load_q_frags(p.q + (size_t)s * kOutRow + g * kGroup * kHeadDim, tl, qb);
    st.reset();

    for (int i = set; i < n; i += SETS) {
      for (const int kk = kbase + i; c_kk < kk; ++c_kk) {
        if (++c_stage == STAGES) {
          c_stage = 0;
          ++c_round;
        }
      }
      const int stage = c_stage;
      bool ready = false;
      int tag = 0;
      if (!*abort_flag) {
        tag = SETS > 1 ? stage_tag_wait(stage_tag + stage, c_round, abort_flag) : 1;
        ready = tag != 0 &&
                mbar_wait_bounded(smem_addr(&full_bar[stage]), (uint32_t)(c_round & 1));
      }
      ready = __all_sync(0xffffffffu, ready);
      if (!ready && lane == 0 && !*abort_flag) {
        *abort_flag = 1;
        record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
      }
      // Pull this head's K and V fragments of the page into registers, then
      // release the stage at once: the producer refills it while the math runs,
      // so almost every stage stays in flight (a fetch takes ~4 us at full load).
      if (SETS == 1 && ready) tag = stage_tag[stage];  // read after the copies landed
      const bool have = ready && (tag & 1);
      bool zeroed = false;
      int valid = kPage;
      uint32_t kf[4][4], vf[4][4];
      if (have) {
        const int j = pg - first + i;
        valid = min(kPage, L - j * kPage);
        if (valid < kPage) {
          zero_stale_v_rows(smem + stage * kStageBytes + v_off, valid, lane);
          zeroed = true;
          __syncwarp();
        }
        const uint32_t sb = smem_base + stage * kStageBytes;
        load_tile_frags(sb + k_off, sb + v_off, tl, kf, vf);
      }
      if (zeroed) fence_proxy_async_smem();
      __syncwarp();
      // A stage is released only after its copies landed (a consumer that gave
      // up keeps it, so the producer cannot reuse a slot with a copy in flight).
      if (ready && lane == 0) mbar_arrive(smem_addr(&empty_bar[stage]));
      if (have) attend_tile<LAZY>(st, kf, vf, qb, valid, tl, p.scale_log2);
    }

    if (SETS > 1) {
      // Set 1 hands its (m, l, O) state to set 0 through a 2 x 32-float slot
      // per KV head, two values per lane per round (m, l, then the 16 output
      // fragments in pairs whose columns use the two rescale weights).
      float* mg = merge + g * kMergeFields * 32;
      float wa0 = 1.f, wa1 = 1.f, wb0 = 0.f, wb1 = 0.f;
      auto exchange = [&](float x0, float x1, float& y0, float& y1) {
        if (set == 1) {
          mg[lane] = x0;
          mg[32 + lane] = x1;
        }
        named_barrier_sync(1 + g, 64);
        if (set == 0) {
          y0 = mg[lane];
          y1 = mg[32 + lane];
        }
        named_barrier_sync(1 + g, 64);
      };
      float mb0 = 0.f, mb1 = 0.f;
      exchange(st.m0, st.m1, mb0, mb1);
      if (set == 0) {
        const float M0 = fmaxf(st.m0, mb0), M1 = fmaxf(st.m1, mb1);
        wa0 = st.m0 == -INFINITY ? 0.f : exp2f(st.m0 - M0);
        wa1 = st.m1 == -INFINITY ? 0.f : exp2f(st.m1 - M1);
        wb0 = mb0 == -INFINITY ? 0.f : exp2f(mb0 - M0);
        wb1 = mb1 == -INFINITY ? 0.f : exp2f(mb1 - M1);
        st.m0 = M0;
        st.m1 = M1;
      }
      float lb0 = 0.f, lb1 = 0.f;
      exchange(st.l0, st.l1, lb0, lb1);
      st.l0 = st.l0 * wa0 + lb0 * wb0;
      st.l1 = st.l1 * wa1 + lb1 * wb1;
#pragma unroll
      for (int d = 0; d < 4; ++d) {
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          float b0 = 0.f, b1 = 0.f;
          exchange(st.acc[d][e], st.acc[d][e + 1], b0, b1);
          st.acc[d][e] = st.acc[d][e] * wa0 + b0 * wb0;          // columns 2hc
          st.acc[d][e + 1] = st.acc[d][e + 1] * wa1 + b1 * wb1;  // columns 2hc + 1
        }
      }
    }

    if (piece_end == p_end && !complete) {
      last_partial = true;  // published and merged below
      break;
    }
    if (set == 0) {
      reduce_l(st);
      const OutGroup out_group = local_out(p.out + (size_t)s * kOutRow + g * kGroup * kHeadDim);
      if (complete)
        write_output(st, out_group, tl);
      else
        // combine batch 2: the largest that fits this consumer's registers
        finish_partial<2>(st, p.partials, p.counters, kMaxKvHeads, g, s,
                       partial_slot((int)c, first, T, C), first, end, T, C, out_group, tl, lane);
    }
    kbase += n;
    pg = piece_end;
  }
  if (last_partial) {
    // The range's last piece ends inside a sequence that started earlier; a
    // short step's merges all come from such pieces.  Once every consumer warp
    // has read its last tile the stages are free (every copy issued has landed
    // and been consumed), and head g's eighth of them stages the sequence's
    // partials, so that the merge costs one L2 round trip per 27 pieces.
    named_barrier_sync(kTailBarrier, SETS * kMaxKvHeads * 32);
    if (set == 0) {
      reduce_l(st);
      if (publish_partial(st, p.partials, p.counters, kMaxKvHeads, g, s,
                          partial_slot((int)c, first, T, C), first, end, T, C, tl, lane)) {
        constexpr int kShareBytes = STAGES * kStageBytes / kMaxKvHeads;
        combine_partials_staged(
            p.partials, kMaxKvHeads, g, first, end, T, C,
            local_out(p.out + (size_t)s * kOutRow + g * kGroup * kHeadDim), lane,
            reinterpret_cast<float*>(smem + (size_t)g * kShareBytes), (kShareBytes - 512) / 1024);
      }
    }
  }
}

// Two forms, both persistent with one CTA per SM:
//  * split (default): 2 consumer sets (16 warps, 4 per SMSP) behind a producer
//    warpgroup that hands its registers to them (setmaxnreg), 7 stages of
//    32 KiB plus a 2 KiB set-merge scratch;
//  * plain (fallback when the launch's register pool could not satisfy the
//    split): 1 consumer set and 7 stages.
constexpr int kSplitStages = 7;
constexpr int kPlainStages = 7;

template <int STAGES, int SETS>
constexpr size_t decode_smem_bytes() {
  return (size_t)STAGES * kStageBytes + 2 * STAGES * 8 + (STAGES + 4) * 4 + 16 +
         (SETS > 1 ? (size_t)kMaxKvHeads * kMergeFields * 32 * 4 : 0);
}

cudaError_t launch_decode_plan(const int32_t* lens, int batch, int table_stride, int num_ctas,
                               int kv_heads, int32_t* header, int32_t* cu, int4* cta_start,
                               int32_t* counters, int32_t* err, cudaStream_t stream) {
  decode_plan_kernel<<<1, 1024, 0, stream>>>(lens, batch, table_stride, num_ctas, kv_heads,
                                             header, cu, cta_start, counters, err);
  return cudaGetLastError();
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool resolved = false;
  if (!resolved) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    resolved = true;
  }
  return fn;
}

}  // namespace

// Tensor map over one pool viewed as `rows` rows of kv_heads x 64 BF16
// channels; box = 64 channels (one KV head, 128 B) x 16 rows (one page),
// 128-byte swizzle.  Recently used maps are kept per thread (encoding is host
// work).
bool pool_tensor_map(const void* pool, long long rows, int kv_heads, CUtensorMap* out) {
  struct Entry {
    const void* pool;
    long long rows;
    int kv_heads;
    CUtensorMap map;
  };
  static thread_local Entry cache[4];
  static thread_local int next = 0;
  for (const Entry& e : cache)
    if (e.pool == pool && e.rows == rows && e.kv_heads == kv_heads) {
      *out = e.map;
      return true;
    }
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)(kv_heads * kHeadDim), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(kv_heads * kHeadDim * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)kHeadDim, (cuuint32_t)kPage};
  const cuuint32_t elem_strides[2] = {1, 1};
  CUtensorMap map;
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(pool), dims, strides,
             box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache[next] = {pool, rows, kv_heads, map};
  next = (next + 1) % 4;
  *out = map;
  return true;
}

bool page_tensor_map(const void* pool, long long rows, int kv_heads, CUtensorMap* out) {
  struct Entry {
    const void* pool;
    long long rows;
    int kv_heads;
    CUtensorMap map;
  };
  static thread_local Entry cache[4];
  static thread_local int next = 0;
  for (const Entry& e : cache)
    if (e.pool == pool && e.rows == rows && e.kv_heads == kv_heads) {
      *out = e.map;
      return true;
    }
  PFN_cuTensorMapEncodeTiled_v12000 encode = tensor_map_encoder();
  if (!encode) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows, (cuuint64_t)kv_heads};
  const cuuint64_t strides[2] = {(cuuint64_t)(kv_heads * kHeadDim * 2), (cuuint64_t)(kHeadDim * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)kHeadDim, (cuuint32_t)kPage, (cuuint32_t)kv_heads};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  CUtensorMap map;
  if (encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(pool), dims, strides,
             box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  cache[next] = {pool, rows, kv_heads, map};
  next = (next + 1) % 4;
  *out = map;
  return true;
}

namespace {

enum class DecodeForm { kUnknown, kSplit, kPlain };

// Chooses the form once per device: the split needs the launch's register
// pool (threads x registers per thread) to cover what the warpgroups ask for.
DecodeForm decode_form(int dev) {
  static DecodeForm forms[64] = {};
  if (dev >= 0 && dev < 64 && forms[dev] != DecodeForm::kUnknown) return forms[dev];
  DecodeForm form = DecodeForm::kPlain;
  cudaFuncAttributes fa;
  constexpr int threads = decode_threads<2, true>();
  if (cudaFuncGetAttributes(&fa, paged_decode_kernel<kSplitStages, 2, true, true>) == cudaSuccess &&
      regsplit_fits(fa.numRegs, threads) &&
      cudaFuncSetAttribute(paged_decode_kernel<kSplitStages, 2, true, true>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)decode_smem_bytes<kSplitStages, 2>()) == cudaSuccess)
    form = DecodeForm::kSplit;
  if (form == DecodeForm::kPlain &&
      cudaFuncSetAttribute(paged_decode_kernel<kPlainStages, 1, true, false>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)decode_smem_bytes<kPlainStages, 1>()) != cudaSuccess)
    form = DecodeForm::kUnknown;
  if (dev >= 0 && dev < 64) forms[dev] = form;
  return form;
}

}  // namespace

cudaError_t launch_paged_decode(const DecodeParams& p, long long pool_rows, int num_ctas,
                                cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // Page boxes (3-D maps) for pools of 2 or more heads; a 1-head pool's page
  // of one head is already one 2 KiB box of the 2-D map.
  CUtensorMap k_map, v_map;
  const bool paged = p.kv_heads > 1;
  if (!(paged ? page_tensor_map(p.k_pool, pool_rows, p.kv_heads, &k_map)
              : pool_tensor_map(p.k_pool, pool_rows, p.kv_heads, &k_map)) ||
      !(paged ? page_tensor_map(p.v_pool, pool_rows, p.kv_heads, &v_map)
              : pool_tensor_map(p.v_pool, pool_rows, p.kv_heads, &v_map)))
    return cudaErrorInvalidValue;
  if (p.kv_heads != kMaxKvHeads) return launch_paged_decode_heads(p, k_map, v_map, num_ctas, stream);
  const DecodeForm form = decode_form(dev);
  if (form == DecodeForm::kUnknown) return cudaErrorInvalidDeviceFunction;
  // Programmatic dependent launch: the CTAs start their plan reads, table
  // walk and first copies while the previous kernel finishes (see the
  // producer's wait).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)num_ctas);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (form == DecodeForm::kSplit) {
    cfg.blockDim = dim3(decode_threads<2, true>());
    cfg.dynamicSmemBytes = decode_smem_bytes<kSplitStages, 2>();
    return cudaLaunchKernelEx(&cfg, paged_decode_kernel<kSplitStages, 2, true, true>, p, k_map,
                              v_map);
  }
  cfg.blockDim = dim3(decode_threads<1, false>());
  cfg.dynamicSmemBytes = decode_smem_bytes<kPlainStages, 1>();
  return cudaLaunchKernelEx(&cfg, paged_decode_kernel<kPlainStages, 1, true, false>, p, k_map,
                            v_map);
}

}  // namespace tvp
