// K2h — fused GQA paged decode attention over a pool that holds only KVH of
// the model's KV heads (KVH = 1, 2 or 4): the kernel of a KV-head-sharded
// deployment, where GPU r keeps heads [r KVH, (r + 1) KVH) of every page in a
// pool of rows KVH x 64 channels wide, computes query heads 4 r KVH ..
// 4 (r + 1) KVH - 1 and the ranks then all-gather their slices.  The
// logical -> physical block tables are the reference's (src/model/paged_kvcache.cu:72-117);
// the attention is the same as the reference's decode block
// (src/model/paged_transformer.cu:85-94) restricted to these heads.
//
// Work split: as in K2 (tvp_decode.cu), the T pages of the step are cut into
// C = min(gridDim.x, T) contiguous ranges, one per CTA, with split-K partials
// and a last-arriver combine per (sequence, KV head).
//
// Inside a CTA the stage is the same 32 KiB as K2's (8 K tiles, then 8 V
// tiles), but it holds PS = 8 / KVH consecutive pages of the range with all
// KVH heads each: tile t = page t / KVH of the stage, head t % KVH.  Stages
// alternate between the two sets of 8 consumer warps, so every KV head has
// W = 16 / KVH consumer warps ("ways"); way u = set * PS + offset takes the
// pages i of the range with i % (2 PS) == u.  At the end of each sequence
// piece the W ways of a head merge their online-softmax states through shared
// memory in a log2(W)-level tree, and way 0 writes the output or the partial.
// One stage fewer than K2 leaves room for that merge scratch.
#include <cudaTypedefs.h>

#include "tvp_tile.cuh"

namespace tvp {

constexpr int kHeadsStages = 6;
constexpr int kDoneBarrier = 15;  // named barrier of the 16 consumer warps at a gather's end
constexpr int kTailBarrier = 14;  // the 16 consumer warps, before the stages become merge scratch
constexpr int kStateFloats = 20;  // m0, m1, l0, l1, acc[16] per lane
constexpr int kMergeSlots = 8;    // senders of the widest merge level (W / 2 x KVH)

constexpr size_t heads_smem_bytes() {
  return (size_t)kHeadsStages * kStageBytes + 2 * kHeadsStages * 8 + (kHeadsStages + 4) * 4 +
         16 + (size_t)kMergeSlots * kStateFloats * 32 * 4;
}

// Online-softmax state of two ways over disjoint pages, merged into `a`; the
// other way's state is read field by field from its slot (field f at f * 32).
__device__ __forceinline__ void merge_state(HeadState& a, const float* b) {
  const float mb0 = b[0 * 32], mb1 = b[1 * 32];
  const float M0 = fmaxf(a.m0, mb0), M1 = fmaxf(a.m1, mb1);
  const float wa0 = a.m0 == -INFINITY ? 0.f : exp2f(a.m0 - M0);
  const float wa1 = a.m1 == -INFINITY ? 0.f : exp2f(a.m1 - M1);
  const float wb0 = mb0 == -INFINITY ? 0.f : exp2f(mb0 - M0);
  const float wb1 = mb1 == -INFINITY ? 0.f : exp2f(mb1 - M1);
  a.m0 = M0;
  a.m1 = M1;
  a.l0 = a.l0 * wa0 + b[2 * 32] * wb0;
  a.l1 = a.l1 * wa1 + b[3 * 32] * wb1;
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    a.acc[d][0] = a.acc[d][0] * wa0 + b[(4 + 4 * d + 0) * 32] * wb0;  // columns 2hc
    a.acc[d][1] = a.acc[d][1] * wa1 + b[(4 + 4 * d + 1) * 32] * wb1;  // columns 2hc + 1
    a.acc[d][2] = a.acc[d][2] * wa0 + b[(4 + 4 * d + 2) * 32] * wb0;
    a.acc[d][3] = a.acc[d][3] * wa1 + b[(4 + 4 * d + 3) * 32] * wb1;
  }
}

// Tree merge of the W ways of KV head h into way 0.  Slots are [field][lane]
// so that a warp's stores and loads are conflict-free.  Barrier ids: 1 + h for
// the levels (participants: the ways still in the tree), 1 + KVH + h for the
// entry, which all W ways pass, so that no way of the next piece writes a slot
// that way 0 is still reading.
template <int KVH>
__device__ __forceinline__ void merge_ways(HeadState& st, float* scratch, int way, int h,
                                           int lane) {
  constexpr int W = 16 / KVH;
  named_barrier_sync(1 + KVH + h, W * 32);
#pragma unroll
  for (int d = W / 2; d >= 1; d >>= 1) {
    if (way >= d) {  // sender at this level (ways >= 2d have left)
      float* slot = scratch + (size_t)((way - d) * KVH + h) * kStateFloats * 32 + lane;
      slot[0 * 32] = st.m0;
      slot[1 * 32] = st.m1;
      slot[2 * 32] = st.l0;
      slot[3 * 32] = st.l1;
#pragma unroll
      for (int d4 = 0; d4 < 4; ++d4)
#pragma unroll
        for (int e = 0; e < 4; ++e) slot[(4 + 4 * d4 + e) * 32] = st.acc[d4][e];
      named_barrier_sync(1 + h, 2 * d * 32);
      return;
    }
    named_barrier_sync(1 + h, 2 * d * 32);
    merge_state(st, scratch + (size_t)(way * KVH + h) * kStateFloats * 32 + lane);
    // The next level's senders (ways [d/2, d)) overwrite slots that ways
    // [0, d/2) have just read.
    if (d > 1) named_barrier_sync(1 + h, d * 32);
  }
}

// GATHER: the KV-head-shard all-gather fused into the kernel.  Each output
// group is stored straight into every rank's gathered rows [B][2048] at this
// rank's heads (plain stores to peer memory over NVLink, issued as soon as the
// group is final); each CTA counts itself done, the last CTA of the launch
// adds 1 to every rank's flag and waits until its own flag reached
// launches x world, i.e. until every rank's rows of this launch have landed.
template <int KVH, bool REGSPLIT, bool GATHER>
__global__ void __launch_bounds__(decode_threads<2, REGSPLIT>(), 1)
    paged_decode_heads_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap k_map,
                              const __grid_constant__ CUtensorMap v_map) {
  constexpr int PS = kStageTiles / KVH;  // pages per stage
  constexpr int PERIOD = 2 * PS;         // pages between two pages of one way
  constexpr int STAGES = kHeadsStages;
  // 1 KiB alignment of the stage tiles (128-byte swizzle); checked, as in K2.
  extern __shared__ __align__(1024) unsigned char smem[];
  // Plan header, page count and this CTA's start record in one round trip (K2).
  const int4 hdr = __ldg(reinterpret_cast<const int4*>(p.header));
  const int total_pages = __ldg(p.cu + p.batch);
  const int4 start = __ldg(p.cta_start + blockIdx.x);
  if (smem_addr(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_SMEM_ALIGN);
    return;
  }
  if (!(hdr.x == kPlanMagic && hdr.y == p.batch && hdr.z == (int)gridDim.x && hdr.w == KVH)) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_PLAN);
    return;
  }
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  int* stage_mask = reinterpret_cast<int*>(empty_bar + STAGES);  // bit o: page o of the stage loaded
  volatile int* abort_flag = stage_mask + STAGES;
  float* scratch = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem + STAGES * kStageBytes + 2 * STAGES * 8 +
                                   (STAGES + 4) * 4) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kStageTiles);  // one arrival per (page, head) tile
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();

  const long long T = total_pages;
  const long long C = T < (long long)gridDim.x ? T : (long long)gridDim.x;
  const long long c = blockIdx.x;
  const int p_begin = c < C ? (int)(c * T / C) : 0;
  const int p_end = c < C ? (int)((c + 1) * T / C) : 0;
  const int n = p_end - p_begin;
  const uint32_t smem_base = smem_addr(smem);

  const int s0 = n > 0 ? start.x : 0;  // sequence of the range's first page

  if (warp >= 2 * kStageTiles) {
    // ------------------------------ producer ------------------------------
    if (REGSPLIT) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
      if (warp != 2 * kStageTiles) return;
    }
    if (lane == 0) {
      prefetch_tensor_map(&k_map);
      prefetch_tensor_map(&v_map);
    }
    // Lane o < PS walks the range's pages o, o + PS, o + 2 PS, ... (sequence
    // and its page span in registers, next page id loaded one stage ahead).
    int s = s0, seq_first = 0, seq_end = 0, phys = 0;
    int i = lane;
    auto walk = [&]() {
      const int pg = p_begin + i;
      while (pg >= seq_end) {
        ++s;
        seq_first = seq_end;
        seq_end = __ldg(p.cu + s + 1);
      }
      phys = __ldg(p.tables + (size_t)s * p.table_stride + (pg - seq_first));
    };
    if (lane < PS && i < n) {
      seq_first = start.y;
      seq_end = start.z;
      walk();
    }
    const int n_stages = (n + PS - 1) / PS;
    int stage = 0, issued = 0;
    uint32_t empty_parity = 1;
    for (int kk = 0; kk < n_stages; ++kk) {
      const int cur_phys = phys;
      const bool mine = lane < PS && i < n;
      i += PS;
      if (lane < PS && i < n) walk();
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
      const bool ok = mine && cur_phys >= 0 && cur_phys < p.num_pages;
      if (mine && !ok) record_error(p.err, TVP_DEVERR_BAD_PAGE);
      const uint32_t mask = __ballot_sync(0xffffffffu, ok);
      const uint32_t full = smem_addr(&full_bar[stage]);
      if (lane == 0) {
        stage_mask[stage] = (int)mask;
        mbar_arrive_expect_tx(full, (uint32_t)(__popc(mask) * KVH * 2 * kTileBytes));
      }
      __syncwarp();
      // lanes 0..PS-1: the K box of page o = lane, lanes PS..2PS-1: its V box;
      // a box holds the page's KVH heads and lands as KVH tiles t = o KVH + h
      // (a 3-D page box for KVH > 1, the one-head box of the 2-D map for 1).
      const int o = lane % PS;
      const int tile_phys = __shfl_sync(0xffffffffu, cur_phys, o);
      if (lane < 2 * PS && ((mask >> o) & 1u)) {
        const bool is_v = lane >= PS;
        const uint32_t dst = smem_base + stage * kStageBytes +
                             (is_v ? kStageTiles * kTileBytes : 0) + o * KVH * kTileBytes;
        const int y = (int)(p.layer_row_base + (long long)tile_phys * kPage);
        if (KVH > 1)
          tma_load_3d(dst, is_v ? &v_map : &k_map, 0, y, 0, full);
        else
          tma_load_2d(dst, is_v ? &v_map : &k_map, 0, y, full);
      }
      issued = kk + 1;
      if (++stage == STAGES) {
        stage = 0;
        empty_parity ^= 1u;
      }
    }
    drain_issued_stages<STAGES>(full_bar, issued, lane, p.err);
    return;
  }

  // ------------------------------ consumers -------------------------------
  if (REGSPLIT) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
  const int set = warp / kStageTiles;
  const int t = warp % kStageTiles;  // tile of the stage this warp reads
  const int o = t / KVH, h = t % KVH;
  const int way = set * PS + o;
  const TileLane tl(lane);
  const uint32_t k_off = t * kTileBytes, v_off = (kStageTiles + t) * kTileBytes;
  constexpr int kOutRow = KVH * kGroup * kHeadDim;                  // this rank's rows
  constexpr int kGatherRow = kMaxKvHeads * kGroup * kHeadDim;       // gathered rows (2048)
  // Destination of sequence s's output for KV head h.
  auto out_of = [&](int s) -> OutGroup {
    if (GATHER)
      return OutGroup{nullptr, p.peer_rows,
                      (size_t)s * kGatherRow + (size_t)(p.rank * KVH + h) * kGroup * kHeadDim,
                      p.world};
    return local_out(p.out + (size_t)s * kOutRow + h * kGroup * kHeadDim);
  };

  if (way == 0) {
    for (int s = blockIdx.x; s < p.batch; s += gridDim.x)
      if (__ldg(p.cu + s) == __ldg(p.cu + s + 1)) out_of(s).store16(lane * 8, make_uint4(0, 0, 0, 0));
  }

  int s = s0;
  int first = start.y, end = start.z;  // page span of sequence s
  int pg = p_begin;
  int kbase = 0;  // range-local index of the piece's first page
  int c_kk = 0, c_stage = 0;
  uint32_t c_parity = 0;
  HeadState st;
  bool last_partial = false;  // the range ends inside a sequence that started earlier
  while (pg < p_end) {
    while (pg >= end) {  // next non-empty sequence
      ++s;
      first = end;
      end = __ldg(p.cu + s + 1);
    }
    const int piece_end = min(p_end, end);
    const int np = piece_end - pg;
    const bool complete = (pg == first) && (piece_end == end);
    const int L = __ldg(p.seq_lens + s);

    uint32_t qb[4][2];
    load_q_frags(p.q + (size_t)s * kOutRow + h * kGroup * kHeadDim, tl, qb);
    st.reset();

    for (int i = kbase + ((way - kbase) % PERIOD + PERIOD) % PERIOD; i < kbase + np; i += PERIOD) {
      for (const int kk = i / PS; c_kk < kk; ++c_kk) {
        if (++c_stage == STAGES) {
          c_stage = 0;
          c_parity ^= 1u;
        }
      }
      const int stage = c_stage;
      bool ready = false;
      if (!*abort_flag) ready = mbar_wait_bounded(smem_addr(&full_bar[stage]), c_parity);
      ready = __all_sync(0xffffffffu, ready);
      if (!ready && lane == 0 && !*abort_flag) {
        *abort_flag = 1;
        record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_FULL);
      }
      const bool have = ready && ((stage_mask[stage] >> o) & 1);
      bool zeroed = false;
      int valid = kPage;
      uint32_t kf[4][4], vf[4][4];
      if (have) {
        const int j = pg - first + (i - kbase);  // page of the sequence
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
      if (have) attend_tile<true>(st, kf, vf, qb, valid, tl, p.scale_log2);
    }

    merge_ways<KVH>(st, scratch, way, h, lane);
    if (piece_end == p_end && !complete) {
      last_partial = true;  // published and merged below
      break;
    }
    if (way == 0) {
      reduce_l(st);
      const OutGroup out_group = out_of(s);
      if (complete)
        write_output(st, out_group, tl);
      else
        // combine batch 1 (the registers of the staged merge below; the
        // fold's arithmetic does not depend on the batch)
        finish_partial<1>(st, p.partials, p.counters, KVH, h, s,
                                         partial_slot((int)c, first, T, C), first, end, T, C,
                                         out_group, tl, lane);
    }
    kbase += np;
    pg = piece_end;
  }
  if (last_partial) {
    // The range's last piece ends inside a sequence that started earlier.
    // Once every consumer warp has read its last tile, the stage buffers are
    // free (every copy the producer issued has landed and been consumed), and
    // head h's share of them holds the sequence's partials for the merge.
    named_barrier_sync(kTailBarrier, 2 * kStageTiles * 32);
    if (way == 0) {
      reduce_l(st);
      if (publish_partial(st, p.partials, p.counters, KVH, h, s, partial_slot((int)c, first, T, C),
                          first, end, T, C, tl, lane)) {
        constexpr int kShareBytes = STAGES * kStageBytes / KVH;
        combine_partials_staged(p.partials, KVH, h, first, end, T, C, out_of(s), lane,
                                reinterpret_cast<float*>(smem + (size_t)h * kShareBytes),
                                (kShareBytes - 512) / 1024);
      }
    }
  }

  if (GATHER) {
    // The CTA's row stores are ordered before thread 0's fence by the barrier;
    // the fence releases them (system scope) before the CTA counts itself
    // done.  The last CTA acquires every CTA's release, signals every rank
    // (its own included) and waits, bounded, until all ranks have signalled:
    // when the kernel ends, every rank's rows of this launch are here.
    named_barrier_sync(kDoneBarrier, 2 * kStageTiles * 32);
    if (threadIdx.x == 0) {
      __threadfence_system();
      const int done = atomicAdd(p.done_counter, 1);
      if (done == (int)gridDim.x - 1) {
        atomicExch(p.done_counter, 0);  // ready for the next launch
        __threadfence_system();
        const unsigned long long* flags = reinterpret_cast<const unsigned long long*>(p.peer_flags);
        for (int r = 0; r < p.world; ++r) atomicAdd_system(reinterpret_cast<int*>(__ldg(flags + r)), 1);
        const int32_t* mine = reinterpret_cast<const int32_t*>(__ldg(flags + p.rank));
        const unsigned long long start = global_timer_ns();
        while (true) {
          int32_t v;
          asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
          if ((int32_t)((uint32_t)v - (uint32_t)p.flag_target) >= 0) break;
          if (elapsed_ns(start) > (long long)kWaitLimitNs) {
            record_error(p.err, TVP_DEVERR_TIMEOUT | TVP_DEVERR_WAIT_PEERS);
            break;
          }
          __nanosleep(128);
        }
      }
    }
  }
}

namespace {

enum class HeadsForm { kUnknown, kSplit, kPlain };

template <int KVH, bool GATHER>
HeadsForm heads_form(int dev) {
  static HeadsForm forms[64] = {};
  if (dev >= 0 && dev < 64 && forms[dev] != HeadsForm::kUnknown) return forms[dev];
  HeadsForm form = HeadsForm::kPlain;
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, paged_decode_heads_kernel<KVH, true, GATHER>) == cudaSuccess &&
      regsplit_fits(fa.numRegs, decode_threads<2, true>()) &&
      cudaFuncSetAttribute(paged_decode_heads_kernel<KVH, true, GATHER>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)heads_smem_bytes()) == cudaSuccess)
    form = HeadsForm::kSplit;
  if (form == HeadsForm::kPlain &&
      cudaFuncSetAttribute(paged_decode_heads_kernel<KVH, false, GATHER>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)heads_smem_bytes()) != cudaSuccess)
    form = HeadsForm::kUnknown;
  if (dev >= 0 && dev < 64) forms[dev] = form;
  return form;
}

template <int KVH, bool GATHER>
cudaError_t launch_heads(const DecodeParams& p, const CUtensorMap& k_map, const CUtensorMap& v_map,
                         int num_ctas, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const HeadsForm form = heads_form<KVH, GATHER>(dev);
  if (form == HeadsForm::kUnknown) return cudaErrorInvalidDeviceFunction;
  if (form == HeadsForm::kSplit)
    paged_decode_heads_kernel<KVH, true, GATHER>
        <<<num_ctas, decode_threads<2, true>(), heads_smem_bytes(), stream>>>(p, k_map, v_map);
  else
    paged_decode_heads_kernel<KVH, false, GATHER>
        <<<num_ctas, decode_threads<2, false>(), heads_smem_bytes(), stream>>>(p, k_map, v_map);
  return cudaGetLastError();
}

template <bool GATHER>
cudaError_t launch_heads_any(const DecodeParams& p, const CUtensorMap& k_map,
                             const CUtensorMap& v_map, int num_ctas, cudaStream_t stream) {
  switch (p.kv_heads) {
    case 1: return launch_heads<1, GATHER>(p, k_map, v_map, num_ctas, stream);
    case 2: return launch_heads<2, GATHER>(p, k_map, v_map, num_ctas, stream);
    case 4: return launch_heads<4, GATHER>(p, k_map, v_map, num_ctas, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_paged_decode_heads(const DecodeParams& p, const CUtensorMap& k_map,
                                      const CUtensorMap& v_map, int num_ctas,
                                      cudaStream_t stream) {
  if (p.peer_rows != nullptr) return launch_heads_any<true>(p, k_map, v_map, num_ctas, stream);
  return launch_heads_any<false>(p, k_map, v_map, num_ctas, stream);
}

}  // namespace tvp
