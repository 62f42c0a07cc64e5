// Shared device helpers of the paged-KV hot path: BF16 packing, mbarrier,
// bulk-copy (TMA) and warp-level tensor-core primitives for sm_100a.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tvp_paged.h"

namespace tvp {

constexpr int kHeadDim = TVP_HEAD_DIM;     // 64
constexpr int kPage = TVP_PAGE_TOKENS;     // 16
constexpr int kGroup = TVP_GQA_GROUP;      // 4 query heads per KV head
constexpr int kMaxKvHeads = TVP_KV_HEADS;  // 8

// Bound of every pipeline wait, in nanoseconds of %globaltimer.  A wait that
// runs this long records TVP_DEVERR_TIMEOUT and gives up instead of hanging.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Nanoseconds since `start` by %globaltimer, as a signed difference: a timer
// that steps back (it is re-synchronised) reads as no time passed instead of
// wrapping to a huge unsigned interval and ending a wait at once.
__device__ __forceinline__ long long elapsed_ns(unsigned long long start) {
  return (long long)(global_timer_ns() - start);
}

// Bounded wait: true when the phase with `parity` completed, false when the
// wait ran past kWaitLimitNs (the caller records the timeout and stops).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (elapsed_ns(start) > (long long)kWaitLimitNs) return false;
  }
}

// Bounded wait until round `round` of a pipeline stage has been issued.  The
// producer writes the stage's tag, ((round + 1) << 1) | ok, before it issues
// that round's copies.  A consumer that does not take every round of a stage
// (another consumer group takes the round before) calls this before its
// parity wait: a parity wait only tells the current phase from the one before
// it, so on a barrier one round behind (the other group's copy still in
// flight) it would see the round before that as complete and pass at once.
// Once the tag shows `round`, the barrier is at that round or has just
// completed it (the round after needs this consumer's release), so the parity
// wait is exact.  Returns the tag, or 0 when `abort_flag` is set or the wait
// ran past kWaitLimitNs.
__device__ __forceinline__ int stage_tag_wait(const volatile int* tag, int round,
                                              const volatile int* abort_flag) {
  const int want = round + 1;
  int t = *tag;
  if ((t >> 1) >= want) return t;
  const unsigned long long start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i) {
      __nanosleep(32);
      t = *tag;
      if ((t >> 1) >= want) return t;
    }
    if (*abort_flag || elapsed_ns(start) > (long long)kWaitLimitNs) return 0;
  }
}

// ---- bulk copy global -> shared (TMA, no tensor map, this CTA only) -------
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---- tiled TMA load of a 2-D box (tensor map, this CTA only) --------------
// x is the innermost (element) coordinate; x * sizeof(element) must be a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// ---- tiled TMA load of a 3-D box (tensor map, this CTA only) --------------
// x is the innermost coordinate, with the same 16-byte rule as tma_load_2d.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses of the same buffer.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 16-byte global -> shared copy through L2 (cp.async.cg, no registers held
// while it is in flight), and the wait for all of this thread's copies.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- warp-level tensor-core fragments (m16n8k16, BF16 in, FP32 acc) -------
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                            uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                                  uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ void mma_bf16_16816(float& c0, float& c1, float& c2, float& c3,
                                               uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c0), "+f"(c1), "+f"(c2), "+f"(c3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x with the SFU's approximation (ex2.approx.ftz: relative error ~2^-22,
// 2^-inf = +0).  Used by the FAST decode path only.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packs two floats to BF16x2 (round to nearest even); `lo` lands in bits 0..15.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Paired FP32 arithmetic of sm_100 (one instruction for two lanes of work):
// a pair is a 64-bit register holding (lo, hi).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Lane-wise max of two BF16 pairs (a NaN lane yields the other operand).
__device__ __forceinline__ uint32_t bf16x2_max(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

__device__ __forceinline__ float bf16lo_to_f32(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t x) {
  return __uint_as_float(x & 0xffff0000u);
}

__device__ __forceinline__ void record_error(int32_t* err, uint32_t bits) {
  if (err) atomicOr(reinterpret_cast<unsigned int*>(err), bits);
}

}  // namespace tvp
