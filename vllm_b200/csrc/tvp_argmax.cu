// Greedy token selection for a batch of logit rows in one launch.
//
// Replaces the reference's argmaxLogits (src/model/argmax.cu:83-105), which
// the engine calls once per row, two launches and a blocking 4-byte copy each
// (src/model/paged_transformer.cu:119-124, src/engine/scheduler.cu:144-157).
// The selection rule is the reference's (src/model/argmax.cu:16-45):
//   * each logit is rounded to BF16 (round to nearest even) before comparing;
//   * NaNs are skipped;
//   * the largest value wins, ties to the lowest index (-0 equals +0);
//   * a row whose logit 0 rounds to NaN selects token 0.
//
// Grid (kChunks, rows): block (c, r) reduces chunk c of row r to one 64-bit
// key, the order-preserving image of the rounded value in the high word and
// the complement of the index in the low word, so that the larger key is the
// better candidate and a plain max merges them.  The last block of a row to
// finish (a counter per row) merges the row's kChunks keys and writes the
// token; it then zeroes the counter for the next call.
//
// Workspace: the row keys from the start, the per-row counters at the end,
// counter r in the (r + 1)-th int from the end.  A counter's place depends
// only on the workspace's size, never on the row count of a call, so one
// workspace serves calls with any number of rows: every counter a call reads
// was zeroed by the call that last used it (or by the caller, once), and the
// keys, which a call writes before it reads them, never share bytes with a
// counter.  (With the counters right after `rows` rows of keys, a call with
// fewer rows than the one before would read that call's keys as counters.)
#include <cuda_bf16.h>

#include "tvp_common.cuh"

namespace tvp {
namespace {

constexpr int kArgmaxThreads = 256;
constexpr int kChunks = 32;  // blocks per row; 4 rows of 128,256 logits fill 128 of 148 SMs

__device__ __forceinline__ unsigned long long candidate_key(float logit, int index) {
  float v = __bfloat162float(__float2bfloat16_rn(logit));
  if (v != v) return 0ull;  // NaN: never selected
  if (v == 0.f) v = 0.f;    // -0 compares equal to +0
  const uint32_t u = __float_as_uint(v);
  const uint32_t ordered = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)ordered << 32) | (uint32_t)(~(uint32_t)index);
}

__device__ __forceinline__ unsigned long long block_max(unsigned long long key,
                                                        unsigned long long* warp_keys) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) warp_keys[warp] = key;
  __syncthreads();
  key = threadIdx.x < kArgmaxThreads / 32 ? warp_keys[threadIdx.x] : 0ull;
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
  }
  return key;  // valid in thread 0
}

__global__ void __launch_bounds__(kArgmaxThreads)
    greedy_argmax_kernel(const float* __restrict__ logits, int vocab, long long row_stride,
                         unsigned long long* __restrict__ partials, int* __restrict__ counters_end,
                         int32_t* __restrict__ tokens) {
  int* const counter = counters_end - 1 - blockIdx.y;  // this row's counter
  __shared__ unsigned long long warp_keys[kArgmaxThreads / 32];
  __shared__ int is_last;
  const int row = blockIdx.y, chunk = blockIdx.x;
  const float* x = logits + (size_t)row * row_stride;
  const int span = (vocab + kChunks - 1) / kChunks;
  const int begin = chunk * span, end = min(vocab, begin + span);
  unsigned long long best = 0ull;
  for (int i = begin + threadIdx.x; i < end; i += kArgmaxThreads) {
    const unsigned long long k = candidate_key(__ldg(x + i), i);
    best = k > best ? k : best;
  }
  best = block_max(best, warp_keys);
  if (threadIdx.x == 0) {
    partials[(size_t)row * kChunks + chunk] = best;
    __threadfence();
    is_last = atomicAdd(counter, 1) == kChunks - 1;
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long k = 0ull;
  if (threadIdx.x < kChunks) k = __ldcg(partials + (size_t)row * kChunks + threadIdx.x);
  k = block_max(k, warp_keys);
  if (threadIdx.x == 0) {
    const float first = __bfloat162float(__float2bfloat16_rn(x[0]));
    // k != 0 whenever logit 0 is a number (it is a candidate itself)
    tokens[row] = (first != first || k == 0ull) ? 0 : (int32_t)(~(uint32_t)(k & 0xffffffffull));
    *counter = 0;
  }
}

}  // namespace
}  // namespace tvp

using namespace tvp;

extern "C" {

size_t tvp_greedy_argmax_workspace_bytes(int rows) {
  if (rows <= 0) return 0;
  return (size_t)rows * kChunks * sizeof(unsigned long long) + (size_t)rows * sizeof(int);
}

int tvp_greedy_argmax(const float* d_logits, int rows, int vocab, long long row_stride,
                      int32_t* d_tokens, void* d_workspace, size_t workspace_bytes,
                      tvp_stream_t stream) {
  if (!d_logits || !d_tokens || rows <= 0 || rows > 65535 || vocab <= 0 || row_stride < vocab)
    return TVP_ERR_INVALID_ARGUMENT;
  if (!d_workspace || workspace_bytes < tvp_greedy_argmax_workspace_bytes(rows) ||
      (reinterpret_cast<uintptr_t>(d_workspace) & 7u) || (workspace_bytes & 3u))
    return TVP_ERR_WORKSPACE;
  auto* partials = static_cast<unsigned long long*>(d_workspace);
  // counter r at ints_total - 1 - r (see the workspace note above)
  int* counters_end = reinterpret_cast<int*>(static_cast<char*>(d_workspace) + workspace_bytes);
  greedy_argmax_kernel<<<dim3(kChunks, rows), kArgmaxThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      d_logits, vocab, row_stride, partials, counters_end, d_tokens);
  return cudaGetLastError() == cudaSuccess ? TVP_OK : TVP_ERR_RUNTIME;
}

}  // extern "C"
