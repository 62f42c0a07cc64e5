// K2c — decode attention with the reference's rounding points (COMPAT mode).
//
// The reference rounds three times on the decode path: the cuBLAS score GEMV
// writes BF16 scores (alpha = scale applied to the FP32 dot product,
// src/model/attention.cu:53-93), softmaxKernel turns them into BF16
// probabilities with an exact max, expf and a pairwise-tree sum over the row
// (src/model/softmax.cu:6-45), and the P.V GEMV accumulates in FP32 and writes
// BF16 (src/model/attention.cu:95-142).  This kernel keeps every one of those
// rounding points and the tree order of the sum; only the FP32 order inside the
// two dot products is its own (sequential FMA), which cuBLAS does not specify.
// One CTA per (sequence, KV head) of a pool of 1, 2, 4 or 8 KV heads; pages are
// read in place; rows of any length up to 1,048,576 tokens.  Used where the
// reference's rounding matters more than bandwidth.
#include "tvp_params.cuh"

namespace tvp {

// Rows are processed in chunks of kCompatChunk tokens held in shared memory.
// The reference's pairwise tree (for i = 1, 2, 4, ...: e[t] += e[t + i] when
// t % 2i == 0 and t + i < L) splits exactly at a power-of-two chunk size c:
// its levels i < c are the same tree inside each aligned chunk of c tokens
// (t + i < L is the same condition in chunk-local indices), and its levels
// i >= c are the same tree again over the chunk sums, with stride i / c and
// the condition m + i / c < ceil(L / c).  Summing chunk by chunk therefore
// performs the reference's additions in the reference's order, for any L.
// A row longer than one chunk recomputes its BF16 scores in each of the three
// passes (max, sum, P.V) instead of keeping them, from the same inputs by the
// same operations, so the values are the same every time.
constexpr int kCompatChunk = 4096;
constexpr int kCompatMaxChunks = 256;  // rows of up to 1,048,576 tokens
constexpr int kCompatThreads = 256;


__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// sc[h][t - base] = bf16(scale * (q_h . k_t)) for t in [base, base + n), FP32
// accumulation in channel order.
__device__ __forceinline__ void compat_scores(const CompatParams& p, int s, int g, const float* qs,
                                              int base, int n, float* sc, int tid) {
  const int kv_dim = p.kv_heads * kHeadDim;
  for (int tl = tid; tl < n; tl += kCompatThreads) {
    const int t = base + tl;
    const int phys = p.tables[(size_t)s * p.table_stride + t / kPage];
    if (phys < 0 || phys >= p.num_pages) {
      record_error(p.err, TVP_DEVERR_BAD_PAGE);
      for (int h = 0; h < kGroup; ++h) sc[h * kCompatChunk + tl] = -INFINITY;
      continue;
    }
    const uint4* krow = reinterpret_cast<const uint4*>(
        p.k_pool + (size_t)(p.layer_row_base + (long long)phys * kPage + t % kPage) * kv_dim +
        g * kHeadDim);
    float k[kHeadDim];
#pragma unroll
    for (int i = 0; i < kHeadDim / 8; ++i) {
      const uint4 u = __ldg(krow + i);
      k[8 * i + 0] = bf16lo_to_f32(u.x); k[8 * i + 1] = bf16hi_to_f32(u.x);
      k[8 * i + 2] = bf16lo_to_f32(u.y); k[8 * i + 3] = bf16hi_to_f32(u.y);
      k[8 * i + 4] = bf16lo_to_f32(u.z); k[8 * i + 5] = bf16hi_to_f32(u.z);
      k[8 * i + 6] = bf16lo_to_f32(u.w); k[8 * i + 7] = bf16hi_to_f32(u.w);
    }
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < kHeadDim; ++d) acc = fmaf(qs[h * kHeadDim + d], k[d], acc);
      sc[h * kCompatChunk + tl] = round_bf16(p.scale * acc);
    }
  }
}

__global__ void __launch_bounds__(kCompatThreads) compat_decode_kernel(const CompatParams p) {
  extern __shared__ float sm[];
  float* qs = sm;                            // [4][64]
  float* sc = qs + kGroup * kHeadDim;        // [4][kCompatChunk] scores, then probabilities
  float* tree = sc + kGroup * kCompatChunk;  // [4][kCompatChunk] pairwise-sum buffer
  __shared__ float red[kGroup][kCompatThreads / 32];
  __shared__ float row_max[kGroup];
  __shared__ float csum[kGroup][kCompatMaxChunks];  // chunk sums, then their tree

  const int s = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
  const int kv_dim = p.kv_heads * kHeadDim;
  const int out_row = p.kv_heads * kGroup * kHeadDim;
  const int L = p.seq_lens[s];
  __nv_bfloat16* out = p.out + (size_t)s * out_row + g * kGroup * kHeadDim;
  if (L <= 0 || L > kCompatChunk * kCompatMaxChunks || L > p.table_stride * kPage) {
    if (L != 0 && tid == 0) record_error(p.err, TVP_DEVERR_BAD_LENGTH);
    out[tid] = __float2bfloat16_rn(0.f);
    return;
  }
  qs[tid] = __bfloat162float(p.q[(size_t)s * out_row + g * kGroup * kHeadDim + tid]);
  __syncthreads();
  const int chunks = (L + kCompatChunk - 1) / kCompatChunk;
  const bool one_chunk = chunks == 1;  // scores computed once and kept

  // Pass 1: exact row maximum of the BF16 scores (order-free).
  float mx[kGroup];
#pragma unroll
  for (int h = 0; h < kGroup; ++h) mx[h] = -INFINITY;
  for (int c = 0; c < chunks; ++c) {
    const int base = c * kCompatChunk, n = min(kCompatChunk, L - base);
    if (c > 0) __syncthreads();  // every thread is done reading the previous chunk
    compat_scores(p, s, g, qs, base, n, sc, tid);
    __syncthreads();
    for (int t = tid; t < n; t += kCompatThreads)
#pragma unroll
      for (int h = 0; h < kGroup; ++h) mx[h] = fmaxf(mx[h], sc[h * kCompatChunk + t]);
  }
#pragma unroll
  for (int h = 0; h < kGroup; ++h) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], o));
    if ((tid & 31) == 0) red[h][tid >> 5] = mx[h];
  }
  __syncthreads();
  if (tid < kGroup) {
    float m = red[tid][0];
    for (int w = 1; w < kCompatThreads / 32; ++w) m = fmaxf(m, red[tid][w]);
    row_max[tid] = m;
  }
  __syncthreads();

  // Pass 2: e_t = expf(s_t - max) summed by the reference's pairwise tree,
  // inside each chunk, then over the chunk sums (see above).
  for (int c = 0; c < chunks; ++c) {
    const int base = c * kCompatChunk, n = min(kCompatChunk, L - base);
    if (!one_chunk) {
      __syncthreads();
      compat_scores(p, s, g, qs, base, n, sc, tid);
      __syncthreads();
    }
    for (int t = tid; t < n; t += kCompatThreads)
#pragma unroll
      for (int h = 0; h < kGroup; ++h)
        tree[h * kCompatChunk + t] = expf(sc[h * kCompatChunk + t] - row_max[h]);
    __syncthreads();
    for (int i = 1; i < n; i *= 2) {
      for (int t = tid * 2 * i; t < n; t += kCompatThreads * 2 * i) {
        if (t + i < n) {
#pragma unroll
          for (int h = 0; h < kGroup; ++h)
            tree[h * kCompatChunk + t] = tree[h * kCompatChunk + t] + tree[h * kCompatChunk + t + i];
        }
      }
      __syncthreads();
    }
    if (tid < kGroup) csum[tid][c] = tree[tid * kCompatChunk];
  }
  if (tid < kGroup)
    for (int j = 1; j < chunks; j *= 2)
      for (int m = 0; m + j < chunks; m += 2 * j) csum[tid][m] = csum[tid][m] + csum[tid][m + j];
  __syncthreads();

  // Pass 3: p = bf16(expf(s - max) / sum); o[h][d] = bf16(sum_t p[h][t] v[t][d])
  // with FP32 accumulation in token order across the chunks.
  const int h = tid / kHeadDim, d = tid % kHeadDim;
  float acc = 0.f;
  for (int c = 0; c < chunks; ++c) {
    const int base = c * kCompatChunk, n = min(kCompatChunk, L - base);
    if (!one_chunk) {
      __syncthreads();  // every thread is done with the previous chunk's probabilities
      compat_scores(p, s, g, qs, base, n, sc, tid);
      __syncthreads();
    }
    for (int t = tid; t < n; t += kCompatThreads)
#pragma unroll
      for (int hh = 0; hh < kGroup; ++hh)
        sc[hh * kCompatChunk + t] =
            round_bf16(expf(sc[hh * kCompatChunk + t] - row_max[hh]) / csum[hh][0]);
    __syncthreads();
    for (int tl = 0; tl < n; ++tl) {
      const int t = base + tl;
      const int phys = __ldg(p.tables + (size_t)s * p.table_stride + t / kPage);
      if (phys < 0 || phys >= p.num_pages) continue;
      const float v = __bfloat162float(
          p.v_pool[(size_t)(p.layer_row_base + (long long)phys * kPage + t % kPage) * kv_dim +
                   g * kHeadDim + d]);
      acc = fmaf(sc[h * kCompatChunk + tl], v, acc);
    }
  }
  out[h * kHeadDim + d] = __float2bfloat16_rn(acc);
}

size_t compat_smem_bytes() {
  return (size_t)(kGroup * kHeadDim + 2 * kGroup * kCompatChunk) * sizeof(float);
}

cudaError_t launch_compat_decode(const CompatParams& p, int batch, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(compat_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)compat_smem_bytes());
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  compat_decode_kernel<<<dim3(batch, p.kv_heads), kCompatThreads, compat_smem_bytes(), stream>>>(p);
  return cudaGetLastError();
}

}  // namespace tvp
