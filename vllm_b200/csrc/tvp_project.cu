// K5 — the decode step's weight projections over a small batch of rows.
//
// Replaces the projection GEMMs of a decode step: outputProjection, qProjection,
// kProjection, vProjection (src/model/attention.cu:194-323), gateProjection,
// upProjection, downProjection (src/model/mlp.cu:8-102) and lmHeadProjection
// (src/model/lm_head.cu:8-36).
// Each is a cublasGemmEx with W in the reference's layout, [n_out][k] BF16
// (k contiguous, op T), the rows [rows][k] BF16 (op N), FP32 accumulation and
// a BF16 (FP32 for the LM head) result [rows][n_out]:
//     out[t][n] = sum_k W[n][k] x[t][k].
// With 1-8 rows the work is a stream over the weights (121.6 MB per layer of a
// Llama-3.2-1B geometry, 525 MB for its LM head), so the roofline is HBM.
//
// Design:
//  * One CTA per 16 weight rows; its warps split k into equal slices.  Several
//    matrices that share the input rows (Q, K and V; gate and up) run in one
//    launch: the CTAs of matrix i follow those of matrix i - 1.
//  * A lane loads 16 B of weight row r and of row r + 8 and 16 B of input row
//    t = lane / 4 per 32-column block, straight from global memory (weights
//    bypass L1: they are read once), and feeds them to two m16n8k16 BF16
//    tensor-core MMAs.  The dot product does not depend on which k goes to
//    which MMA slot as long as the weight and the input use the same slot, so
//    the lane's 8 contiguous k fill its 4 k-slots of two MMAs: no shared-memory
//    staging and no shuffles.  Input rows t >= rows are zero columns.
//  * The warps' 16 x 8 FP32 partial tiles are summed in shared memory in warp
//    order, so the result does not depend on timing (deterministic), then
//    rounded once to the output type.
//  * Launched as a programmatic dependent launch: the kernel lets the next
//    launch in the stream start at once (griddepcontrol.launch_dependents)
//    and issues its first weight loads before it waits for the previous grid
//    (griddepcontrol.wait), since weights never depend on it; the input rows
//    are read, and every output written, only after the wait.  Two
//    projections in a row (gate+up, then down) so overlap the second's weight
//    stream with the first's tail.
//  * Epilogues fold the reference's next elementwise kernel into the store,
//    with its exact operations and rounding points: the residual connection
//    (residualKernel, src/model/resConnection.cu:6-10: a BF16 add into the
//    hidden rows) and SwiGLU (siluKernel, src/model/SiLU.cu:5-10:
//    bf16(g (1 / (1 + expf(-g))) u) of the BF16-rounded gate and up).  For
//    SwiGLU one CTA streams the same 16 rows of both matrices, so both sums of
//    an element meet in its epilogue.
#include <cuda_bf16.h>

#include "tvp_common.cuh"

namespace tvp {
namespace {

constexpr int kProjRows = 16;      // weight rows per CTA (the MMA's M)
constexpr int kProjMaxTokens = 8;  // input rows (the MMA's N)
constexpr int kProjBlock = 32;     // k columns per lane step (two MMAs)

struct ProjParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w[TVP_PROJ_MAX];
  void* out[TVP_PROJ_MAX];
  int n[TVP_PROJ_MAX];
  int cta_end[TVP_PROJ_MAX];  // prefix sums of n / 16 (one matrix per CTA)
  int count, rows, k, epilogue;
};

// Weights: read-only for the whole life of every launch, so the
// non-coherent path is valid for them.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Input rows: with a programmatic launch they are the previous grid's output,
// written while this grid is already resident, so they must not go through
// the non-coherent (read-only) path.  A plain weak global load after
// griddepcontrol.wait sees them.
__device__ __forceinline__ uint4 ld_coherent_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p)
               : "memory");
  return r;
}

// kMats = 1: the CTA streams 16 rows of one matrix; kMats = 2 (SwiGLU): the
// same 16 rows of matrices 0 and 1.  kUnroll blocks of loads are in flight.
template <int kWarps, int kMats, int kUnroll>
__global__ void __launch_bounds__(kWarps * 32, 16 / kWarps)
    decode_projection_kernel(const ProjParams p) {
  __shared__ float red[kMats][kWarps][4][32];
  // This CTA's matrix, selected with constant indices (a runtime index into
  // the parameter arrays would copy them to local memory).
  const __nv_bfloat16* w0 = p.w[0];
  void* out = p.out[0];
  int n_out = p.n[0], first = 0;
  if (kMats == 1) {
#pragma unroll
    for (int i = 1; i < TVP_PROJ_MAX; ++i)
      if (i < p.count && (int)blockIdx.x >= p.cta_end[i - 1]) {
        w0 = p.w[i];
        out = p.out[i];
        n_out = p.n[i];
        first = p.cta_end[i - 1];
      }
  }
  const int group = blockIdx.x - first;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int slice = p.k / kWarps;  // a multiple of kProjBlock
  const size_t k0 = (size_t)(group * kProjRows + g) * p.k + warp * slice + 8 * q;
  const __nv_bfloat16* wa[kMats];
  wa[0] = w0 + k0;
  if (kMats == 2) wa[kMats - 1] = p.w[1] + k0;
  const bool has_x = g < p.rows;
  const __nv_bfloat16* xr = p.x + (size_t)(has_x ? g : 0) * p.k + warp * slice + 8 * q;

  float c[kMats][4];
#pragma unroll
  for (int m = 0; m < kMats; ++m) c[m][0] = c[m][1] = c[m][2] = c[m][3] = 0.f;
  const int blocks = slice / kProjBlock;
  const size_t row8 = (size_t)8 * p.k;
  // The next launch in the stream may start now; it reads nothing this grid
  // writes before its own wait below.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int b0 = 0; b0 < blocks; b0 += kUnroll) {
    uint4 va[kMats][kUnroll], vb[kMats][kUnroll], vx[kUnroll];
#pragma unroll
    for (int i = 0; i < kUnroll; ++i) {
      if (b0 + i < blocks) {
        const int off = (b0 + i) * kProjBlock;
#pragma unroll
        for (int m = 0; m < kMats; ++m) {
          va[m][i] = ld_stream_v4(wa[m] + off);
          vb[m][i] = ld_stream_v4(wa[m] + row8 + off);
        }
      }
    }
    // The input rows may be the previous grid's output: wait for it (a no-op
    // after the first batch, and when this launch was not programmatic).
    if (b0 == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
#pragma unroll
    for (int i = 0; i < kUnroll; ++i)
      if (b0 + i < blocks)
        vx[i] = has_x ? ld_coherent_v4(xr + (b0 + i) * kProjBlock) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < kUnroll; ++i) {
      if (b0 + i < blocks) {
#pragma unroll
        for (int m = 0; m < kMats; ++m) {
          // k 8q + 0..3 of the block in the first MMA, 8q + 4..7 in the second
          mma_bf16_16816(c[m][0], c[m][1], c[m][2], c[m][3], va[m][i].x, vb[m][i].x, va[m][i].y,
                         vb[m][i].y, vx[i].x, vx[i].y);
          mma_bf16_16816(c[m][0], c[m][1], c[m][2], c[m][3], va[m][i].z, vb[m][i].z, va[m][i].w,
                         vb[m][i].w, vx[i].z, vx[i].w);
        }
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kMats; ++m)
#pragma unroll
    for (int r = 0; r < 4; ++r) red[m][warp][r][lane] = c[m][r];
  __syncthreads();
  if (threadIdx.x < 128) {
    const int r = threadIdx.x >> 5, ln = threadIdx.x & 31;
    float s[kMats];
#pragma unroll
    for (int m = 0; m < kMats; ++m) {
      s[m] = 0.f;
#pragma unroll
      for (int wi = 0; wi < kWarps; ++wi) s[m] += red[m][wi][r][ln];
    }
    // accumulator r of lane ln: weight row (ln / 4) + 8 (r / 2), input row 2 (ln % 4) + r % 2
    const int row = group * kProjRows + (ln >> 2) + ((r & 2) ? 8 : 0);
    const int t = 2 * (ln & 3) + (r & 1);
    if (t < p.rows) {
      const size_t idx = (size_t)t * n_out + row;
      __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(out);
      if (kMats == 2) {
        // siluKernel's expression on the BF16 gate and up
        const float gt = __bfloat162float(__float2bfloat16_rn(s[0]));
        const float up = __bfloat162float(__float2bfloat16_rn(s[kMats - 1]));
        ob[idx] = (__nv_bfloat16)(gt * (1 / (1 + expf(-gt))) * up);
      } else if (p.epilogue == TVP_PROJ_F32) {
        static_cast<float*>(out)[idx] = s[0];
      } else if (p.epilogue == TVP_PROJ_RESIDUAL) {
        ob[idx] = ob[idx] + __float2bfloat16_rn(s[0]);  // residualKernel's BF16 add
      } else {
        ob[idx] = __float2bfloat16_rn(s[0]);
      }
    }
  }
}

}  // namespace
}  // namespace tvp

using namespace tvp;

extern "C" {

int tvp_decode_projections(const tvp_bf16* x, int rows, int k, int count, const tvp_bf16* const* w,
                           const int* n, void* const* out, int epilogue, tvp_stream_t stream) {
  if (!x || !w || !n || !out || rows < 1 || rows > kProjMaxTokens || count < 1 ||
      count > TVP_PROJ_MAX || k < 256 || k % 256 != 0 || epilogue < TVP_PROJ_BF16 ||
      epilogue > TVP_PROJ_SWIGLU || (reinterpret_cast<uintptr_t>(x) & 15u))
    return TVP_ERR_INVALID_ARGUMENT;
  const bool swiglu = epilogue == TVP_PROJ_SWIGLU;
  if (swiglu && (count != 2 || n[0] != n[1])) return TVP_ERR_INVALID_ARGUMENT;
  ProjParams p{};
  p.x = reinterpret_cast<const __nv_bfloat16*>(x);
  p.count = count;
  p.rows = rows;
  p.k = k;
  p.epilogue = epilogue;
  const size_t xb = (size_t)rows * k * sizeof(tvp_bf16);
  long long ctas = 0;
  for (int i = 0; i < count; ++i) {
    const bool stored = !swiglu || i == 0;  // SwiGLU writes out[0] only
    const size_t esize = epilogue == TVP_PROJ_F32 ? 4 : 2;
    if (!w[i] || (stored && !out[i]) || n[i] < kProjRows || n[i] % kProjRows != 0 ||
        (reinterpret_cast<uintptr_t>(w[i]) & 15u) ||
        (stored && (reinterpret_cast<uintptr_t>(out[i]) & (esize - 1))))
      return TVP_ERR_INVALID_ARGUMENT;
    if (stored) {  // an output must not overlap the input rows
      const uintptr_t o = reinterpret_cast<uintptr_t>(out[i]), xa = reinterpret_cast<uintptr_t>(x);
      if (o < xa + xb && xa < o + (size_t)rows * n[i] * esize) return TVP_ERR_INVALID_ARGUMENT;
    }
    if (!swiglu || i == 0) ctas += n[i] / kProjRows;
    if (ctas > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
    p.w[i] = reinterpret_cast<const __nv_bfloat16*>(w[i]);
    p.out[i] = out[i];
    p.n[i] = n[i];
    p.cta_end[i] = (int)ctas;
  }
  // 16 warps (one CTA per SM) when each of 8 warps would stream more than
  // 512 columns, so that long rows keep enough loads in flight per SM.
  const bool wide = k > 4096 && k % 512 == 0;
  void (*kernel)(const ProjParams) =
      swiglu ? (wide ? decode_projection_kernel<16, 2, 4> : decode_projection_kernel<8, 2, 4>)
             : (wide ? decode_projection_kernel<16, 1, 8> : decode_projection_kernel<8, 1, 8>);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(wide ? 16 * 32 : 8 * 32);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? TVP_OK : TVP_ERR_RUNTIME;
}

}  // extern "C"
