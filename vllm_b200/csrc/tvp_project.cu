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
//  * The RMSNorm after a residual epilogue (O, down) is spread over the grid:
//    each CTA holds both features of 8 of the reference's sum-of-squares
//    leaves, publishes that subtree's sum, and after a bounded grid-wide
//    arrival normalises its own features (the same tree order, so the same
//    bits).  The down launch can also run the next layer's Q/K/V with RoPE and
//    the page append (down_norm_qkv_kernel), loading their weights before the
//    arrival.
#include <cuda_bf16.h>

#include "tvp_common.cuh"
#include "tvp_rope.cuh"

namespace tvp {
namespace {

constexpr int kProjRows = 16;      // weight rows per CTA (the MMA's M)
constexpr int kProjMaxTokens = 8;  // input rows (the MMA's N)
constexpr int kProjBlock = 32;     // k columns per lane step (two MMAs)

constexpr int kHidden = 2048;       // rows of the RMSNorm fused after a residual epilogue
constexpr int kEpiRopeAppend = 16;  // internal epilogue: Q/K/V with RoPE and the page append

struct ProjParams {
  const __nv_bfloat16* x;
  const __nv_bfloat16* w[TVP_PROJ_MAX];
  void* out[TVP_PROJ_MAX];
  int n[TVP_PROJ_MAX];
  int cta_end[TVP_PROJ_MAX];  // prefix sums of n / 16 (one matrix per CTA)
  int count, rows, k, epilogue;
  // Residual epilogue followed by the next RMSNorm (norm_out != nullptr):
  // norm_out = rmsnorm(out[0]) x norm_gain.  With norm_spread, every CTA
  // publishes the sum-of-squares subtree of its rows (norm_part), waits for
  // all CTAs of the grid at the arrival counter and normalises its own
  // outputs; otherwise the last CTA to finish normalises all of them.
  const __nv_bfloat16* norm_gain;
  __nv_bfloat16* norm_out;
  int* counter;
  float* norm_part;   // [8][128]: one subtree sum per (row, CTA)
  int32_t* norm_err;  // TVP_DEVERR_TIMEOUT when a CTA gave up waiting for the others
  int norm_spread;
  // kEpiRopeAppend: matrix 0 = q, 1 = k, 2 = v of one token per row; q is
  // stored rotated into out[0], k rotated and v as is into their page slots.
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  long long layer_row_base;
  int num_pages, table_stride;
  const int32_t* tables;
  const int32_t* pos;
  int32_t* err;
};

// Leaf of the reference's sum of squares, (float)a * (float)a +
// (float)b * (float)b, with the rounding nvcc gives that expression under its
// default FMA contraction: fma(a, a, b * b) (found by comparing outputs with
// the reference kernel's over thousands of rows of every magnitude).
__device__ __forceinline__ float norm_leaf(float a, float b) {
  return __fmaf_rn(a, a, __fmul_rn(b, b));
}

// RMSNorm of `rows` finished rows of 2048 by one CTA of kThreads threads, with
// the reference's arithmetic (rmsNormKernel, src/model/rmsNorm.cu:3-22): the
// sum of squares by its tree (leaf t < 1024 is x[t]^2 + x[t + 1024]^2, then
// for i = 1, 2, ..., 512: leaf[t] += leaf[t + i] where t % 2i == 0), r =
// sqrt(sum / 2048 + 1e-5) evaluated in double as the reference writes it, and
// out = bf16((x / r) g) with IEEE division.  Warp w < rows sums row w: lane l
// forms leaves 32 l .. 32 l + 31 and sums them by the same tree, and the
// lanes' sums meet by the tree's upper levels through shuffles.  Every thread
// then writes its share of all rows' outputs; it issues the loads of that
// share (through L2: other CTAs of the grid wrote the rows) before the sums.
template <int kThreads>
__device__ __forceinline__ void rmsnorm_rows_cta(const __nv_bfloat16* x, const __nv_bfloat16* gain,
                                                 __nv_bfloat16* out, int rows) {
  constexpr int kVecPerRow = kHidden / 8;                          // 256 uint4 per row
  constexpr int kMaxVec = kProjMaxTokens * kVecPerRow / kThreads;  // per thread
  __shared__ float r_row[kProjMaxTokens];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const uint4* gv = reinterpret_cast<const uint4*>(gain);
  uint4 mine[kMaxVec], mine_g[kMaxVec];
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < rows * kVecPerRow) {
      mine[j] = __ldcg(xv + i);
      mine_g[j] = __ldg(gv + i % kVecPerRow);
    }
  }
  if (warp < rows) {
    uint4 a[4], b[4];
    const uint4* xa = xv + warp * kVecPerRow + 4 * lane;
    const uint4* xb = xa + kVecPerRow / 2;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = __ldcg(xa + i);
      b[i] = __ldcg(xb + i);
    }
    float leaf[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t wa[4] = {a[i].x, a[i].y, a[i].z, a[i].w};
      const uint32_t wb[4] = {b[i].x, b[i].y, b[i].z, b[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        leaf[8 * i + 2 * j] = norm_leaf(bf16lo_to_f32(wa[j]), bf16lo_to_f32(wb[j]));
        leaf[8 * i + 2 * j + 1] = norm_leaf(bf16hi_to_f32(wa[j]), bf16hi_to_f32(wb[j]));
      }
    }
#pragma unroll
    for (int st = 1; st < 32; st *= 2)
#pragma unroll
      for (int i = 0; i < 32; i += 2 * st) leaf[i] = __fadd_rn(leaf[i], leaf[i + st]);
    float v = leaf[0];
#pragma unroll
    for (int off = 1; off < 32; off *= 2) {
      const float o = __shfl_down_sync(0xffffffffu, v, off);
      if ((lane & (2 * off - 1)) == 0) v = __fadd_rn(v, o);
    }
    if (lane == 0) r_row[warp] = (float)sqrt((double)v / 2048.0 + 1.0e-5);
  }
  __syncthreads();
  auto norm2 = [](uint32_t xw, uint32_t gw, float r) {
    const float y0 = __fmul_rn(__fdiv_rn(bf16lo_to_f32(xw), r), bf16lo_to_f32(gw));
    const float y1 = __fmul_rn(__fdiv_rn(bf16hi_to_f32(xw), r), bf16hi_to_f32(gw));
    return pack_bf16x2(y0, y1);
  };
  uint4* ov = reinterpret_cast<uint4*>(out);
#pragma unroll
  for (int j = 0; j < kMaxVec; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < rows * kVecPerRow) {
      const float r = r_row[i / kVecPerRow];
      ov[i] = make_uint4(norm2(mine[j].x, mine_g[j].x, r), norm2(mine[j].y, mine_g[j].y, r),
                         norm2(mine[j].z, mine_g[j].z, r), norm2(mine[j].w, mine_g[j].w, r));
    }
  }
}

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

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Epilogue of the Q/K/V projection of one decode token per row, fused with
// RoPE and the page append (K1's work, tvp_append.cu): thread (r, ln) of the
// first 128 holds the FP32 sum of MMA row (ln / 4) + 8 (r / 2) for token
// row t.  For q and k the two MMA rows of a thread pair are the two halves
// (d, d + 32) of a rotate-half pair, exchanged through shared memory; each
// half is rounded to BF16 (the projection's output) and rotated with K1's
// arithmetic, bit for bit.  q goes to out[0]; k and v go into slot pos % 16
// of page tables[t][pos / 16] of the layer's pools.  Threads with
// (r & 2) == 0 and ln < 4 hold MMA row 0 for each of the 8 token rows: they
// report a row's bad position or page once.
// `tid` is the thread's index in the group of threads that runs the epilogue
// (a whole CTA, or half of one), `half` that group's exchange buffer and
// `sync` its barrier.
template <typename Sync>
__device__ __forceinline__ void rope_append_epilogue(const ProjParams& p, float sum, int mat,
                                                     int group, int r, int ln, int t, int tid,
                                                     float (*half)[32], Sync sync) {
  const float own = __bfloat162float(__float2bfloat16_rn(sum));
  if (tid < 128) half[r][ln] = own;
  sync();
  if (tid >= 128 || t >= p.rows) return;
  const int pos = __ldg(p.pos + t);
  if (pos < 0 || pos / kPage >= p.table_stride) {
    if (mat == 0 && (r & 2) == 0 && (ln >> 2) == 0) record_error(p.err, TVP_DEVERR_BAD_TOKEN);
    return;
  }
  const int kv_dim = kMaxKvHeads * kHeadDim;
  float val = own;
  int feature;
  if (mat < 2) {
    const int pair = (group & 3) * 8 + (ln >> 2), head = group >> 2;
    const bool upper = (r & 2) != 0;  // the d + 32 half
    const float other = half[r ^ 2][ln];
    const float angle = pos * llama3_theta(pair);
    const float c = cosf(angle), sn = sinf(angle);
    __nv_bfloat16 xo, yo;
    rope_rotate(__float2bfloat16_rn(upper ? other : own), __float2bfloat16_rn(upper ? own : other),
                c, sn, xo, yo);
    val = __bfloat162float(upper ? yo : xo);
    feature = head * kHeadDim + pair + (upper ? kHeadDim / 2 : 0);
    if (mat == 0) {
      static_cast<__nv_bfloat16*>(p.out[0])[(size_t)t * p.n[0] + feature] = __float2bfloat16_rn(val);
      return;
    }
  } else {
    feature = group * kProjRows + (ln >> 2) + ((r & 2) ? 8 : 0);
  }
  const int phys = __ldg(p.tables + (size_t)t * p.table_stride + pos / kPage);
  if (phys < 0 || phys >= p.num_pages) {
    if ((r & 2) == 0 && (ln >> 2) == 0) record_error(p.err, TVP_DEVERR_BAD_PAGE);
    return;
  }
  const size_t dst =
      (size_t)(p.layer_row_base + (long long)phys * kPage + pos % kPage) * kv_dim + feature;
  (mat == 1 ? p.k_pool : p.v_pool)[dst] = __float2bfloat16_rn(val);
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
  int n_out = p.n[0], first = 0, mat = 0;
  if (kMats == 1) {
#pragma unroll
    for (int i = 1; i < TVP_PROJ_MAX; ++i)
      if (i < p.count && (int)blockIdx.x >= p.cta_end[i - 1]) {
        w0 = p.w[i];
        out = p.out[i];
        n_out = p.n[i];
        first = p.cta_end[i - 1];
        mat = i;
      }
  }
  const int group = blockIdx.x - first;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int slice = p.k / kWarps;  // a multiple of kProjBlock
  // Rows of the CTA's 16-row tile: MMA rows g and g + 8 are weight rows
  // 16 group + g and + 8; for q and k with the RoPE epilogue they are rows
  // h 64 + 8 u + g and + 32 (group = 4 h + u), the two halves of one
  // rotate-half pair, so that both halves of every pair meet in this CTA.
  const bool pair_rows = kMats == 1 && p.epilogue == kEpiRopeAppend && mat < 2;
  // With the spread RMSNorm, CTA a takes rows 8 a + g and 1024 + 8 a + g:
  // the two features of the norm's leaves 8 a .. 8 a + 7.
  const bool leaf_rows = kMats == 1 && p.norm_out != nullptr && p.norm_spread;
  const int row0 = pair_rows   ? (group >> 2) * kHeadDim + (group & 3) * 8
                   : leaf_rows ? group * 8
                               : group * kProjRows;
  const size_t k0 = (size_t)(row0 + g) * p.k + warp * slice + 8 * q;
  const __nv_bfloat16* wa[kMats];
  wa[0] = w0 + k0;
  if (kMats == 2) wa[kMats - 1] = p.w[1] + k0;
  const bool has_x = g < p.rows;
  const __nv_bfloat16* xr = p.x + (size_t)(has_x ? g : 0) * p.k + warp * slice + 8 * q;

  float c[kMats][4];
#pragma unroll
  for (int m = 0; m < kMats; ++m) c[m][0] = c[m][1] = c[m][2] = c[m][3] = 0.f;
  const int blocks = slice / kProjBlock;
  const size_t row8 = (size_t)(pair_rows ? kHeadDim / 2 : leaf_rows ? kHidden / 2 : 8) * p.k;
  // The residual epilogue's operand (thread (r, ln) < 128: token row t of
  // feature `row`) is the previous grids' output: loaded right after the
  // wait, so that its latency hides behind the weight stream.
  const int r = (threadIdx.x >> 5) & 3, ln = threadIdx.x & 31;
  const int t = 2 * (ln & 3) + (r & 1);
  const int row = leaf_rows ? group * 8 + (ln >> 2) + ((r & 2) ? kHidden / 2 : 0)
                            : group * kProjRows + (ln >> 2) + ((r & 2) ? 8 : 0);
  const bool res_load =
      kMats == 1 && p.epilogue == TVP_PROJ_RESIDUAL && threadIdx.x < 128 && t < p.rows;
  __nv_bfloat16* const res_ptr = static_cast<__nv_bfloat16*>(out) + (size_t)t * n_out + row;
  __nv_bfloat16 res_old = __float2bfloat16_rn(0.f);
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
    if (b0 == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      if (res_load) res_old = *res_ptr;
    }
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
  // accumulator r of lane ln: MMA row (ln / 4) + 8 (r / 2), input row 2 (ln % 4) + r % 2
  float s[kMats];
#pragma unroll
  for (int m = 0; m < kMats; ++m) {
    s[m] = 0.f;
    if (threadIdx.x < 128) {
#pragma unroll
      for (int wi = 0; wi < kWarps; ++wi) s[m] += red[m][wi][r][ln];
    }
  }
  if (kMats == 1 && p.epilogue == kEpiRopeAppend) {
    __shared__ float rope_half[4][32];
    rope_append_epilogue(p, s[0], mat, group, r, ln, t, threadIdx.x, rope_half,
                         [] { __syncthreads(); });
    return;
  }
  float h = 0.f;  // the residual epilogue's new hidden value
  if (threadIdx.x < 128) {
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
        const __nv_bfloat16 hb = res_old + __float2bfloat16_rn(s[0]);  // residualKernel's BF16 add
        ob[idx] = hb;
        h = __bfloat162float(hb);
      } else {
        ob[idx] = __float2bfloat16_rn(s[0]);
      }
    }
  }
  if (leaf_rows) {
    // The reference's sum of squares is a tree over leaves x[i]^2 + x[i +
    // 1024]^2; this CTA holds both features of leaves 8 a .. 8 a + 7, a whole
    // subtree.  Its sum per row goes to norm_part; after every CTA's has
    // arrived, each CTA sums the 128 subtrees by the tree's upper levels
    // (the same order as the reference, so the same r) and normalises its
    // own 16 features.  The CTAs of the grid wait for one another: the host
    // uses this form only when they all fit on the device at once, and the
    // wait is bounded.
    __shared__ float hv[4][32];
    __shared__ float r_rows[kProjMaxTokens];
    __shared__ int arrived;
    if (threadIdx.x < 128) hv[r][ln] = h;
    __syncthreads();
    if (threadIdx.x < 64) {  // r < 2: leaf ln / 4 of row t
      float v = norm_leaf(hv[r][ln], hv[r + 2][ln]);
      float o = __shfl_down_sync(0xffffffffu, v, 4);
      if (((ln >> 2) & 1) == 0) v = __fadd_rn(v, o);
      o = __shfl_down_sync(0xffffffffu, v, 8);
      if (((ln >> 2) & 3) == 0) v = __fadd_rn(v, o);
      o = __shfl_down_sync(0xffffffffu, v, 16);
      if ((ln >> 2) == 0) v = __fadd_rn(v, o);
      if ((ln >> 2) == 0 && t < p.rows) p.norm_part[t * (kHidden / 16) + group] = v;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      // The counter grows by gridDim.x per launch: this launch is complete
      // when it reaches the next multiple.
      unsigned* ctr = reinterpret_cast<unsigned*>(p.counter);
      const unsigned old = atomicAdd(ctr, 1u);
      const unsigned target = (old / gridDim.x + 1u) * gridDim.x;
      bool done = (int)(ld_acquire_u32(ctr) - target) >= 0;
      const unsigned long long start = global_timer_ns();
      while (!done) {
        for (int i = 0; i < 32 && !done; ++i) done = (int)(ld_acquire_u32(ctr) - target) >= 0;
        if (!done && elapsed_ns(start) > (long long)kWaitLimitNs) break;
      }
      if (!done) record_error(p.norm_err, TVP_DEVERR_TIMEOUT);
      arrived = done;
    }
    __syncthreads();
    if (!arrived) return;
    if (warp < p.rows) {  // row `warp`: subtrees 4 lane .. 4 lane + 3, then across lanes
      const float4 v4 = __ldcg(reinterpret_cast<const float4*>(p.norm_part + warp * (kHidden / 16)) + lane);
      float v = __fadd_rn(__fadd_rn(v4.x, v4.y), __fadd_rn(v4.z, v4.w));
#pragma unroll
      for (int off = 1; off < 32; off *= 2) {
        const float o = __shfl_down_sync(0xffffffffu, v, off);
        if ((lane & (2 * off - 1)) == 0) v = __fadd_rn(v, o);
      }
      if (lane == 0) r_rows[warp] = (float)sqrt((double)v / 2048.0 + 1.0e-5);
    }
    __syncthreads();
    if (threadIdx.x < 128 && t < p.rows)
      p.norm_out[(size_t)t * kHidden + row] = __float2bfloat16_rn(
          __fmul_rn(__fdiv_rn(h, r_rows[t]), __bfloat162float(p.norm_gain[row])));
  } else if (kMats == 1 && p.norm_out != nullptr) {
    // The last CTA to finish normalises the rows: every CTA releases its row
    // stores and counts itself done; the last one acquires them all.
    __shared__ int is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(p.counter, 1) == (int)gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    rmsnorm_rows_cta<kWarps * 32>(static_cast<const __nv_bfloat16*>(out), p.norm_gain, p.norm_out,
                                  p.rows);
    if (threadIdx.x == 0) *p.counter = 0;  // ready for the next launch
  }
}

// Down projection + residual + spread RMSNorm, then the next layer's Q, K and
// V projections with RoPE and the page append, in one launch of 128 CTAs x 16
// warps.  The down part is decode_projection_kernel<16, 1, 8> with the spread
// norm, instruction for instruction.  Then, instead of ending:
//  * each CTA's two halves of 8 warps take one Q/K/V item each (items c and
//    128 + c: all 128 q items, and the 64 k and v items on CTAs 0..63), and
//    issue that item's weight loads (its whole k-slice, 8 blocks per lane)
//    right after the down loop, so they fly during the residual epilogue and
//    the grid-wide arrival;
//  * after the arrival every CTA has r for every row, and the hidden rows are
//    final: it normalises all 2048 features of every row into shared memory
//    (the norm's own arithmetic, so the same bits as norm_out), and writes its
//    own 16 features to norm_out as the plain form does;
//  * each half then runs the Q/K/V item exactly as decode_projection_kernel<8,
//    1, 8> does (same k-slices and order, x read from shared memory), with
//    the RoPE + page-append epilogue under its own named barrier.
// So every output has the bits of the two launches it replaces.
constexpr int kXnRow = kHidden + 32;  // normalised row stride in shared memory (conflict-free reads)

__global__ void __launch_bounds__(512, 1)
    down_norm_qkv_kernel(const ProjParams pd, const ProjParams pq) {
  constexpr int kWarps = 16, kUnroll = 8;
  extern __shared__ __align__(16) __nv_bfloat16 xn[];  // [rows][kXnRow]
  __shared__ float red[kWarps][4][32];
  __shared__ float hv[4][32];
  __shared__ float r_rows[kProjMaxTokens];
  __shared__ float rope_half[2][4][32];
  __shared__ int arrived;
  const int group = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, q = lane & 3;
  const int r = warp & 3, ln = lane;
  const int t = 2 * (ln & 3) + (r & 1);

  // ---- down: rows 8a + g and 1024 + 8a + g of w_down (the norm's leaves)
  const int slice = pd.k / kWarps;
  const size_t k0 = (size_t)(group * 8 + g) * pd.k + warp * slice + 8 * q;
  const __nv_bfloat16* wa = pd.w[0] + k0;
  const size_t row8 = (size_t)(kHidden / 2) * pd.k;
  const bool has_x = g < pd.rows;
  const __nv_bfloat16* xr = pd.x + (size_t)(has_x ? g : 0) * pd.k + warp * slice + 8 * q;
  float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
  const int blocks = slice / kProjBlock;
  const int row = group * 8 + (ln >> 2) + ((r & 2) ? kHidden / 2 : 0);
  __nv_bfloat16* hidden = static_cast<__nv_bfloat16*>(pd.out[0]);
  const bool res_load = threadIdx.x < 128 && t < pd.rows;
  __nv_bfloat16* const res_ptr = hidden + (size_t)t * kHidden + row;
  __nv_bfloat16 res_old = __float2bfloat16_rn(0.f);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int b0 = 0; b0 < blocks; b0 += kUnroll) {
    uint4 va[kUnroll], vb[kUnroll], vx[kUnroll];
#pragma unroll
    for (int i = 0; i < kUnroll; ++i) {
      if (b0 + i < blocks) {
        const int off = (b0 + i) * kProjBlock;
        va[i] = ld_stream_v4(wa + off);
        vb[i] = ld_stream_v4(wa + row8 + off);
      }
    }
    if (b0 == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      if (res_load) res_old = *res_ptr;
    }
#pragma unroll
    for (int i = 0; i < kUnroll; ++i)
      if (b0 + i < blocks)
        vx[i] = has_x ? ld_coherent_v4(xr + (b0 + i) * kProjBlock) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int i = 0; i < kUnroll; ++i) {
      if (b0 + i < blocks) {
        mma_bf16_16816(c0, c1, c2, c3, va[i].x, vb[i].x, va[i].y, vb[i].y, vx[i].x, vx[i].y);
        mma_bf16_16816(c0, c1, c2, c3, va[i].z, vb[i].z, va[i].w, vb[i].w, vx[i].z, vx[i].w);
      }
    }
  }

  // ---- this half's Q/K/V item: its weights, loaded now
  const int hh = warp >> 3, hw = warp & 7;
  const int qitem = blockIdx.x + hh * (int)gridDim.x;
  const bool has_q = qitem < pq.cta_end[2];
  int qmat = 0, qgroup = qitem;
  const __nv_bfloat16* qw = pq.w[0];
#pragma unroll
  for (int i = 1; i < 3; ++i)
    if (qitem >= pq.cta_end[i - 1]) {
      qw = pq.w[i];
      qgroup = qitem - pq.cta_end[i - 1];
      qmat = i;
    }
  const bool pair_rows = qmat < 2;
  const int qrow0 = pair_rows ? (qgroup >> 2) * kHeadDim + (qgroup & 3) * 8 : qgroup * kProjRows;
  const size_t qrow8 = (size_t)(pair_rows ? kHeadDim / 2 : 8) * pq.k;
  const int qslice = pq.k / 8;  // 256: 8 blocks of 32
  const __nv_bfloat16* qwa = qw + (size_t)(qrow0 + g) * pq.k + hw * qslice + 8 * q;
  uint4 qa[8], qb[8];
  if (has_q) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      qa[i] = ld_stream_v4(qwa + i * kProjBlock);
      qb[i] = ld_stream_v4(qwa + qrow8 + i * kProjBlock);
    }
  }

  // ---- down epilogue: residual add, leaves, subtree sums, arrival
  red[warp][0][lane] = c0;
  red[warp][1][lane] = c1;
  red[warp][2][lane] = c2;
  red[warp][3][lane] = c3;
  __syncthreads();
  float h = 0.f;
  if (res_load) {
    float sd = 0.f;
#pragma unroll
    for (int wi = 0; wi < kWarps; ++wi) sd += red[wi][r][ln];
    const __nv_bfloat16 hb = res_old + __float2bfloat16_rn(sd);  // residualKernel's BF16 add
    *res_ptr = hb;
    h = __bfloat162float(hb);
  }
  if (threadIdx.x < 128) hv[r][ln] = h;
  __syncthreads();
  if (threadIdx.x < 64) {
    float v = norm_leaf(hv[r][ln], hv[r + 2][ln]);
    float o = __shfl_down_sync(0xffffffffu, v, 4);
    if (((ln >> 2) & 1) == 0) v = __fadd_rn(v, o);
    o = __shfl_down_sync(0xffffffffu, v, 8);
    if (((ln >> 2) & 3) == 0) v = __fadd_rn(v, o);
    o = __shfl_down_sync(0xffffffffu, v, 16);
    if ((ln >> 2) == 0) v = __fadd_rn(v, o);
    if ((ln >> 2) == 0 && t < pd.rows) pd.norm_part[t * (kHidden / 16) + group] = v;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* ctr = reinterpret_cast<unsigned*>(pd.counter);
    const unsigned old = atomicAdd(ctr, 1u);
    const unsigned target = (old / gridDim.x + 1u) * gridDim.x;
    bool done = (int)(ld_acquire_u32(ctr) - target) >= 0;
    const unsigned long long start = global_timer_ns();
    while (!done) {
      for (int i = 0; i < 32 && !done; ++i) done = (int)(ld_acquire_u32(ctr) - target) >= 0;
      if (!done && elapsed_ns(start) > (long long)kWaitLimitNs) break;
    }
    if (!done) record_error(pd.norm_err, TVP_DEVERR_TIMEOUT);
    arrived = done;
  }
  __syncthreads();
  if (!arrived) return;
  if (warp < pd.rows) {
    const float4 v4 =
        __ldcg(reinterpret_cast<const float4*>(pd.norm_part + warp * (kHidden / 16)) + lane);
    float v = __fadd_rn(__fadd_rn(v4.x, v4.y), __fadd_rn(v4.z, v4.w));
#pragma unroll
    for (int off = 1; off < 32; off *= 2) {
      const float o = __shfl_down_sync(0xffffffffu, v, off);
      if ((lane & (2 * off - 1)) == 0) v = __fadd_rn(v, o);
    }
    if (lane == 0) r_rows[warp] = (float)sqrt((double)v / 2048.0 + 1.0e-5);
  }
  __syncthreads();
  if (threadIdx.x < 128 && t < pd.rows)
    pd.norm_out[(size_t)t * kHidden + row] = __float2bfloat16_rn(
        __fmul_rn(__fdiv_rn(h, r_rows[t]), __bfloat162float(pd.norm_gain[row])));
  // every normalised row into shared memory, 8 features per step
  {
    const uint4* hvv = reinterpret_cast<const uint4*>(hidden);
    const uint4* gv = reinterpret_cast<const uint4*>(pd.norm_gain);
    for (int i = threadIdx.x; i < pd.rows * (kHidden / 8); i += 512) {
      const int tr = i / (kHidden / 8), f8 = i % (kHidden / 8);
      const uint4 xw = __ldcg(hvv + i), gw = __ldg(gv + f8);
      const float rr = r_rows[tr];
      auto n2 = [rr](uint32_t a, uint32_t b) {
        return pack_bf16x2(__fmul_rn(__fdiv_rn(bf16lo_to_f32(a), rr), bf16lo_to_f32(b)),
                           __fmul_rn(__fdiv_rn(bf16hi_to_f32(a), rr), bf16hi_to_f32(b)));
      };
      *reinterpret_cast<uint4*>(xn + tr * kXnRow + 8 * f8) =
          make_uint4(n2(xw.x, gw.x), n2(xw.y, gw.y), n2(xw.z, gw.z), n2(xw.w, gw.w));
    }
  }
  __syncthreads();

  // ---- Q/K/V of this half: decode_projection_kernel<8, 1, 8>'s sums
  if (!has_q) return;  // a whole half (every thread of it has the same item)
  float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
  const bool has_xq = g < pq.rows;
  const __nv_bfloat16* xq = xn + (has_xq ? g : 0) * kXnRow + hw * qslice + 8 * q;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint4 vx = has_xq ? *reinterpret_cast<const uint4*>(xq + i * kProjBlock)
                            : make_uint4(0, 0, 0, 0);
    mma_bf16_16816(d0, d1, d2, d3, qa[i].x, qb[i].x, qa[i].y, qb[i].y, vx.x, vx.y);
    mma_bf16_16816(d0, d1, d2, d3, qa[i].z, qb[i].z, qa[i].w, qb[i].w, vx.z, vx.w);
  }
  auto half_sync = [hh] { asm volatile("bar.sync %0, 256;" ::"r"(1 + hh) : "memory"); };
  red[warp][0][lane] = d0;
  red[warp][1][lane] = d1;
  red[warp][2][lane] = d2;
  red[warp][3][lane] = d3;
  half_sync();
  const int tid = threadIdx.x - 256 * hh;
  float sq = 0.f;
  if (tid < 128) {
#pragma unroll
    for (int wi = 0; wi < 8; ++wi) sq += red[8 * hh + wi][r][ln];
  }
  rope_append_epilogue(pq, sq, qmat, qgroup, r, ln, t, tid, rope_half[hh], half_sync);
}

}  // namespace
}  // namespace tvp

using namespace tvp;

namespace {

// Launches K5 over `ctas` CTAs (16 weight rows each): 16 warps (one CTA per
// SM) when each of 8 warps would stream more than 512 columns, so that long
// rows keep enough loads in flight per SM; programmatic dependent launch.
int launch_projection(const ProjParams& p, long long ctas, bool swiglu, cudaStream_t stream) {
  const bool wide = p.k > 4096 && p.k % 512 == 0;
  void (*kernel)(const ProjParams) =
      swiglu ? (wide ? decode_projection_kernel<16, 2, 4> : decode_projection_kernel<8, 2, 4>)
             : (wide ? decode_projection_kernel<16, 1, 8> : decode_projection_kernel<8, 1, 8>);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(wide ? 16 * 32 : 8 * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? TVP_OK : TVP_ERR_RUNTIME;
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

inline bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
  return x < y + nb && y < x + na;
}

// Whether every CTA of a `ctas`-CTA residual+RMSNorm launch of width k can be
// resident at once on the current device (per device, cached), so that they
// may wait for one another.
int norm_spread_fits(int k, int ctas, int* fits) {
  static int cache[64][2] = {};  // 0 unknown, 1 no, 2 yes; [device][16-warp form]
  const bool wide = k > 4096 && k % 512 == 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TVP_ERR_RUNTIME;
  if (dev >= 0 && dev < 64 && cache[dev][wide]) {
    *fits = cache[dev][wide] == 2;
    return TVP_OK;
  }
  int sms = 0, per_sm = 0;
  if (tvp_device_sm_count(&sms) != TVP_OK ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &per_sm, wide ? decode_projection_kernel<16, 1, 8> : decode_projection_kernel<8, 1, 8>,
          wide ? 16 * 32 : 8 * 32, 0) != cudaSuccess)
    return TVP_ERR_RUNTIME;
  *fits = (long long)sms * per_sm >= ctas;
  if (dev >= 0 && dev < 64) cache[dev][wide] = *fits ? 2 : 1;
  return TVP_OK;
}

}  // namespace

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
    // an output must not overlap the input rows
    if (stored && overlaps(out[i], (size_t)rows * n[i] * esize, x, xb)) return TVP_ERR_INVALID_ARGUMENT;
    if (!swiglu || i == 0) ctas += n[i] / kProjRows;
    if (ctas > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
    p.w[i] = reinterpret_cast<const __nv_bfloat16*>(w[i]);
    p.out[i] = out[i];
    p.n[i] = n[i];
    p.cta_end[i] = (int)ctas;
  }
  return launch_projection(p, ctas, swiglu, static_cast<cudaStream_t>(stream));
}

static int prep_residual_rmsnorm(const tvp_bf16* x, int rows, int k, const tvp_bf16* w,
                                 tvp_bf16* hidden, const tvp_bf16* norm_gain, tvp_bf16* norm_out,
                                 void* d_scratch, ProjParams* out) {
  if (!x || !w || !hidden || !norm_gain || !norm_out || !d_scratch || rows < 1 ||
      rows > kProjMaxTokens || k < 256 || k % 256 != 0 || !aligned16(x) || !aligned16(w) ||
      !aligned16(hidden) || !aligned16(norm_gain) || !aligned16(norm_out) || !aligned16(d_scratch))
    return TVP_ERR_INVALID_ARGUMENT;
  const size_t xb = (size_t)rows * k * 2, hb = (size_t)rows * kHidden * 2;
  if (overlaps(hidden, hb, x, xb) || overlaps(norm_out, hb, x, xb) ||
      overlaps(norm_out, hb, hidden, hb) || overlaps(norm_out, hb, norm_gain, kHidden * 2) ||
      overlaps(d_scratch, TVP_NORM_SCRATCH_BYTES, x, xb) ||
      overlaps(d_scratch, TVP_NORM_SCRATCH_BYTES, hidden, hb) ||
      overlaps(d_scratch, TVP_NORM_SCRATCH_BYTES, norm_out, hb) ||
      overlaps(d_scratch, TVP_NORM_SCRATCH_BYTES, norm_gain, kHidden * 2))
    return TVP_ERR_INVALID_ARGUMENT;
  ProjParams& p = *out;
  p = ProjParams{};
  p.x = reinterpret_cast<const __nv_bfloat16*>(x);
  p.count = 1;
  p.rows = rows;
  p.k = k;
  p.epilogue = TVP_PROJ_RESIDUAL;
  p.w[0] = reinterpret_cast<const __nv_bfloat16*>(w);
  p.out[0] = hidden;
  p.n[0] = kHidden;
  p.cta_end[0] = kHidden / kProjRows;
  p.norm_gain = reinterpret_cast<const __nv_bfloat16*>(norm_gain);
  p.norm_out = reinterpret_cast<__nv_bfloat16*>(norm_out);
  uint8_t* scratch = static_cast<uint8_t*>(d_scratch);
  p.counter = reinterpret_cast<int*>(scratch);
  p.norm_err = reinterpret_cast<int32_t*>(scratch + 4);
  p.norm_part = reinterpret_cast<float*>(scratch + 256);
  return TVP_OK;
}

// The spread form's CTAs wait for one another: only when the device holds the
// whole grid at once (148 SMs for 128 CTAs on a B200).  After every argument
// check, since it asks the device.
static int choose_norm_form(ProjParams* p) {
  int spread = 0;
  if (norm_spread_fits(p->k, kHidden / kProjRows, &spread) != TVP_OK) return TVP_ERR_RUNTIME;
  p->norm_spread = spread;
  return TVP_OK;
}

int tvp_decode_projection_residual_rmsnorm(const tvp_bf16* x, int rows, int k, const tvp_bf16* w,
                                           tvp_bf16* hidden, const tvp_bf16* norm_gain,
                                           tvp_bf16* norm_out, void* d_scratch,
                                           tvp_stream_t stream) {
  ProjParams p;
  int rc = prep_residual_rmsnorm(x, rows, k, w, hidden, norm_gain, norm_out, d_scratch, &p);
  if (rc == TVP_OK) rc = choose_norm_form(&p);
  if (rc != TVP_OK) return rc;
  return launch_projection(p, kHidden / kProjRows, false, static_cast<cudaStream_t>(stream));
}

static int prep_qkv_rope_append(const tvp_bf16* x, int rows, int k, const tvp_bf16* w_q,
                                const tvp_bf16* w_k, const tvp_bf16* w_v, tvp_bf16* q_out,
                                tvp_bf16* k_pool, tvp_bf16* v_pool, int num_pages, int num_layers,
                                int layer, const int32_t* d_block_tables, int table_stride,
                                const int32_t* d_positions, int32_t* d_error, ProjParams* out) {
  constexpr int kQ = TVP_Q_HEADS * kHeadDim, kKv = kMaxKvHeads * kHeadDim;
  if (!x || !w_q || !w_k || !w_v || !q_out || !k_pool || !v_pool || !d_block_tables ||
      !d_positions || rows < 1 || rows > kProjMaxTokens || k < 256 || k % 256 != 0 ||
      num_pages <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || table_stride <= 0 ||
      !aligned16(x) || !aligned16(w_q) || !aligned16(w_k) || !aligned16(w_v) ||
      (reinterpret_cast<uintptr_t>(q_out) & 1u) || (reinterpret_cast<uintptr_t>(k_pool) & 1u) ||
      (reinterpret_cast<uintptr_t>(v_pool) & 1u))
    return TVP_ERR_INVALID_ARGUMENT;
  if ((long long)num_layers * num_pages * kPage > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
  if (overlaps(q_out, (size_t)rows * kQ * 2, x, (size_t)rows * k * 2)) return TVP_ERR_INVALID_ARGUMENT;
  ProjParams& p = *out;
  p = ProjParams{};
  p.x = reinterpret_cast<const __nv_bfloat16*>(x);
  p.count = 3;
  p.rows = rows;
  p.k = k;
  p.epilogue = kEpiRopeAppend;
  p.w[0] = reinterpret_cast<const __nv_bfloat16*>(w_q);
  p.w[1] = reinterpret_cast<const __nv_bfloat16*>(w_k);
  p.w[2] = reinterpret_cast<const __nv_bfloat16*>(w_v);
  p.out[0] = q_out;
  p.n[0] = kQ;
  p.n[1] = kKv;
  p.n[2] = kKv;
  p.cta_end[0] = kQ / kProjRows;
  p.cta_end[1] = (kQ + kKv) / kProjRows;
  p.cta_end[2] = (kQ + 2 * kKv) / kProjRows;
  p.k_pool = reinterpret_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = reinterpret_cast<__nv_bfloat16*>(v_pool);
  p.layer_row_base = (long long)layer * num_pages * kPage;
  p.num_pages = num_pages;
  p.table_stride = table_stride;
  p.tables = d_block_tables;
  p.pos = d_positions;
  p.err = d_error;
  return TVP_OK;
}

int tvp_decode_qkv_rope_append(const tvp_bf16* x, int rows, int k, const tvp_bf16* w_q,
                               const tvp_bf16* w_k, const tvp_bf16* w_v, tvp_bf16* q_out,
                               tvp_bf16* k_pool, tvp_bf16* v_pool, int num_pages, int num_layers,
                               int layer, const int32_t* d_block_tables, int table_stride,
                               const int32_t* d_positions, int32_t* d_error, tvp_stream_t stream) {
  ProjParams p;
  const int rc = prep_qkv_rope_append(x, rows, k, w_q, w_k, w_v, q_out, k_pool, v_pool, num_pages,
                                      num_layers, layer, d_block_tables, table_stride, d_positions,
                                      d_error, &p);
  if (rc != TVP_OK) return rc;
  return launch_projection(p, p.cta_end[2], false, static_cast<cudaStream_t>(stream));
}

int tvp_decode_down_norm_qkv(const tvp_bf16* x, int rows, int k, const tvp_bf16* w_down,
                             tvp_bf16* hidden, const tvp_bf16* norm_gain, tvp_bf16* norm_out,
                             void* d_scratch, const tvp_bf16* w_q, const tvp_bf16* w_k,
                             const tvp_bf16* w_v, tvp_bf16* q_out, tvp_bf16* k_pool,
                             tvp_bf16* v_pool, int num_pages, int num_layers, int layer,
                             const int32_t* d_block_tables, int table_stride,
                             const int32_t* d_positions, int32_t* d_error, tvp_stream_t stream) {
  ProjParams pd, pq;
  int rc = prep_residual_rmsnorm(x, rows, k, w_down, hidden, norm_gain, norm_out, d_scratch, &pd);
  if (rc != TVP_OK) return rc;
  rc = prep_qkv_rope_append(norm_out, rows, kHidden, w_q, w_k, w_v, q_out, k_pool, v_pool,
                            num_pages, num_layers, layer, d_block_tables, table_stride,
                            d_positions, d_error, &pq);
  if (rc != TVP_OK) return rc;
  if (overlaps(q_out, (size_t)rows * kHidden * 2, hidden, (size_t)rows * kHidden * 2))
    return TVP_ERR_INVALID_ARGUMENT;
  if (k % 512 != 0 || k <= 4096) return TVP_ERR_UNSUPPORTED;
  rc = choose_norm_form(&pd);
  if (rc != TVP_OK) return rc;
  // the fused kernel's fixed shape: 16 warps over k, the spread norm, 128
  // CTAs whose two halves cover the 192 Q/K/V items
  if (!pd.norm_spread) return TVP_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kHidden / kProjRows);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = (size_t)rows * kXnRow * sizeof(__nv_bfloat16);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, down_norm_qkv_kernel, pd, pq) == cudaSuccess ? TVP_OK
                                                                             : TVP_ERR_RUNTIME;
}



}  // extern "C"
