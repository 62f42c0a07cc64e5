// K1 — fused llama3 RoPE + paged KV append (prefill and decode forms).
//
// One CTA per token row.  The CTA rotates the row's q heads in place (optional),
// rotates its K heads, and writes K and V straight into the token's physical
// page slot.  Replaces rope/ropeBatch (src/model/RoPe.cu:31-62) followed by
// storePagedKV (src/model/paged_kvcache.cu:119-139, a host loop of synchronous
// D2D copies) or storePagedKVBatchKernel (src/model/paged_attention.cu:89-99).
#include "tvp_params.cuh"
#include "tvp_rope.cuh"

namespace tvp {

__global__ void __launch_bounds__(256) rope_append_kernel(AppendParams p) {
  // A decode attention launched after this one (programmatic dependent
  // launch) may start its own prologue now: it reads what this kernel writes
  // (q and each row's last page) only after its griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int t = blockIdx.x;
  const int pos = p.token_pos[t];
  const int seq = p.token_seq ? p.token_seq[t] : t;
  const int kv_dim = p.kv_heads * kHeadDim;

  // cos and sin of angle = pos * theta(pair) for the 32 pairs, shared by all
  // of the row's q and K heads.
  __shared__ float cos_pair[kHeadDim / 2], sin_pair[kHeadDim / 2];
  if (p.flags & (TVP_APPEND_ROPE_Q | TVP_APPEND_ROPE_K)) {
    if (threadIdx.x < kHeadDim / 2) {
      const float angle = pos * llama3_theta(threadIdx.x);
      cos_pair[threadIdx.x] = cosf(angle);
      sin_pair[threadIdx.x] = sinf(angle);
    }
    __syncthreads();
  }

  if (p.flags & TVP_APPEND_ROPE_Q) {
    __nv_bfloat16* qrow = p.q + (size_t)t * p.q_heads * kHeadDim;
    const int pairs = p.q_heads * (kHeadDim / 2);
    for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
      const int pair = i % (kHeadDim / 2);
      const int x_index = (i / (kHeadDim / 2)) * kHeadDim + pair;
      const int y_index = x_index + kHeadDim / 2;
      __nv_bfloat16 xo, yo;
      rope_rotate(qrow[x_index], qrow[y_index], cos_pair[pair], sin_pair[pair], xo, yo);
      qrow[x_index] = xo;
      qrow[y_index] = yo;
    }
  }

  const bool row_ok = seq >= 0 && seq < p.num_seqs && pos >= 0 && (pos / kPage) < p.table_stride;
  if (!row_ok) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_TOKEN);
    return;
  }
  const int phys = p.tables[(size_t)seq * p.table_stride + pos / kPage];
  if (phys < 0 || phys >= p.num_pages) {
    if (threadIdx.x == 0) record_error(p.err, TVP_DEVERR_BAD_PAGE);
    return;
  }
  const size_t dst = (size_t)(p.layer_row_base + (long long)phys * kPage + pos % kPage) * kv_dim;
  __nv_bfloat16* krow = p.k + (size_t)t * kv_dim;

  const int kpairs = p.kv_heads * (kHeadDim / 2);
  for (int i = threadIdx.x; i < kpairs; i += blockDim.x) {
    const int pair = i % (kHeadDim / 2);
    const int x_index = (i / (kHeadDim / 2)) * kHeadDim + pair;
    const int y_index = x_index + kHeadDim / 2;
    __nv_bfloat16 xo = krow[x_index], yo = krow[y_index];
    if (p.flags & TVP_APPEND_ROPE_K) rope_rotate(xo, yo, cos_pair[pair], sin_pair[pair], xo, yo);
    p.k_pool[dst + x_index] = xo;
    p.k_pool[dst + y_index] = yo;
    if (p.flags & TVP_APPEND_WRITEBACK_K) {
      krow[x_index] = xo;
      krow[y_index] = yo;
    }
  }

  const uint4* vsrc = reinterpret_cast<const uint4*>(p.v + (size_t)t * kv_dim);
  uint4* vdst = reinterpret_cast<uint4*>(p.v_pool + dst);
  for (int i = threadIdx.x; i < kv_dim / 8; i += blockDim.x) vdst[i] = vsrc[i];
}

cudaError_t launch_rope_append(const AppendParams& p, int num_tokens, cudaStream_t stream) {
  rope_append_kernel<<<num_tokens, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace tvp
