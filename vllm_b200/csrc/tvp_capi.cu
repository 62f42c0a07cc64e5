// C-ABI entry points of the kernels (include/tvp_paged.h): argument checks on
// the host, workspace layout, launch.  No allocation happens here.
#include <cmath>
#include <cstring>

#include "tvp_params.cuh"

namespace tvp {

namespace {

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WorkspaceLayout {
  size_t header, cu, cta_start, counters, partials, total;
};

// header | cu[batch + 1] | cta_start[num_ctas] (int4) | counters[batch][kv_heads] |
// partials[2 num_ctas][kv_heads]
WorkspaceLayout workspace_layout(int batch, int kv_heads, int num_ctas) {
  WorkspaceLayout w;
  w.header = 0;
  w.cu = 256;
  w.cta_start = align_up(w.cu + (size_t)(batch + 1) * 4, 256);
  w.counters = align_up(w.cta_start + (size_t)num_ctas * 16, 256);
  w.partials = align_up(w.counters + (size_t)batch * kv_heads * 4, 256);
  w.total = align_up(w.partials + (size_t)num_ctas * 2 * kv_heads * kPartialFloats * 4, 256);
  return w;
}

// KV heads per pool the decode kernels provide: the model's 8, or the 4, 2 or
// 1 that each GPU holds when the heads are sharded over 2, 4 or 8 GPUs.
inline bool decode_heads_supported(int kv_heads) {
  return kv_heads == 1 || kv_heads == 2 || kv_heads == 4 || kv_heads == kMaxKvHeads;
}

int sm_count_cached(int* out) {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return TVP_ERR_RUNTIME;
  if (dev >= 0 && dev < 64 && counts[dev] > 0) {
    *out = counts[dev];
    return TVP_OK;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return TVP_ERR_RUNTIME;
  if (dev >= 0 && dev < 64) counts[dev] = sms;
  *out = sms;
  return TVP_OK;
}

int resolve_ctas(int num_ctas, int* out) {
  if (num_ctas < 0) return TVP_ERR_INVALID_ARGUMENT;
  if (num_ctas > 0) {
    *out = num_ctas;
    return TVP_OK;
  }
  return sm_count_cached(out);
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int map_cuda(cudaError_t e) { return e == cudaSuccess ? TVP_OK : TVP_ERR_RUNTIME; }

}  // namespace

int check_decode_args(const void* q, const void* k_pool, const void* v_pool, const void* out,
                      int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                      const int32_t* d_block_tables, int table_stride, const int32_t* d_seq_lens,
                      int batch, float scale, int mode, int num_ctas) {
  if (!q || !k_pool || !v_pool || !out || !d_block_tables || !d_seq_lens || num_pages <= 0 ||
      num_layers <= 0 || layer < 0 || layer >= num_layers || table_stride <= 0 || batch <= 0 ||
      num_ctas < 0 || !std::isfinite(scale))
    return TVP_ERR_INVALID_ARGUMENT;
  if (!decode_heads_supported(kv_heads) || q_heads != kv_heads * kGroup) return TVP_ERR_UNSUPPORTED;
  if (mode != TVP_MODE_FAST && mode != TVP_MODE_COMPAT) return TVP_ERR_UNSUPPORTED;
  // TMA row coordinates are 32-bit: the pools may hold at most 2^31 - 1 token rows.
  if ((long long)num_layers * num_pages * kPage > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4) || !aligned(out, 16))
    return TVP_ERR_INVALID_ARGUMENT;
  return TVP_OK;
}

int prepare_decode(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                   int num_layers, int layer, int kv_heads, int q_heads,
                   const int32_t* d_block_tables, int table_stride, const int32_t* d_seq_lens,
                   int batch, float scale, int num_ctas, void* d_workspace,
                   size_t workspace_bytes, int32_t* d_error, DecodeParams* p, long long* pool_rows,
                   int* ctas) {
  if (!q || !k_pool || !v_pool || !d_block_tables || !d_seq_lens || num_pages <= 0 ||
      num_layers <= 0 || layer < 0 || layer >= num_layers || table_stride <= 0 || batch <= 0 ||
      num_ctas < 0 || !std::isfinite(scale))
    return TVP_ERR_INVALID_ARGUMENT;
  if (!decode_heads_supported(kv_heads) || q_heads != kv_heads * kGroup) return TVP_ERR_UNSUPPORTED;
  if ((long long)num_layers * num_pages * kPage > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4))
    return TVP_ERR_INVALID_ARGUMENT;
  const int rc = resolve_ctas(num_ctas, ctas);
  if (rc != TVP_OK) return rc;
  const WorkspaceLayout w = workspace_layout(batch, kv_heads, *ctas);
  if (!d_workspace || workspace_bytes < w.total || !aligned(d_workspace, 256)) return TVP_ERR_WORKSPACE;
  char* base = static_cast<char*>(d_workspace);
  *p = DecodeParams{};
  p->q = reinterpret_cast<const __nv_bfloat16*>(q);
  p->k_pool = reinterpret_cast<const __nv_bfloat16*>(k_pool);
  p->v_pool = reinterpret_cast<const __nv_bfloat16*>(v_pool);
  p->tables = d_block_tables;
  p->seq_lens = d_seq_lens;
  p->header = reinterpret_cast<const int32_t*>(base + w.header);
  p->cu = reinterpret_cast<const int32_t*>(base + w.cu);
  p->cta_start = reinterpret_cast<const int4*>(base + w.cta_start);
  p->counters = reinterpret_cast<int32_t*>(base + w.counters);
  p->partials = reinterpret_cast<float*>(base + w.partials);
  p->layer_row_base = (long long)layer * num_pages * kPage;
  p->num_pages = num_pages;
  p->table_stride = table_stride;
  p->batch = batch;
  p->kv_heads = kv_heads;
  p->scale_log2 = scale * 1.4426950408889634f;
  p->err = d_error;
  p->world = 1;
  *pool_rows = (long long)num_layers * num_pages * kPage;
  return TVP_OK;
}

}  // namespace tvp

using namespace tvp;

extern "C" {

const char* tvp_strerror(int code) {
  switch (code) {
    case TVP_OK: return "ok";
    case TVP_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TVP_ERR_RUNTIME: return "CUDA runtime error";
    case TVP_ERR_NO_FREE_BLOCKS: return "paged KV cache has no free blocks";
    case TVP_ERR_UNSUPPORTED: return "unsupported geometry or mode";
    case TVP_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown error";
  }
}

int tvp_version(void) { return 1; }

int tvp_device_sm_count(int* out_sms) {
  if (!out_sms) return TVP_ERR_INVALID_ARGUMENT;
  return sm_count_cached(out_sms);
}

int tvp_rope_append(tvp_bf16* k_pool, tvp_bf16* v_pool, int num_pages, int num_layers, int layer,
                    int kv_heads, const int32_t* d_block_tables, int table_stride, int num_seqs,
                    const int32_t* d_token_seq, const int32_t* d_token_pos, int num_tokens,
                    tvp_bf16* k, const tvp_bf16* v, tvp_bf16* q, int q_heads, int flags,
                    int32_t* d_error, tvp_stream_t stream) {
  if (num_tokens < 0 || !k_pool || !v_pool || !d_block_tables || !d_token_pos || !k || !v ||
      num_pages <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || table_stride <= 0 ||
      num_seqs <= 0 || (flags & ~(TVP_APPEND_ROPE_K | TVP_APPEND_ROPE_Q | TVP_APPEND_WRITEBACK_K)))
    return TVP_ERR_INVALID_ARGUMENT;
  if ((flags & TVP_APPEND_ROPE_Q) && (!q || q_heads <= 0 || q_heads > 64))
    return TVP_ERR_INVALID_ARGUMENT;
  if (kv_heads <= 0 || kv_heads > kMaxKvHeads) return TVP_ERR_UNSUPPORTED;
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(v, 16) || !aligned(k, 2))
    return TVP_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return TVP_OK;
  AppendParams p;
  p.k_pool = reinterpret_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = reinterpret_cast<__nv_bfloat16*>(v_pool);
  p.layer_row_base = (long long)layer * num_pages * kPage;
  p.num_pages = num_pages;
  p.tables = d_block_tables;
  p.table_stride = table_stride;
  p.num_seqs = num_seqs;
  p.token_seq = d_token_seq;
  p.token_pos = d_token_pos;
  p.k = reinterpret_cast<__nv_bfloat16*>(k);
  p.v = reinterpret_cast<const __nv_bfloat16*>(v);
  p.q = reinterpret_cast<__nv_bfloat16*>(q);
  p.kv_heads = kv_heads;
  p.q_heads = q_heads;
  p.flags = flags;
  p.err = d_error;
  return map_cuda(launch_rope_append(p, num_tokens, static_cast<cudaStream_t>(stream)));
}

size_t tvp_decode_workspace_bytes(int batch, int kv_heads, int num_ctas) {
  if (batch <= 0 || !decode_heads_supported(kv_heads)) return 0;
  int ctas = 0;
  if (resolve_ctas(num_ctas, &ctas) != TVP_OK) return 0;
  return workspace_layout(batch, kv_heads, ctas).total;
}

int tvp_decode_plan(const int32_t* d_seq_lens, int batch, int table_stride, int kv_heads,
                    int num_ctas, void* d_workspace, size_t workspace_bytes, int32_t* d_error,
                    tvp_stream_t stream) {
  if (!d_seq_lens || batch <= 0 || table_stride <= 0 || num_ctas < 0)
    return TVP_ERR_INVALID_ARGUMENT;
  if (!decode_heads_supported(kv_heads)) return TVP_ERR_UNSUPPORTED;
  int ctas = 0;
  int rc = resolve_ctas(num_ctas, &ctas);
  if (rc != TVP_OK) return rc;
  const WorkspaceLayout w = workspace_layout(batch, kv_heads, ctas);
  if (!d_workspace || workspace_bytes < w.total || !aligned(d_workspace, 256)) return TVP_ERR_WORKSPACE;
  char* base = static_cast<char*>(d_workspace);
  return map_cuda(launch_decode_plan(d_seq_lens, batch, table_stride, ctas, kv_heads,
                                     reinterpret_cast<int32_t*>(base + w.header),
                                     reinterpret_cast<int32_t*>(base + w.cu),
                                     reinterpret_cast<int4*>(base + w.cta_start),
                                     reinterpret_cast<int32_t*>(base + w.counters), d_error,
                                     static_cast<cudaStream_t>(stream)));
}

int tvp_paged_decode_attention(const tvp_bf16* q, const tvp_bf16* k_pool, const tvp_bf16* v_pool,
                               int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                               const int32_t* d_block_tables, int table_stride,
                               const int32_t* d_seq_lens, int batch, float scale, int mode,
                               int num_ctas, void* d_workspace, size_t workspace_bytes,
                               tvp_bf16* out, int32_t* d_error, tvp_stream_t stream) {
  const int arc = check_decode_args(q, k_pool, v_pool, out, num_pages, num_layers, layer, kv_heads,
                                    q_heads, d_block_tables, table_stride, d_seq_lens, batch,
                                    scale, mode, num_ctas);
  if (arc != TVP_OK) return arc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (mode == TVP_MODE_COMPAT) {
    CompatParams p;
    p.q = reinterpret_cast<const __nv_bfloat16*>(q);
    p.k_pool = reinterpret_cast<const __nv_bfloat16*>(k_pool);
    p.v_pool = reinterpret_cast<const __nv_bfloat16*>(v_pool);
    p.out = reinterpret_cast<__nv_bfloat16*>(out);
    p.tables = d_block_tables;
    p.seq_lens = d_seq_lens;
    p.layer_row_base = (long long)layer * num_pages * kPage;
    p.num_pages = num_pages;
    p.table_stride = table_stride;
    p.kv_heads = kv_heads;
    p.scale = scale;
    p.err = d_error;
    return map_cuda(launch_compat_decode(p, batch, st));
  }
  DecodeParams p;
  long long pool_rows = 0;
  int ctas = 0;
  const int rc = prepare_decode(q, k_pool, v_pool, num_pages, num_layers, layer, kv_heads, q_heads,
                                d_block_tables, table_stride, d_seq_lens, batch, scale, num_ctas,
                                d_workspace, workspace_bytes, d_error, &p, &pool_rows, &ctas);
  if (rc != TVP_OK) return rc;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  return map_cuda(launch_paged_decode(p, pool_rows, ctas, st));
}

int tvp_paged_prefill_attention(const tvp_bf16* q, const tvp_bf16* k_pool, const tvp_bf16* v_pool,
                                int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                                const int32_t* d_block_tables, int table_stride,
                                const int32_t* d_cu_q, const int32_t* d_q_pos0, int num_seqs,
                                int max_q_len, float scale, tvp_bf16* out, int32_t* d_error,
                                tvp_stream_t stream) {
  if (!q || !k_pool || !v_pool || !out || !d_block_tables || !d_cu_q || !d_q_pos0 ||
      num_pages <= 0 || num_layers <= 0 || layer < 0 || layer >= num_layers || table_stride <= 0 ||
      num_seqs <= 0 || num_seqs > 65535 || max_q_len < 0 || !std::isfinite(scale))
    return TVP_ERR_INVALID_ARGUMENT;
  if (max_q_len > 65535 * 32) return TVP_ERR_UNSUPPORTED;  // one grid row per 32-token tile
  if (!decode_heads_supported(kv_heads) || q_heads != kv_heads * kGroup) return TVP_ERR_UNSUPPORTED;
  if ((long long)num_layers * num_pages * kPage > 0x7fffffffLL) return TVP_ERR_UNSUPPORTED;
  // q rows are read and output rows written as 16-byte vectors.
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 16) || !aligned(out, 16))
    return TVP_ERR_INVALID_ARGUMENT;
  if (max_q_len == 0) return TVP_OK;
  PrefillParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.k_pool = reinterpret_cast<const __nv_bfloat16*>(k_pool);
  p.v_pool = reinterpret_cast<const __nv_bfloat16*>(v_pool);
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.tables = d_block_tables;
  p.cu_q = d_cu_q;
  p.q_pos0 = d_q_pos0;
  p.layer_row_base = (long long)layer * num_pages * kPage;
  p.num_pages = num_pages;
  p.table_stride = table_stride;
  p.kv_heads = kv_heads;
  p.scale = scale;
  int e2 = 0;
  p.scale_pow2 = scale > 0.f && std::frexp(scale, &e2) == 0.5f;
  p.err = d_error;
  return map_cuda(launch_paged_prefill(p, (long long)num_layers * num_pages * kPage, max_q_len,
                                       num_seqs, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
