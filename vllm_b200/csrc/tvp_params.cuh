// Kernel parameter blocks of the paged-KV hot path and the launchers that
// take them, shared by the kernel files and the C-ABI layer.
#pragma once

#include "tvp_common.cuh"

namespace tvp {

// K1 (tvp_append.cu)
struct AppendParams {
  __nv_bfloat16* k_pool;
  __nv_bfloat16* v_pool;
  long long layer_row_base;  // layer * num_pages * 16
  int num_pages;
  const int32_t* tables;
  int table_stride;
  int num_seqs;
  const int32_t* token_seq;  // nullable: token i -> block-table row i
  const int32_t* token_pos;
  __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* q;
  int kv_heads;
  int q_heads;
  int flags;
  int32_t* err;
};

// K2 (tvp_decode.cu)
struct DecodeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_pool;
  const __nv_bfloat16* v_pool;
  __nv_bfloat16* out;
  const int32_t* tables;
  const int32_t* seq_lens;
  const int32_t* header;
  const int32_t* cu;
  // Per CTA taking pages: {s0, cu[s0], cu[s0 + 1], 0}, s0 the sequence holding
  // its first page (so the CTA starts without walking the prefix sums).
  const int4* cta_start;
  int32_t* counters;
  float* partials;
  long long layer_row_base;  // layer * num_pages * 16
  int num_pages;
  int table_stride;
  int batch;
  int kv_heads;      // KV heads the pools hold (1, 2, 4 or 8)
  float scale_log2;  // scale * log2(e)
  int32_t* err;
  // KV-head-shard gather (tvp_paged_decode_attention_gather), else null / 0:
  // outputs go to every rank's gathered rows [B][2048] at this rank's heads
  // instead of `out`, and the last CTA to finish adds 1 to every rank's flag.
  __nv_bfloat16* const* peer_rows;  // [world] device pointers
  int32_t* const* peer_flags;       // [world] device pointers
  int32_t* done_counter;            // CTAs finished in this launch (the last resets it)
  int world, rank;
  int32_t flag_target;              // this rank's flag once every rank signalled this launch
};

// K2c (tvp_compat.cu)
struct CompatParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k_pool;
  const __nv_bfloat16* v_pool;
  __nv_bfloat16* out;
  const int32_t* tables;
  const int32_t* seq_lens;
  long long layer_row_base;
  int num_pages;
  int table_stride;
  int kv_heads;
  float scale;
  int32_t* err;
};

// K3 (tvp_prefill.cu)
struct PrefillParams {
  const __nv_bfloat16* q;  // [num_tokens][q_heads * 64]
  const __nv_bfloat16* k_pool;
  const __nv_bfloat16* v_pool;
  __nv_bfloat16* out;      // [num_tokens][q_heads * 64]
  const int32_t* tables;   // [num_seqs][table_stride]
  const int32_t* cu_q;     // [num_seqs + 1] query-token offsets
  const int32_t* q_pos0;   // [num_seqs] position of each sequence's first query token
  long long layer_row_base;
  int num_pages;
  int table_stride;
  int kv_heads;
  float scale;
  int scale_pow2;  // scale is a positive power of two (the score rounding commutes with it)
  int32_t* err;
};

// m[4], l[4], o[4][64] of one (split-K slot, KV head).
constexpr int kPartialFloats = 2 * kGroup + kGroup * kHeadDim;

cudaError_t launch_rope_append(const AppendParams& p, int num_tokens, cudaStream_t stream);
cudaError_t launch_decode_plan(const int32_t* lens, int batch, int table_stride, int num_ctas,
                               int kv_heads, int32_t* header, int32_t* cu, int4* cta_start,
                               int32_t* counters, int32_t* err, cudaStream_t stream);
// Dispatches on p.kv_heads: 8 -> tvp_decode.cu, 1, 2, 4 -> tvp_decode_heads.cu.
cudaError_t launch_paged_decode(const DecodeParams& p, long long pool_rows, int num_ctas,
                                cudaStream_t stream);
cudaError_t launch_paged_decode_heads(const DecodeParams& p, const CUtensorMap& k_map,
                                      const CUtensorMap& v_map, int num_ctas,
                                      cudaStream_t stream);
// Host-side argument checks of tvp_paged_decode_attention, everything but the
// workspace: TVP_OK or the error code that entry point returns.  No CUDA call.
int check_decode_args(const void* q, const void* k_pool, const void* v_pool, const void* out,
                      int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                      const int32_t* d_block_tables, int table_stride, const int32_t* d_seq_lens,
                      int batch, float scale, int mode, int num_ctas);
// Argument checks, workspace layout and parameter block of the FAST decode
// (shared by tvp_paged_decode_attention and its gather form); TVP_OK or an error.
int prepare_decode(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                   int num_layers, int layer, int kv_heads, int q_heads,
                   const int32_t* d_block_tables, int table_stride, const int32_t* d_seq_lens,
                   int batch, float scale, int num_ctas, void* d_workspace,
                   size_t workspace_bytes, int32_t* d_error, DecodeParams* p, long long* pool_rows,
                   int* ctas);
// 2-D tensor map over a pool of `rows` token rows of kv_heads x 64 channels;
// box = one KV head of one page (64 channels x 16 rows).
bool pool_tensor_map(const void* pool, long long rows, int kv_heads, CUtensorMap* out);
// 3-D view of the same pool, (channel, row, head) with strides (2 B,
// kv_heads x 128 B, 128 B); box = a whole page of every head ({64, 16,
// kv_heads}), which lands as kv_heads head-major 2 KiB tiles with the same
// 128-byte swizzle as kv_heads boxes of the 2-D map.
bool page_tensor_map(const void* pool, long long rows, int kv_heads, CUtensorMap* out);
cudaError_t launch_compat_decode(const CompatParams& p, int batch, cudaStream_t stream);
cudaError_t launch_paged_prefill(const PrefillParams& p, long long pool_rows, int max_q_len,
                                 int num_seqs, cudaStream_t stream);

}  // namespace tvp
