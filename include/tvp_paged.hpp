// tvp_paged.hpp — C++ host API of the B200 paged-KV path, namespace tvp.
//
// Mirrors the reference's host interface for the paged path
// (include/paged_kvcache.cuh:6-28, include/paged_attention.cuh:6-27,
// include/rope.cuh:5-6): same type and function names, same argument meaning,
// same exception types (std::invalid_argument for bad arguments,
// std::runtime_error for CUDA failures and exhaustion).  Differences, all
// deliberate:
//   * the 1024-token context cap is PagedKVCache::max_seq_len (default 1024);
//   * PagedBatchMetadata keeps its device tables between steps (no per-step
//     cudaMalloc/cudaFree) and carries the decode plan workspace;
//   * computePagedAttentionScores + softmaxRows + pagedAttentionScoresTimesV
//     become one call, pagedDecodeAttention, and ropeBatch(q) + ropeBatch(k) +
//     storePagedKVBatch become storePagedKVBatch(..., q, k, v);
//   * every call takes an optional cudaStream_t (default: legacy stream).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <vector>

#include "tvp_paged.h"

namespace tvp {

constexpr int BLOCK_SIZE = TVP_PAGE_TOKENS;

struct PagedKVCache {
  __nv_bfloat16* k_blocks = nullptr;
  __nv_bfloat16* v_blocks = nullptr;
  int num_blocks = 0;
  int block_size = BLOCK_SIZE;
  std::vector<int> free_blocks;
  int num_layers = 16;
  int kv_heads = TVP_KV_HEADS;
  int max_seq_len = 1024;
  bool device_storage = true;
  // Device staging for prefill appends (block table + token positions).
  int* d_scratch = nullptr;
  size_t scratch_ints = 0;
  int* d_error = nullptr;
};

struct SequenceKVState {
  std::vector<int> block_table;
  int current_seq_len = 0;
};

struct PagedBatchMetadata {
  int* block_tables = nullptr;  // device [max_batch][table_stride], -1 padded
  int* positions = nullptr;     // device [max_batch]: current_seq_len per row
  int* lengths_dev = nullptr;   // device [max_batch]: attended length = position + 1
  int batch_size = 0;
  int table_stride = 0;
  int max_batch = 0;
  int num_ctas = 0;
  std::vector<int> lengths;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  int* d_error = nullptr;
  int* h_staging = nullptr;  // pinned host staging of tables | positions | lengths
  cudaEvent_t staged = nullptr;
};

void allocatePagedKVCache(PagedKVCache& cache, int num_blocks, int num_layers = 16,
                          int max_seq_len = 1024, bool device_storage = true);
void freePagedKVCache(PagedKVCache& cache);
int allocatePhysicalBlock(PagedKVCache& cache);
void freePhysicalBlock(PagedKVCache& cache, int physical_block);
void freeSequenceBlocks(PagedKVCache& cache, SequenceKVState& sequence);
void reserveSequenceBlocks(PagedKVCache& cache, SequenceKVState& sequence, int total_seq_len);
// storePagedKV: k, v device [num_tokens][512].  With apply_rope the fused
// kernel also applies llama3 RoPE to k (in place) and, when rope_q is given,
// to q [num_tokens][2048] — rope(q), rope(k), storePagedKV in one launch.
void storePagedKV(PagedKVCache& cache, SequenceKVState& sequence, int layer,
                  __nv_bfloat16* k, const __nv_bfloat16* v, int num_tokens,
                  bool apply_rope = false, __nv_bfloat16* rope_q = nullptr,
                  cudaStream_t stream = nullptr);

void createPagedBatch(PagedBatchMetadata& metadata, int max_batch, int table_stride);
void destroyPagedBatch(PagedBatchMetadata& metadata);
void preparePagedBatch(PagedKVCache& cache, const std::vector<SequenceKVState*>& sequences,
                       PagedBatchMetadata& metadata, cudaStream_t stream = nullptr);
void storePagedKVBatch(PagedKVCache& cache, const PagedBatchMetadata& metadata, int layer,
                       __nv_bfloat16* q, __nv_bfloat16* k, const __nv_bfloat16* v,
                       cudaStream_t stream = nullptr);
void pagedDecodeAttention(const PagedKVCache& cache, PagedBatchMetadata& metadata, int layer,
                          const __nv_bfloat16* q, __nv_bfloat16* attention_output,
                          int mode = TVP_MODE_FAST, cudaStream_t stream = nullptr);
// Reads and clears the device error word (synchronises the stream).
int takePagedBatchError(PagedBatchMetadata& metadata, cudaStream_t stream = nullptr);

}  // namespace tvp
