// Drop-in replacement for the reference engine's src/model/paged_transformer.cu.
//
// Compiled against the reference's headers (include/paged_transformer.cuh and
// the op headers it names) and linked with the reference's other sources in
// place of its paged_transformer.cu, it keeps every reference op around the
// paged-KV path (RMSNorm, the one-row cuBLAS projections, the contiguous
// prefill attention, MLP, LM head, argmax, the page allocator) and replaces
// only the path itself with the C-ABI of include/tvp_paged.h:
//   prefill  rope(q), rope(k), storePagedKV        (paged_transformer.cu:34-36)
//            -> one tvp_rope_append
//   decode   preparePagedBatch's per-step mallocs  (paged_transformer.cu:65,135)
//            -> persistent device tables + one tvp_decode_plan per step
//            ropeBatch(q), ropeBatch(k), storePagedKVBatch, the paged gather,
//            32*B score GEMVs, 32*B softmax launches, the second gather and
//            32*B P.V GEMVs                        (paged_transformer.cu:80-94)
//            -> one tvp_rope_append + one tvp_paged_decode_attention per layer
// The layer loop around them calls the reference's functions in the
// reference's order, because its outputs (tokens) are what must not change.
//
// Decode numerics: TVP_DECODE_MODE=fast selects TVP_MODE_FAST, which also
// swaps the prefill attention (paged_transformer.cu:37-40) for
// tvp_paged_prefill_attention over the pages; the default is TVP_MODE_COMPAT
// (the reference's BF16 score/probability rounding, and its own prefill
// attention), which is what greedy-token identity with the unmodified engine
// needs.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "argmax.cuh"
#include "attention.cuh"
#include "causalMask.cuh"
#include "lm_head.cuh"
#include "mlp.cuh"
#include "paged_transformer.cuh"
#include "residual.cuh"
#include "rmsnorm.cuh"
#include "silu.cuh"
#include "softmax.cuh"
#include "tvp_paged.h"

namespace {

constexpr int kLayers = 16;
constexpr int kQHeads = 32;
constexpr int kKvHeads = 8;
constexpr int kHidden = 2048;
constexpr int kMaxContext = 1024;                     // the engine's context cap
constexpr int kTableStride = kMaxContext / BLOCK_SIZE;  // 64, as MAX_BLOCKS_PER_SEQUENCE
constexpr int kMaxBatch = 4;                          // MAX_BATCH_SIZE of the scheduler

void check_cuda(cudaError_t status) {
  if (status != cudaSuccess) throw std::runtime_error(cudaGetErrorString(status));
}

void check_tvp(int rc) {
  if (rc == TVP_OK) return;
  if (rc == TVP_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tvp_strerror(rc));
  throw std::runtime_error(tvp_strerror(rc));
}

// Device buffers that live for the process (one set per device in use).
struct PathState {
  int32_t* prefill = nullptr;  // [table (64) | positions (1024) | rows (1024) | cu_q (2) | pos0 (1)]
  int32_t* decode = nullptr;   // [tables (4 x 64) | positions (4) | lengths (4)]
  int32_t* error = nullptr;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  int mode = TVP_MODE_COMPAT;
};

PathState& path_state() {
  static std::mutex mutex;
  static PathState states[64];
  static bool ready[64] = {};
  int dev = 0;
  check_cuda(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw std::runtime_error("device index out of range");
  std::lock_guard<std::mutex> lock(mutex);
  PathState& st = states[dev];
  if (!ready[dev]) {
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&st.prefill),
                          (kTableStride + 2 * kMaxContext + 4) * sizeof(int32_t)));
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&st.decode),
                          (kMaxBatch * kTableStride + 2 * kMaxBatch) * sizeof(int32_t)));
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&st.error), sizeof(int32_t)));
    check_cuda(cudaMemset(st.error, 0, sizeof(int32_t)));
    st.workspace_bytes = tvp_decode_workspace_bytes(kMaxBatch, kKvHeads, 0);
    if (st.workspace_bytes == 0) throw std::runtime_error("decode workspace size query failed");
    check_cuda(cudaMalloc(&st.workspace, st.workspace_bytes));
    const char* mode = std::getenv("TVP_DECODE_MODE");
    st.mode = (mode && std::string(mode) == "fast") ? TVP_MODE_FAST : TVP_MODE_COMPAT;
    ready[dev] = true;
  }
  return st;
}

void raise_device_errors(PathState& st) {
  int32_t bits = 0;
  check_cuda(cudaMemcpy(&bits, st.error, sizeof(bits), cudaMemcpyDeviceToHost));
  if (bits) {
    check_cuda(cudaMemset(st.error, 0, sizeof(int32_t)));
    throw std::runtime_error("paged-KV kernels reported device error bits " + std::to_string(bits));
  }
}

}  // namespace

int transformerForwardPaged(cublasHandle_t cublas_handle, __nv_bfloat16* hidden_states,
                            const ModelWeights& weights, PagedKVCache& cache,
                            SequenceKVState& sequence, TransformerBuffers& buffers, float* logits,
                            int num_tokens) {
  if (sequence.current_seq_len != 0 || num_tokens <= 0 || num_tokens > kMaxContext)
    throw std::invalid_argument("Paged prefill requires an empty sequence and 1..1024 tokens");
  reserveSequenceBlocks(cache, sequence, num_tokens);
  PathState& st = path_state();
  const int pages = static_cast<int>(sequence.block_table.size());
  std::vector<int32_t> staging(kTableStride + 2 * num_tokens + 3, 0);
  std::copy(sequence.block_table.begin(), sequence.block_table.end(), staging.begin());
  for (int t = 0; t < num_tokens; ++t) staging[kTableStride + t] = t;
  staging[kTableStride + 2 * num_tokens + 1] = num_tokens;  // cu_q = {0, n}, pos0 = {0}
  check_cuda(cudaMemcpy(st.prefill, staging.data(), staging.size() * sizeof(int32_t),
                        cudaMemcpyHostToDevice));
  const int32_t* d_table = st.prefill;
  const int32_t* d_pos = st.prefill + kTableStride;
  const int32_t* d_rows = st.prefill + kTableStride + num_tokens;
  const int32_t* d_cu_q = st.prefill + kTableStride + 2 * num_tokens;
  const int32_t* d_pos0 = d_cu_q + 2;
  for (int layer = 0; layer < kLayers; ++layer) {
    const LayerWeights& lw = weights.layers[layer];
    rmsNormKernel<<<num_tokens, 1024>>>(hidden_states, buffers.rms_output, lw.input_norm);
    qProjection(cublas_handle, buffers.rms_output, lw.w_q, buffers.q, num_tokens);
    kProjection(cublas_handle, buffers.rms_output, lw.w_k, buffers.k, num_tokens);
    vProjection(cublas_handle, buffers.rms_output, lw.w_v, buffers.v, num_tokens);
    // RoPE(q), RoPE(k) in place and the page append, in one launch.
    check_tvp(tvp_rope_append(reinterpret_cast<tvp_bf16*>(cache.k_blocks),
                              reinterpret_cast<tvp_bf16*>(cache.v_blocks), cache.num_blocks,
                              kLayers, layer, kKvHeads, d_table, pages, 1, d_rows, d_pos,
                              num_tokens, reinterpret_cast<tvp_bf16*>(buffers.k),
                              reinterpret_cast<const tvp_bf16*>(buffers.v),
                              reinterpret_cast<tvp_bf16*>(buffers.q), kQHeads,
                              TVP_APPEND_ROPE_K | TVP_APPEND_ROPE_Q | TVP_APPEND_WRITEBACK_K,
                              st.error, nullptr));
    if (st.mode == TVP_MODE_FAST) {
      // Causal attention over the pages just written (no score matrix).
      check_tvp(tvp_paged_prefill_attention(
          reinterpret_cast<const tvp_bf16*>(buffers.q),
          reinterpret_cast<const tvp_bf16*>(cache.k_blocks),
          reinterpret_cast<const tvp_bf16*>(cache.v_blocks), cache.num_blocks, kLayers, layer,
          kKvHeads, kQHeads, d_table, pages, d_cu_q, d_pos0, 1, num_tokens, 0.125f,
          reinterpret_cast<tvp_bf16*>(buffers.attn_output), st.error, nullptr));
    } else {
      // COMPAT keeps the reference's own prefill attention (token identity).
      computeAttentionScores(cublas_handle, buffers.q, buffers.k, buffers.attn_scores, num_tokens);
      causalMask(buffers.attn_scores, num_tokens);
      softmaxRows(buffers.attn_scores, kQHeads * num_tokens, num_tokens);
      attentionScoresTimesV(cublas_handle, buffers.attn_scores, buffers.v, buffers.attn_output,
                            num_tokens);
    }
    outputProjection(cublas_handle, buffers.attn_output, lw.w_o, buffers.o_output, num_tokens);
    residualAdd(hidden_states, buffers.o_output, num_tokens);
    rmsNormKernel<<<num_tokens, 1024>>>(hidden_states, buffers.rms_output, lw.post_attention_norm);
    gateProjection(cublas_handle, buffers.rms_output, lw.w_gate, buffers.gate, num_tokens);
    upProjection(cublas_handle, buffers.rms_output, lw.w_up, buffers.up, num_tokens);
    silu(buffers.gate, buffers.up, num_tokens);
    downProjection(cublas_handle, buffers.gate, lw.w_down, buffers.down, num_tokens);
    residualAdd(hidden_states, buffers.down, num_tokens);
  }
  sequence.current_seq_len += num_tokens;
  rmsNormKernel<<<num_tokens, 1024>>>(hidden_states, buffers.rms_output, weights.final_norm);
  lmHeadProjection(cublas_handle, buffers.rms_output + (num_tokens - 1) * kHidden,
                   weights.embedding, logits);
  const int token = argmaxLogits(logits);
  raise_device_errors(st);
  return token;
}

std::vector<int> decodeBatchPaged(cublasHandle_t cublas_handle, __nv_bfloat16* hidden_states,
                                  const ModelWeights& weights, PagedKVCache& cache,
                                  const std::vector<SequenceKVState*>& sequences,
                                  TransformerBuffers& buffers, float* logits) {
  // Validation and page reservation with the semantics of preparePagedBatch
  // (src/model/paged_attention.cu:30-65), into persistent device tables.
  if (!cache.k_blocks || !cache.v_blocks || cache.num_blocks <= 0 || cache.block_size != BLOCK_SIZE ||
      sequences.empty() || sequences.size() > static_cast<size_t>(kMaxBatch))
    throw std::invalid_argument("Invalid paged decode batch");
  size_t needed = 0;
  std::vector<int> owners(cache.num_blocks, -1);
  for (size_t row = 0; row < sequences.size(); ++row) {
    const SequenceKVState* sequence = sequences[row];
    if (!sequence || sequence->current_seq_len < 1 || sequence->current_seq_len >= kMaxContext)
      throw std::invalid_argument("Paged decode requires 1..1023 cached tokens");
    for (int block : sequence->block_table) {
      if (block < 0 || block >= cache.num_blocks || owners[block] != -1)
        throw std::invalid_argument("Paged decode sequences must own distinct blocks");
      owners[block] = static_cast<int>(row);
    }
    const size_t required = (sequence->current_seq_len + BLOCK_SIZE) / BLOCK_SIZE;
    if (required > sequence->block_table.size()) needed += required - sequence->block_table.size();
  }
  if (needed > cache.free_blocks.size()) throw std::runtime_error("Insufficient blocks for decode batch");
  const int batch = static_cast<int>(sequences.size());
  std::vector<int32_t> staging(kMaxBatch * kTableStride + 2 * kMaxBatch, -1);
  for (int row = 0; row < batch; ++row) {
    SequenceKVState& sequence = *sequences[row];
    reserveSequenceBlocks(cache, sequence, sequence.current_seq_len + 1);
    if (sequence.block_table.size() > static_cast<size_t>(kTableStride))
      throw std::invalid_argument("Paged block table exceeds context limit");
    std::copy(sequence.block_table.begin(), sequence.block_table.end(),
              staging.begin() + row * kTableStride);
    staging[kMaxBatch * kTableStride + row] = sequence.current_seq_len;
    staging[kMaxBatch * kTableStride + kMaxBatch + row] = sequence.current_seq_len + 1;
  }
  PathState& st = path_state();
  check_cuda(cudaMemcpy(st.decode, staging.data(), staging.size() * sizeof(int32_t),
                        cudaMemcpyHostToDevice));
  const int32_t* d_tables = st.decode;
  const int32_t* d_pos = st.decode + kMaxBatch * kTableStride;
  const int32_t* d_len = d_pos + kMaxBatch;
  check_tvp(tvp_decode_plan(d_len, batch, kTableStride, kKvHeads, 0, st.workspace,
                            st.workspace_bytes, st.error, nullptr));
  for (int layer = 0; layer < kLayers; ++layer) {
    const LayerWeights& lw = weights.layers[layer];
    rmsNormKernel<<<batch, 1024>>>(hidden_states, buffers.rms_output, lw.input_norm);
    // Row-stable one-row GEMMs, exactly as the reference (its BF16 rounding contract).
    for (int row = 0; row < batch; ++row)
      qProjection(cublas_handle, buffers.rms_output + row * kHidden, lw.w_q, buffers.q + row * kHidden, 1);
    for (int row = 0; row < batch; ++row)
      kProjection(cublas_handle, buffers.rms_output + row * kHidden, lw.w_k, buffers.k + row * 512, 1);
    for (int row = 0; row < batch; ++row)
      vProjection(cublas_handle, buffers.rms_output + row * kHidden, lw.w_v, buffers.v + row * 512, 1);
    check_tvp(tvp_rope_append(reinterpret_cast<tvp_bf16*>(cache.k_blocks),
                              reinterpret_cast<tvp_bf16*>(cache.v_blocks), cache.num_blocks,
                              kLayers, layer, kKvHeads, d_tables, kTableStride, batch, nullptr,
                              d_pos, batch, reinterpret_cast<tvp_bf16*>(buffers.k),
                              reinterpret_cast<const tvp_bf16*>(buffers.v),
                              reinterpret_cast<tvp_bf16*>(buffers.q), kQHeads,
                              TVP_APPEND_ROPE_K | TVP_APPEND_ROPE_Q | TVP_APPEND_WRITEBACK_K,
                              st.error, nullptr));
    check_tvp(tvp_paged_decode_attention(
        reinterpret_cast<const tvp_bf16*>(buffers.q), reinterpret_cast<const tvp_bf16*>(cache.k_blocks),
        reinterpret_cast<const tvp_bf16*>(cache.v_blocks), cache.num_blocks, kLayers, layer, kKvHeads,
        kQHeads, d_tables, kTableStride, d_len, batch, 0.125f, st.mode, 0, st.workspace,
        st.workspace_bytes, reinterpret_cast<tvp_bf16*>(buffers.attn_output), st.error, nullptr));
    for (int row = 0; row < batch; ++row)
      outputProjection(cublas_handle, buffers.attn_output + row * kHidden, lw.w_o,
                       buffers.o_output + row * kHidden, 1);
    residualAdd(hidden_states, buffers.o_output, batch);
    rmsNormKernel<<<batch, 1024>>>(hidden_states, buffers.rms_output, lw.post_attention_norm);
    for (int row = 0; row < batch; ++row)
      gateProjection(cublas_handle, buffers.rms_output + row * kHidden, lw.w_gate, buffers.gate + row * 8192, 1);
    for (int row = 0; row < batch; ++row)
      upProjection(cublas_handle, buffers.rms_output + row * kHidden, lw.w_up, buffers.up + row * 8192, 1);
    silu(buffers.gate, buffers.up, batch);
    for (int row = 0; row < batch; ++row)
      downProjection(cublas_handle, buffers.gate + row * 8192, lw.w_down, buffers.down + row * kHidden, 1);
    residualAdd(hidden_states, buffers.down, batch);
  }
  rmsNormKernel<<<batch, 1024>>>(hidden_states, buffers.rms_output, weights.final_norm);
  for (int row = 0; row < batch; ++row)
    lmHeadProjection(cublas_handle, buffers.rms_output + row * kHidden, weights.embedding,
                     logits + static_cast<size_t>(row) * VOCAB_SIZE);
  check_cuda(cudaGetLastError());
  std::vector<int> tokens;
  tokens.reserve(batch);
  for (int row = 0; row < batch; ++row)
    tokens.push_back(argmaxLogits(logits + static_cast<size_t>(row) * VOCAB_SIZE));
  raise_device_errors(st);
  for (auto* sequence : sequences) sequence->current_seq_len += 1;
  return tokens;
}

int decodeForwardPaged(cublasHandle_t cublas_handle, __nv_bfloat16* hidden_states,
                       const ModelWeights& weights, PagedKVCache& cache, SequenceKVState& sequence,
                       TransformerBuffers& buffers, float* logits) {
  return decodeBatchPaged(cublas_handle, hidden_states, weights, cache, {&sequence}, buffers,
                          logits)[0];
}
