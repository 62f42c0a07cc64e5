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
//            -> persistent device tables updated in place (only the entries
//               that changed, asynchronously) + one tvp_decode_plan per step
//            ropeBatch(q), ropeBatch(k), storePagedKVBatch, the paged gather,
//            32*B score GEMVs, 32*B softmax launches, the second gather and
//            32*B P.V GEMVs                        (paged_transformer.cu:80-94)
//            -> one tvp_rope_append + one tvp_paged_decode_attention per layer
// The layer loop around them calls the reference's functions in the
// reference's order, because its outputs (tokens) are what must not change.
//
// Modes (TVP_DECODE_MODE):
//   compat (default)  TVP_MODE_COMPAT decode (the reference's BF16 score and
//                     probability rounding) and the reference's own prefill
//                     attention: greedy-token identity with the unmodified
//                     engine.
//   fast              TVP_MODE_FAST decode, and tvp_paged_prefill_attention
//                     over the pages in place of the prefill attention
//                     (paged_transformer.cu:37-40).
//   batched           fast, plus the decode step's projections and LM head as
//                     one GEMM over the batch (n = B) instead of B one-row
//                     GEMMs (paged_transformer.cu:71-78,96-113,119-121), and
//                     the B greedy tokens from one tvp_greedy_argmax launch
//                     and one device-to-host copy instead of B argmaxLogits
//                     calls (argmax.cu:83-105).  The batched GEMMs sum in
//                     another order than the one-row ones, so this mode has
//                     its own parity policy (near-ties only, as fast).
//   native            batched, with every projection and the LM head on K5
//                     instead of cuBLAS: Q, K and V with RoPE and the page
//                     append in one launch (tvp_decode_qkv_rope_append); O
//                     with the residual add and the post-attention RMSNorm
//                     (tvp_decode_projection_residual_rmsnorm); gate and up
//                     with silu in their epilogue; down with the residual add,
//                     the next layer's RMSNorm and that layer's Q, K, V,
//                     RoPE and page append (tvp_decode_down_norm_qkv).  Four
//                     launches per layer with the attention.
//                     The same operands and FP32 accumulation in another
//                     summation order (the fused residual, silu, RoPE and
//                     RMSNorm keep the reference's rounding points bit for
//                     bit), so fast's parity policy again.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <initializer_list>
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

// The reference's residual and SwiGLU kernels (src/model/resConnection.cu:6-10,
// src/model/SiLU.cu:5-10), defined in its sources.  Their host wrappers
// launch on the legacy default stream, which a stream capture cannot record;
// the batched decode step launches the same kernels, with the wrappers'
// launch shape, on its own stream.
__global__ void residualKernel(__nv_bfloat16* input, __nv_bfloat16* input_embeds);
__global__ void siluKernel(__nv_bfloat16* a, __nv_bfloat16* b);

namespace {

constexpr int kLayers = 16;
constexpr int kQHeads = 32;
constexpr int kKvHeads = 8;
constexpr int kHidden = 2048;
constexpr int kMaxContext = 1024;                     // the engine's context cap
constexpr int kTableStride = kMaxContext / BLOCK_SIZE;  // 64, as MAX_BLOCKS_PER_SEQUENCE
constexpr int kMaxBatch = 4;                          // MAX_BATCH_SIZE of the scheduler
constexpr size_t kCublasWorkspace = 32u << 20;        // cuBLAS workspace of captured steps
constexpr int kNormScratchAt = 64;                     // ints: 256 B into the error buffer

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
  // Pinned mirror of `decode` as last uploaded: a step copies only the
  // entries that differ from it (the positions and lengths, and a table row
  // when it gained a page or its slot took a new request), asynchronously on
  // the stream the step runs on.
  int32_t* h_decode = nullptr;
  bool h_decode_valid = false;
  int32_t* error = nullptr;    // [error word | tokens (kMaxBatch)]: one read per step
  // native mode: scratch of the fused RMSNorm launches, inside the `error`
  // allocation at int kNormScratchAt, so that its error word (int 1 of it)
  // comes back with the step's one read
  void* norm_scratch = nullptr;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  void* argmax_workspace = nullptr;
  size_t argmax_workspace_bytes = 0;
  int mode = TVP_MODE_COMPAT;
  bool batched = false;
  bool native_proj = false;  // native mode: projections on tvp_decode_projections
  // Batched mode: the decode step runs on `stream` (a blocking stream, so it
  // is ordered after the engine's legacy-stream work) as a CUDA graph per
  // batch size, captured on the second step that uses the same buffers.
  cudaStream_t stream = nullptr;
  void* cublas_workspace = nullptr;
  int32_t* h_out = nullptr;  // pinned copy of [error word | tokens ... | norm scratch's first 2]
  struct StepGraph {
    std::vector<const void*> key;  // every buffer the captured launches point at
    bool warm = false;             // one eager step ran with `key`
    cudaGraphExec_t exec = nullptr;
  } graphs[kMaxBatch + 1];
  // Batched and native modes: the prefill of a prompt runs on `stream` too, as
  // a CUDA graph per prompt length (the last kPrefillGraphs lengths seen),
  // captured on the second prefill of that length on the same buffers.
  static constexpr int kPrefillGraphs = 8;
  struct PrefillGraph {
    int num_tokens = 0;
    StepGraph g;
  } prefill_graphs[kPrefillGraphs];
  int prefill_next = 0;
};

// Runs `enqueue(st.stream)` as the graph `g` keyed by `key`: replayed when it
// was recorded for `key`, recorded (and launched) on the second call with
// `key`, eager on the first, which also loads every kernel.
template <typename Enqueue>
void run_step_graph(PathState& st, PathState::StepGraph& g, const std::vector<const void*>& key,
                    cublasHandle_t cublas_handle, Enqueue&& enqueue) {
  if (g.exec && g.key == key) {
    check_cuda(cudaGraphLaunch(g.exec, st.stream));
  } else if (g.warm && g.key == key) {
    if (cublasSetWorkspace(cublas_handle, st.cublas_workspace, kCublasWorkspace) !=
        CUBLAS_STATUS_SUCCESS)
      throw std::runtime_error("cuBLAS workspace setup failed");
    check_cuda(cudaStreamBeginCapture(st.stream, cudaStreamCaptureModeThreadLocal));
    cudaGraph_t graph = nullptr;
    try {
      enqueue(st.stream);
    } catch (...) {
      cudaStreamEndCapture(st.stream, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    check_cuda(cudaStreamEndCapture(st.stream, &graph));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t made = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    check_cuda(made);
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g.exec = exec;
    check_cuda(cudaGraphLaunch(g.exec, st.stream));
  } else {
    if (g.exec) cudaGraphExecDestroy(g.exec);
    g.exec = nullptr;
    enqueue(st.stream);
    g.key = key;
    g.warm = true;
  }
}

// cuBLAS works on the path's stream while a batched call runs; the caller's
// stream (and with it cuBLAS's default workspace) is restored on return.
struct CublasOnStream {
  cublasHandle_t handle;
  cudaStream_t caller = nullptr;
  CublasOnStream(cublasHandle_t h, cudaStream_t stream) : handle(h) {
    if (cublasGetStream(handle, &caller) != CUBLAS_STATUS_SUCCESS ||
        cublasSetStream(handle, stream) != CUBLAS_STATUS_SUCCESS)
      throw std::runtime_error("cuBLAS stream setup failed");
  }
  ~CublasOnStream() { cublasSetStream(handle, caller); }
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
    check_cuda(cudaMallocHost(reinterpret_cast<void**>(&st.h_decode),
                              (kMaxBatch * kTableStride + 2 * kMaxBatch) * sizeof(int32_t)));
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&st.error),
                          kNormScratchAt * sizeof(int32_t) + TVP_NORM_SCRATCH_BYTES));
    check_cuda(cudaMemset(st.error, 0, kNormScratchAt * sizeof(int32_t) + TVP_NORM_SCRATCH_BYTES));
    st.norm_scratch = st.error + kNormScratchAt;
    st.argmax_workspace_bytes = tvp_greedy_argmax_workspace_bytes(kMaxBatch);
    check_cuda(cudaMalloc(&st.argmax_workspace, st.argmax_workspace_bytes));
    check_cuda(cudaMemset(st.argmax_workspace, 0, st.argmax_workspace_bytes));
    st.workspace_bytes = tvp_decode_workspace_bytes(kMaxBatch, kKvHeads, 0);
    if (st.workspace_bytes == 0) throw std::runtime_error("decode workspace size query failed");
    check_cuda(cudaMalloc(&st.workspace, st.workspace_bytes));
    const std::string mode = std::getenv("TVP_DECODE_MODE") ? std::getenv("TVP_DECODE_MODE") : "";
    st.native_proj = mode == "native";
    st.batched = mode == "batched" || st.native_proj;
    st.mode = (mode == "fast" || st.batched) ? TVP_MODE_FAST : TVP_MODE_COMPAT;
    if (st.batched) {
      check_cuda(cudaStreamCreate(&st.stream));
      check_cuda(cudaMalloc(&st.cublas_workspace, kCublasWorkspace));
      check_cuda(cudaMallocHost(reinterpret_cast<void**>(&st.h_out),
                                (kNormScratchAt + 2) * sizeof(int32_t)));
    }
    ready[dev] = true;
  }
  return st;
}

// Brings st.decode up to `want` with one cudaMemcpyAsync per run of changed
// entries inside a table row or the positions/lengths block, from the pinned
// mirror, on `stream` (ahead of the step's kernels there).  The mirror entries
// a copy reads are not rewritten before the copy ran: every step ends with a
// synchronisation with the device (the token read) before the next one starts.
void upload_decode_tables(PathState& st, const std::vector<int32_t>& want, cudaStream_t stream) {
  const int regions[kMaxBatch + 1][2] = {
      {0, kTableStride}, {kTableStride, 2 * kTableStride}, {2 * kTableStride, 3 * kTableStride},
      {3 * kTableStride, 4 * kTableStride}, {kMaxBatch * kTableStride,
                                             kMaxBatch * kTableStride + 2 * kMaxBatch}};
  static_assert(kMaxBatch == 4, "one region per table row plus positions/lengths");
  for (const auto& region : regions) {
    int i = region[0];
    while (i < region[1]) {
      if (st.h_decode_valid && st.h_decode[i] == want[i]) {
        ++i;
        continue;
      }
      int j = i;
      while (j < region[1] && !(st.h_decode_valid && st.h_decode[j] == want[j])) {
        st.h_decode[j] = want[j];
        ++j;
      }
      check_cuda(cudaMemcpyAsync(st.decode + i, st.h_decode + i, (j - i) * sizeof(int32_t),
                                 cudaMemcpyHostToDevice, stream));
      i = j;
    }
  }
  st.h_decode_valid = true;
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
  // The prefill's device work on `stream`; nullptr is the legacy default
  // stream, where the reference's own op wrappers are called.
  auto enqueue = [&](cudaStream_t stream) {
    auto norm = [&](__nv_bfloat16* gain) {
      rmsNormKernel<<<num_tokens, 1024, 0, stream>>>(hidden_states, buffers.rms_output, gain);
    };
    auto residual = [&](__nv_bfloat16* add) {
      if (stream) residualKernel<<<num_tokens, 1024, 0, stream>>>(hidden_states, add);
      else residualAdd(hidden_states, add, num_tokens);
    };
    for (int layer = 0; layer < kLayers; ++layer) {
      const LayerWeights& lw = weights.layers[layer];
      norm(lw.input_norm);
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
                                st.error, stream));
      if (st.mode == TVP_MODE_FAST) {
        // Causal attention over the pages just written (no score matrix).
        check_tvp(tvp_paged_prefill_attention(
            reinterpret_cast<const tvp_bf16*>(buffers.q),
            reinterpret_cast<const tvp_bf16*>(cache.k_blocks),
            reinterpret_cast<const tvp_bf16*>(cache.v_blocks), cache.num_blocks, kLayers, layer,
            kKvHeads, kQHeads, d_table, pages, d_cu_q, d_pos0, 1, num_tokens, 0.125f,
            reinterpret_cast<tvp_bf16*>(buffers.attn_output), st.error, stream));
      } else {
        // COMPAT keeps the reference's own prefill attention (token identity);
        // it only runs on the legacy stream.
        computeAttentionScores(cublas_handle, buffers.q, buffers.k, buffers.attn_scores, num_tokens);
        causalMask(buffers.attn_scores, num_tokens);
        softmaxRows(buffers.attn_scores, kQHeads * num_tokens, num_tokens);
        attentionScoresTimesV(cublas_handle, buffers.attn_scores, buffers.v, buffers.attn_output,
                              num_tokens);
      }
      outputProjection(cublas_handle, buffers.attn_output, lw.w_o, buffers.o_output, num_tokens);
      residual(buffers.o_output);
      norm(lw.post_attention_norm);
      gateProjection(cublas_handle, buffers.rms_output, lw.w_gate, buffers.gate, num_tokens);
      upProjection(cublas_handle, buffers.rms_output, lw.w_up, buffers.up, num_tokens);
      if (stream) siluKernel<<<num_tokens, 1024, 0, stream>>>(buffers.gate, buffers.up);
      else silu(buffers.gate, buffers.up, num_tokens);
      downProjection(cublas_handle, buffers.gate, lw.w_down, buffers.down, num_tokens);
      residual(buffers.down);
    }
    norm(weights.final_norm);
    lmHeadProjection(cublas_handle, buffers.rms_output + (num_tokens - 1) * kHidden,
                     weights.embedding, logits);
  };
  if (!st.batched) {
    enqueue(nullptr);
  } else {
    // On the path's blocking stream, so ordered after the engine's
    // legacy-stream work (the embedding gather) and before its argmax below.
    CublasOnStream on_stream(cublas_handle, st.stream);
    PathState::PrefillGraph* slot = nullptr;
    for (auto& e : st.prefill_graphs)
      if (e.num_tokens == num_tokens) slot = &e;
    if (!slot) {
      slot = &st.prefill_graphs[st.prefill_next];
      st.prefill_next = (st.prefill_next + 1) % PathState::kPrefillGraphs;
      if (slot->g.exec) cudaGraphExecDestroy(slot->g.exec);
      *slot = PathState::PrefillGraph{};
      slot->num_tokens = num_tokens;
    }
    const std::vector<const void*> key = {
        hidden_states, buffers.rms_output, buffers.q, buffers.k, buffers.v, buffers.attn_output,
        buffers.o_output, buffers.gate, buffers.up, buffers.down, logits, cache.k_blocks,
        cache.v_blocks, reinterpret_cast<const void*>(static_cast<intptr_t>(cache.num_blocks)),
        reinterpret_cast<const void*>(static_cast<intptr_t>(pages)), weights.embedding,
        weights.final_norm, weights.layers[0].w_q, cublas_handle};
    if (cublasSetWorkspace(cublas_handle, st.cublas_workspace, kCublasWorkspace) !=
        CUBLAS_STATUS_SUCCESS)
      throw std::runtime_error("cuBLAS workspace setup failed");
    run_step_graph(st, slot->g, key, cublas_handle, enqueue);
  }
  check_cuda(cudaGetLastError());
  sequence.current_seq_len += num_tokens;
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
  // Only what changed since the last step, asynchronously on the step's
  // stream: the legacy default stream (compat, fast) or the batched step's
  // stream, where the graph launch follows it.
  upload_decode_tables(st, staging, st.batched ? st.stream : nullptr);
  const int32_t* d_tables = st.decode;
  const int32_t* d_pos = st.decode + kMaxBatch * kTableStride;
  const int32_t* d_len = d_pos + kMaxBatch;
  // A projection of the step: one GEMM over the batch (batched mode) or the
  // reference's row-stable one-row GEMMs (its BF16 rounding contract).
  auto project = [&](auto projection, auto* in, int in_dim, auto* w, __nv_bfloat16* out,
                     int out_dim) {
    if (st.batched) {
      projection(cublas_handle, in, w, out, batch);
      return;
    }
    for (int row = 0; row < batch; ++row)
      projection(cublas_handle, in + row * in_dim, w, out + row * out_dim, 1);
  };
  // Native mode: up to three projections of the same rows in one launch.
  auto native = [&](const __nv_bfloat16* in, int in_dim,
                    std::initializer_list<const __nv_bfloat16*> ws, std::initializer_list<int> ns,
                    std::initializer_list<__nv_bfloat16*> outs, int epilogue) {
    const tvp_bf16* w[TVP_PROJ_MAX];
    int n[TVP_PROJ_MAX];
    void* out[TVP_PROJ_MAX] = {};
    int count = 0;
    for (auto* p : ws) w[count++] = reinterpret_cast<const tvp_bf16*>(p);
    count = 0;
    for (int v : ns) n[count++] = v;
    int stored = 0;
    for (auto* p : outs) out[stored++] = p;
    check_tvp(tvp_decode_projections(reinterpret_cast<const tvp_bf16*>(in), batch, in_dim, count,
                                     w, n, out, epilogue, st.stream));
  };
  // The step's device work on `stream`; nullptr is the legacy default stream,
  // where the reference's own op wrappers are called.
  auto enqueue = [&](cudaStream_t stream) {
    auto residual = [&](__nv_bfloat16* add) {
      if (stream) residualKernel<<<batch, 1024, 0, stream>>>(hidden_states, add);
      else residualAdd(hidden_states, add, batch);
    };
    check_tvp(tvp_decode_plan(d_len, batch, kTableStride, kKvHeads, 0, st.workspace,
                              st.workspace_bytes, st.error, stream));
    bool qkv_done = false;  // native: this layer's Q/K/V ran in the previous layer's down launch
    for (int layer = 0; layer < kLayers; ++layer) {
      const LayerWeights& lw = weights.layers[layer];
      // native: every RMSNorm but the first runs in the residual projection
      // before it (tvp_decode_projection_residual_rmsnorm)
      if (!st.native_proj || layer == 0)
        rmsNormKernel<<<batch, 1024, 0, stream>>>(hidden_states, buffers.rms_output, lw.input_norm);
      if (st.native_proj && qkv_done) {
        qkv_done = false;
      } else if (st.native_proj) {
        // Q, K, V, RoPE and the page append in one launch
        check_tvp(tvp_decode_qkv_rope_append(
            reinterpret_cast<const tvp_bf16*>(buffers.rms_output), batch, kHidden,
            reinterpret_cast<const tvp_bf16*>(lw.w_q), reinterpret_cast<const tvp_bf16*>(lw.w_k),
            reinterpret_cast<const tvp_bf16*>(lw.w_v), reinterpret_cast<tvp_bf16*>(buffers.q),
            reinterpret_cast<tvp_bf16*>(cache.k_blocks), reinterpret_cast<tvp_bf16*>(cache.v_blocks),
            cache.num_blocks, kLayers, layer, d_tables, kTableStride, d_pos, st.error, stream));
      } else {
        project(qProjection, buffers.rms_output, kHidden, lw.w_q, buffers.q, kHidden);
        project(kProjection, buffers.rms_output, kHidden, lw.w_k, buffers.k, 512);
        project(vProjection, buffers.rms_output, kHidden, lw.w_v, buffers.v, 512);
        check_tvp(tvp_rope_append(reinterpret_cast<tvp_bf16*>(cache.k_blocks),
                                  reinterpret_cast<tvp_bf16*>(cache.v_blocks), cache.num_blocks,
                                  kLayers, layer, kKvHeads, d_tables, kTableStride, batch, nullptr,
                                  d_pos, batch, reinterpret_cast<tvp_bf16*>(buffers.k),
                                  reinterpret_cast<const tvp_bf16*>(buffers.v),
                                  reinterpret_cast<tvp_bf16*>(buffers.q), kQHeads,
                                  TVP_APPEND_ROPE_K | TVP_APPEND_ROPE_Q | TVP_APPEND_WRITEBACK_K,
                                  st.error, stream));
      }
      check_tvp(tvp_paged_decode_attention(
          reinterpret_cast<const tvp_bf16*>(buffers.q),
          reinterpret_cast<const tvp_bf16*>(cache.k_blocks),
          reinterpret_cast<const tvp_bf16*>(cache.v_blocks), cache.num_blocks, kLayers, layer,
          kKvHeads, kQHeads, d_tables, kTableStride, d_len, batch, 0.125f, st.mode, 0,
          st.workspace, st.workspace_bytes, reinterpret_cast<tvp_bf16*>(buffers.attn_output),
          st.error, stream));
      // native: hidden += O attn, then its post-attention RMSNorm, one launch
      auto residual_norm = [&](const __nv_bfloat16* in, int in_dim, const __nv_bfloat16* w,
                               const __nv_bfloat16* gain) {
        check_tvp(tvp_decode_projection_residual_rmsnorm(
            reinterpret_cast<const tvp_bf16*>(in), batch, in_dim,
            reinterpret_cast<const tvp_bf16*>(w), reinterpret_cast<tvp_bf16*>(hidden_states),
            reinterpret_cast<const tvp_bf16*>(gain), reinterpret_cast<tvp_bf16*>(buffers.rms_output),
            st.norm_scratch, stream));
      };
      if (st.native_proj) {
        residual_norm(buffers.attn_output, kHidden, lw.w_o, lw.post_attention_norm);
      } else {
        project(outputProjection, buffers.attn_output, kHidden, lw.w_o, buffers.o_output, kHidden);
        residual(buffers.o_output);
        rmsNormKernel<<<batch, 1024, 0, stream>>>(hidden_states, buffers.rms_output,
                                                  lw.post_attention_norm);
      }
      if (st.native_proj) {  // gate = silu(gate x) * (up x), one launch
        native(buffers.rms_output, kHidden, {lw.w_gate, lw.w_up}, {8192, 8192}, {buffers.gate},
               TVP_PROJ_SWIGLU);
      } else {
        project(gateProjection, buffers.rms_output, kHidden, lw.w_gate, buffers.gate, 8192);
        project(upProjection, buffers.rms_output, kHidden, lw.w_up, buffers.up, 8192);
        if (stream) siluKernel<<<batch, 1024, 0, stream>>>(buffers.gate, buffers.up);
        else silu(buffers.gate, buffers.up, batch);
      }
      if (st.native_proj) {  // hidden += down, then the next RMSNorm (the final one last)
        // with the next layer's Q, K, V, RoPE and page append in the same launch
        if (layer + 1 < kLayers) {
          const LayerWeights& nw = weights.layers[layer + 1];
          const int rc = tvp_decode_down_norm_qkv(
              reinterpret_cast<const tvp_bf16*>(buffers.gate), batch, 8192,
              reinterpret_cast<const tvp_bf16*>(lw.w_down), reinterpret_cast<tvp_bf16*>(hidden_states),
              reinterpret_cast<const tvp_bf16*>(nw.input_norm),
              reinterpret_cast<tvp_bf16*>(buffers.rms_output), st.norm_scratch,
              reinterpret_cast<const tvp_bf16*>(nw.w_q), reinterpret_cast<const tvp_bf16*>(nw.w_k),
              reinterpret_cast<const tvp_bf16*>(nw.w_v), reinterpret_cast<tvp_bf16*>(buffers.q),
              reinterpret_cast<tvp_bf16*>(cache.k_blocks),
              reinterpret_cast<tvp_bf16*>(cache.v_blocks), cache.num_blocks, kLayers, layer + 1,
              d_tables, kTableStride, d_pos, st.error, stream);
          if (rc != TVP_ERR_UNSUPPORTED) {
            check_tvp(rc);
            qkv_done = true;
            continue;
          }
        }
        residual_norm(buffers.gate, 8192, lw.w_down,
                      layer + 1 < kLayers ? weights.layers[layer + 1].input_norm : weights.final_norm);
      } else {
        project(downProjection, buffers.gate, 8192, lw.w_down, buffers.down, kHidden);
        residual(buffers.down);
      }
    }
    if (!st.native_proj)
      rmsNormKernel<<<batch, 1024, 0, stream>>>(hidden_states, buffers.rms_output, weights.final_norm);
    if (!st.batched) return;
    // The LM head of lm_head.cu:8-36 over all rows: logits[row] = E h_row.
    const float alpha = 1.0f, beta = 0.0f;
    if (st.native_proj) {
      const tvp_bf16* w = reinterpret_cast<const tvp_bf16*>(weights.embedding);
      const int n = VOCAB_SIZE;
      void* out = logits;
      check_tvp(tvp_decode_projections(reinterpret_cast<const tvp_bf16*>(buffers.rms_output),
                                       batch, kHidden, 1, &w, &n, &out, TVP_PROJ_F32, stream));
    } else if (cublasGemmEx(cublas_handle, CUBLAS_OP_T, CUBLAS_OP_N, VOCAB_SIZE, batch, kHidden, &alpha,
                     weights.embedding, CUDA_R_16BF, kHidden, buffers.rms_output, CUDA_R_16BF,
                     kHidden, &beta, logits, CUDA_R_32F, VOCAB_SIZE, CUBLAS_COMPUTE_32F,
                     CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
      throw std::runtime_error("LM head projection failed");
    check_tvp(tvp_greedy_argmax(logits, batch, VOCAB_SIZE, VOCAB_SIZE, st.error + 1,
                                st.argmax_workspace, st.argmax_workspace_bytes, stream));
  };

  std::vector<int> tokens;
  tokens.reserve(batch);
  if (!st.batched) {
    enqueue(nullptr);
    for (int row = 0; row < batch; ++row)
      lmHeadProjection(cublas_handle, buffers.rms_output + row * kHidden, weights.embedding,
                       logits + static_cast<size_t>(row) * VOCAB_SIZE);
    check_cuda(cudaGetLastError());
    for (int row = 0; row < batch; ++row)
      tokens.push_back(argmaxLogits(logits + static_cast<size_t>(row) * VOCAB_SIZE));
    raise_device_errors(st);
  } else {
    CublasOnStream on_stream(cublas_handle, st.stream);
    PathState::StepGraph& g = st.graphs[batch];
    const std::vector<const void*> key = {
        hidden_states, buffers.rms_output, buffers.q, buffers.k, buffers.v, buffers.attn_output,
        buffers.o_output, buffers.gate, buffers.up, buffers.down, logits, cache.k_blocks,
        cache.v_blocks, reinterpret_cast<const void*>(static_cast<intptr_t>(cache.num_blocks)),
        weights.embedding, weights.final_norm, weights.layers[0].w_q, cublas_handle};
    run_step_graph(st, g, key, cublas_handle, enqueue);
    check_cuda(cudaMemcpyAsync(st.h_out, st.error, (kNormScratchAt + 2) * sizeof(int32_t),
                               cudaMemcpyDeviceToHost, st.stream));
    check_cuda(cudaStreamSynchronize(st.stream));
    if (st.h_out[0] || st.h_out[kNormScratchAt + 1]) {
      const int32_t bits = st.h_out[0] | st.h_out[kNormScratchAt + 1];
      check_cuda(cudaMemset(st.error, 0, sizeof(int32_t)));
      check_cuda(cudaMemset(st.error + kNormScratchAt + 1, 0, sizeof(int32_t)));
      throw std::runtime_error("paged-KV kernels reported device error bits " +
                               std::to_string(bits));
    }
    tokens.assign(st.h_out + 1, st.h_out + 1 + batch);
  }
  for (auto* sequence : sequences) sequence->current_seq_len += 1;
  return tokens;
}

int decodeForwardPaged(cublasHandle_t cublas_handle, __nv_bfloat16* hidden_states,
                       const ModelWeights& weights, PagedKVCache& cache, SequenceKVState& sequence,
                       TransformerBuffers& buffers, float* logits) {
  return decodeBatchPaged(cublas_handle, hidden_states, weights, cache, {&sequence}, buffers,
                          logits)[0];
}
