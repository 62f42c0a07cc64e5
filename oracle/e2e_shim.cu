// e2e_shim.cu — TEST INFRASTRUCTURE ONLY (the checker, never the product).
//
// End-to-end driver for the e2e workload (Llama-3.2-1B geometry, random
// weights): builds seeded N(0, 0.02) BF16 weights in the reference's
// ModelWeights layout (HF tensor shapes, as mapWeights in src/main.cu:172-208
// maps them; RMSNorm gains 1.0, LM head tied to the embedding), then runs the
// reference's own continuous-batching scheduler, generateContinuous
// (src/engine/scheduler.cu:17-169), on caller-given prompts.
//
// oracle/Makefile links it twice with the reference sources: once with the
// reference's src/model/paged_transformer.cu (the unmodified engine) and once
// with vllm_b200/csrc/integration/paged_transformer_tvp.cu (the engine with
// the B200 paged-KV path dropped in), so the two can be compared token by token.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <exception>
#include <stdexcept>
#include <vector>

#include "argmax.cuh"
#include "embedding.cuh"
#include "rmsnorm.cuh"
#include "paged_transformer.cuh"
#include "request.cuh"
#include "scheduler.cuh"
#include "weights.cuh"

namespace {

// Counter-based N(mean, stddev) BF16 fill: splitmix64 of (seed, index) gives
// two uniforms, Box-Muller turns them into one normal draw.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

__global__ void fill_normal(__nv_bfloat16* p, size_t n, uint64_t seed, float stddev) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const uint64_t r = mix64(seed * 0x100000001b3ull + i);
    const float u1 = ((uint32_t)(r >> 40) + 1.0f) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (uint32_t)(r & 0xffffff) * (1.0f / 16777216.0f);        // [0, 1)
    const float z = sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
    p[i] = __float2bfloat16_rn(stddev * z);
  }
}

__global__ void fill_value(__nv_bfloat16* p, size_t n, float v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = __float2bfloat16_rn(v);
}

struct Model {
  ModelWeights weights;
  std::vector<void*> allocations;
  cublasHandle_t handle = nullptr;
};

Model* g_model = nullptr;

__nv_bfloat16* tensor(Model& m, size_t n, uint64_t seed, bool norm_gain) {
  void* p = nullptr;
  if (cudaMalloc(&p, n * sizeof(__nv_bfloat16)) != cudaSuccess)
    throw std::runtime_error("cudaMalloc weights");
  m.allocations.push_back(p);
  auto* t = static_cast<__nv_bfloat16*>(p);
  if (norm_gain)
    fill_value<<<1024, 256>>>(t, n, 1.0f);
  else
    fill_normal<<<4096, 256>>>(t, n, seed, 0.02f);
  return t;
}

}  // namespace

extern "C" {

int e2e_init(unsigned long long seed) {
  try {
    if (g_model) return 0;
    Model* m = new Model();
    uint64_t s = seed * 1000;
    m->weights.embedding = tensor(*m, (size_t)VOCAB_SIZE * 2048, ++s, false);
    for (int layer = 0; layer < 16; ++layer) {
      LayerWeights lw;
      lw.input_norm = tensor(*m, 2048, ++s, true);
      lw.w_q = tensor(*m, (size_t)2048 * 2048, ++s, false);
      lw.w_k = tensor(*m, (size_t)512 * 2048, ++s, false);
      lw.w_v = tensor(*m, (size_t)512 * 2048, ++s, false);
      lw.w_o = tensor(*m, (size_t)2048 * 2048, ++s, false);
      lw.w_gate = tensor(*m, (size_t)8192 * 2048, ++s, false);
      lw.w_up = tensor(*m, (size_t)8192 * 2048, ++s, false);
      lw.w_down = tensor(*m, (size_t)2048 * 8192, ++s, false);
      lw.post_attention_norm = tensor(*m, 2048, ++s, true);
      m->weights.layers.push_back(lw);
    }
    m->weights.final_norm = tensor(*m, 2048, ++s, true);
    if (cudaDeviceSynchronize() != cudaSuccess) return -2;
    if (cublasCreate(&m->handle) != CUBLAS_STATUS_SUCCESS) return -2;
    g_model = m;
    return 0;
  } catch (const std::exception&) {
    return -2;
  }
}

// prompts: [num_requests][prompt_len]; out_tokens: [num_requests][max_new];
// out_counts[r]: tokens generated for request r (EOS can end it early).
int e2e_generate(const int* prompts, int num_requests, int prompt_len, int max_new, int max_batch,
                 int max_seq_len, int* out_tokens, int* out_counts, double* seconds) {
  if (!g_model) return -1;
  try {
    std::vector<Request> requests(num_requests);
    for (int r = 0; r < num_requests; ++r) {
      requests[r].request_id = r;
      requests[r].prompt_tokens.assign(prompts + (size_t)r * prompt_len,
                                       prompts + (size_t)(r + 1) * prompt_len);
      requests[r].max_new_tokens = max_new;
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return -2;
    const auto t0 = std::chrono::steady_clock::now();
    generateContinuous(g_model->handle, g_model->weights, requests, max_batch, max_seq_len);
    if (cudaDeviceSynchronize() != cudaSuccess) return -2;
    *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    for (int r = 0; r < num_requests; ++r) {
      const auto& g = requests[r].generated_tokens;
      out_counts[r] = (int)g.size();
      for (int i = 0; i < max_new; ++i) out_tokens[(size_t)r * max_new + i] = i < (int)g.size() ? g[i] : -1;
    }
    return 0;
  } catch (const std::invalid_argument&) {
    return -1;
  } catch (const std::exception&) {
    return -2;
  }
}

// The reference's RMSNorm over `rows` rows of 2048 (src/model/rmsNorm.cu:3-22),
// launched with the shape its engine uses (paged_transformer.cu:68), on the
// legacy default stream.
int e2e_ref_rmsnorm(void* input, void* output, void* gain, int rows) {
  rmsNormKernel<<<rows, 1024>>>(static_cast<__nv_bfloat16*>(input),
                                static_cast<__nv_bfloat16*>(output),
                                static_cast<__nv_bfloat16*>(gain));
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Continuous batching over ragged requests: request r has prompt
// prompts[prompt_offsets[r] .. prompt_offsets[r + 1]) and max_new[r] new
// tokens; generateContinuous runs them through max_batch slots.  out_tokens:
// [num_requests][max_out] (-1 padded), out_counts[r] tokens generated.
// The scheduler's events are written as records of
//   {iteration, slot, request_id, admitted, free_blocks, n_blocks, blocks[n_blocks]}
// into events (capacity events_cap ints); *events_len is the ints written.
int e2e_generate_requests(const int* prompts, const int* prompt_offsets, const int* max_new,
                          int num_requests, int max_batch, int max_seq_len, int max_out,
                          int* out_tokens, int* out_counts, int* events, int events_cap,
                          int* events_len) {
  if (!g_model || num_requests < 0) return -1;
  try {
    std::vector<Request> requests(num_requests);
    for (int r = 0; r < num_requests; ++r) {
      requests[r].request_id = r;
      requests[r].prompt_tokens.assign(prompts + prompt_offsets[r], prompts + prompt_offsets[r + 1]);
      requests[r].max_new_tokens = max_new[r];
    }
    std::vector<SchedulerEvent> ev;
    generateContinuous(g_model->handle, g_model->weights, requests, max_batch, max_seq_len, &ev);
    if (cudaDeviceSynchronize() != cudaSuccess) return -2;
    for (int r = 0; r < num_requests; ++r) {
      const auto& g = requests[r].generated_tokens;
      out_counts[r] = (int)g.size();
      for (int i = 0; i < max_out; ++i) out_tokens[(size_t)r * max_out + i] = i < (int)g.size() ? g[i] : -1;
      if (!requests[r].finished || !requests[r].kv_state.block_table.empty() ||
          requests[r].kv_state.current_seq_len != 0)
        return -3;  // a finished request must hold no pages
    }
    int n = 0;
    for (const auto& e : ev) {
      const int need = 6 + (int)e.blocks.size();
      if (n + need > events_cap) return -4;
      events[n++] = e.iteration;
      events[n++] = e.slot;
      events[n++] = e.request_id;
      events[n++] = e.admitted ? 1 : 0;
      events[n++] = e.free_blocks;
      events[n++] = (int)e.blocks.size();
      for (int b : e.blocks) events[n++] = b;
    }
    *events_len = n;
    return 0;
  } catch (const std::invalid_argument&) {
    return -1;
  } catch (const std::exception&) {
    return -2;
  }
}

// Teacher-forced decode: prefill every prompt, then feed forced[r][step] as
// the input token of step `step` for all rows at once through decodeBatchPaged
// (whichever paged_transformer is linked), recording per row and step the
// engine's argmax token and the FP32 logits row (logits_out: [steps][B][VOCAB],
// may be NULL).  first_tokens[r] is the prefill's argmax and
// prefill_logits_out[r] (may be NULL) its FP32 logits row.
int e2e_teacher_forced(const int* prompts, int num_requests, int prompt_len, const int* forced,
                       int steps, int max_seq_len, int* first_tokens, int* step_tokens,
                       float* logits_out, float* prefill_logits_out) {
  if (!g_model || num_requests < 1 || num_requests > MAX_BATCH_SIZE) return -1;
  PagedKVCache cache{};
  TransformerBuffers prefill{}, decode{};
  __nv_bfloat16* hidden = nullptr;
  int* gpu_tokens = nullptr;
  float* logits = nullptr;
  std::vector<SequenceKVState> states(num_requests);
  int rc = 0;
  try {
    allocatePagedKVCache(cache, num_requests * ((max_seq_len + BLOCK_SIZE - 1) / BLOCK_SIZE));
    allocateTransformerBuffers(prefill, prompt_len, max_seq_len);
    allocateTransformerBuffers(decode, num_requests, num_requests * max_seq_len);
    const int cap = prompt_len > num_requests ? prompt_len : num_requests;
    if (cudaMalloc(&hidden, (size_t)cap * 2048 * sizeof(__nv_bfloat16)) != cudaSuccess ||
        cudaMalloc(&gpu_tokens, cap * sizeof(int)) != cudaSuccess ||
        cudaMalloc(&logits, (size_t)num_requests * VOCAB_SIZE * sizeof(float)) != cudaSuccess)
      throw std::runtime_error("cudaMalloc");
    for (int r = 0; r < num_requests; ++r) {
      cudaMemcpy(gpu_tokens, prompts + (size_t)r * prompt_len, prompt_len * sizeof(int),
                 cudaMemcpyHostToDevice);
      embeddingGatherKernel<<<prompt_len, 1024>>>(gpu_tokens, hidden, g_model->weights.embedding);
      first_tokens[r] = transformerForwardPaged(g_model->handle, hidden, g_model->weights, cache,
                                                states[r], prefill, logits, prompt_len);
      if (prefill_logits_out &&
          cudaMemcpy(prefill_logits_out + (size_t)r * VOCAB_SIZE, logits,
                     (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost) != cudaSuccess)
        throw std::runtime_error("prefill logits copy");
    }
    std::vector<SequenceKVState*> rows;
    for (auto& s : states) rows.push_back(&s);
    std::vector<int> in(num_requests);
    for (int step = 0; step < steps; ++step) {
      for (int r = 0; r < num_requests; ++r) in[r] = forced[(size_t)r * steps + step];
      cudaMemcpy(gpu_tokens, in.data(), num_requests * sizeof(int), cudaMemcpyHostToDevice);
      embeddingGatherKernel<<<num_requests, 1024>>>(gpu_tokens, hidden, g_model->weights.embedding);
      const std::vector<int> out =
          decodeBatchPaged(g_model->handle, hidden, g_model->weights, cache, rows, decode, logits);
      for (int r = 0; r < num_requests; ++r) step_tokens[(size_t)step * num_requests + r] = out[r];
      if (logits_out &&
          cudaMemcpy(logits_out + (size_t)step * num_requests * VOCAB_SIZE, logits,
                     (size_t)num_requests * VOCAB_SIZE * sizeof(float),
                     cudaMemcpyDeviceToHost) != cudaSuccess)
        throw std::runtime_error("logits copy");
    }
  } catch (const std::invalid_argument&) {
    rc = -1;
  } catch (const std::exception&) {
    rc = -2;
  }
  for (auto& s : states)
    if (cache.k_blocks) freeSequenceBlocks(cache, s);
  freePagedKVCache(cache);
  freeTransformerBuffers(prefill);
  freeTransformerBuffers(decode);
  cudaFree(hidden);
  cudaFree(gpu_tokens);
  cudaFree(logits);
  return rc;
}

}  // extern "C"
