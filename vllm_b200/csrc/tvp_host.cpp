// Host side of the paged-KV path: the reference's allocator and batch
// metadata (src/model/paged_kvcache.cu:19-139, src/model/paged_attention.cu:20-87)
// re-expressed in C++ over the fused kernels, plus the C-ABI handle functions
// of include/tvp_paged.h that expose it without C++ types.
#include <algorithm>
#include <cstring>
#include <limits>
#include <new>
#include <stdexcept>
#include <string>
#include <utility>

#include "tvp_paged.h"
#include "tvp_paged.hpp"

namespace tvp {
namespace {

void check_cuda(cudaError_t status) {
  if (status != cudaSuccess) throw std::runtime_error(cudaGetErrorString(status));
}

void check_rc(int rc) {
  if (rc == TVP_OK) return;
  if (rc == TVP_ERR_INVALID_ARGUMENT) throw std::invalid_argument(tvp_strerror(rc));
  throw std::runtime_error(tvp_strerror(rc));
}

void validate_cache(const PagedKVCache& cache) {
  if ((cache.device_storage && (!cache.k_blocks || !cache.v_blocks)) || cache.num_blocks <= 0 ||
      cache.block_size != BLOCK_SIZE)
    throw std::invalid_argument("Paged cache is not allocated");
}

bool in_free_list(const PagedKVCache& cache, int block) {
  return std::find(cache.free_blocks.begin(), cache.free_blocks.end(), block) !=
         cache.free_blocks.end();
}

// Same checks as validateSequenceBlocks (src/model/paged_kvcache.cu:25-35):
// every entry in range, not free, not repeated earlier in the table.
void validate_sequence_blocks(const PagedKVCache& cache, const SequenceKVState& sequence) {
  validate_cache(cache);
  for (size_t i = 0; i < sequence.block_table.size(); ++i) {
    const int block = sequence.block_table[i];
    if (block < 0 || block >= cache.num_blocks || in_free_list(cache, block) ||
        std::find(sequence.block_table.begin(), sequence.block_table.begin() + i, block) !=
            sequence.block_table.begin() + i)
      throw std::invalid_argument("Invalid or duplicate sequence block");
  }
}

int pages_for(int tokens) { return (tokens + BLOCK_SIZE - 1) / BLOCK_SIZE; }

void ensure_scratch(PagedKVCache& cache, size_t ints) {
  if (cache.scratch_ints >= ints) return;
  if (cache.d_scratch) cudaFree(cache.d_scratch);
  cache.d_scratch = nullptr;
  cache.scratch_ints = 0;
  check_cuda(cudaMalloc(reinterpret_cast<void**>(&cache.d_scratch), ints * sizeof(int)));
  cache.scratch_ints = ints;
}

}  // namespace

void allocatePagedKVCache(PagedKVCache& cache, int num_blocks, int num_layers, int max_seq_len,
                          bool device_storage) {
  if (cache.k_blocks || cache.v_blocks || cache.num_blocks != 0 || !cache.free_blocks.empty())
    throw std::invalid_argument("Paged cache already owns storage");
  const size_t bytes_per_block =
      static_cast<size_t>(num_layers > 0 ? num_layers : 1) * BLOCK_SIZE * TVP_KV_HEADS *
      TVP_HEAD_DIM * sizeof(__nv_bfloat16);
  if (num_blocks <= 0 || num_layers <= 0 || max_seq_len <= 0 ||
      static_cast<size_t>(num_blocks) > std::numeric_limits<size_t>::max() / bytes_per_block)
    throw std::invalid_argument("Invalid paged cache capacity");
  PagedKVCache pending{};
  pending.num_layers = num_layers;
  pending.max_seq_len = max_seq_len;
  pending.device_storage = device_storage;
  try {
    pending.free_blocks.reserve(num_blocks);
    for (int block = num_blocks - 1; block >= 0; --block) pending.free_blocks.push_back(block);
    if (device_storage) {
      const size_t bytes = static_cast<size_t>(num_blocks) * bytes_per_block;
      check_cuda(cudaMalloc(reinterpret_cast<void**>(&pending.k_blocks), bytes));
      check_cuda(cudaMalloc(reinterpret_cast<void**>(&pending.v_blocks), bytes));
      check_cuda(cudaMalloc(reinterpret_cast<void**>(&pending.d_error), sizeof(int)));
      check_cuda(cudaMemset(pending.d_error, 0, sizeof(int)));
    }
    pending.num_blocks = num_blocks;
  } catch (...) {
    freePagedKVCache(pending);
    throw;
  }
  cache = std::move(pending);
}

void freePagedKVCache(PagedKVCache& cache) {
  cudaFree(cache.k_blocks);
  cudaFree(cache.v_blocks);
  cudaFree(cache.d_scratch);
  cudaFree(cache.d_error);
  cache = PagedKVCache{};
}

int allocatePhysicalBlock(PagedKVCache& cache) {
  validate_cache(cache);
  if (cache.free_blocks.empty()) throw std::runtime_error("Paged KV cache has no free blocks");
  const int block = cache.free_blocks.back();
  cache.free_blocks.pop_back();
  return block;
}

void freePhysicalBlock(PagedKVCache& cache, int physical_block) {
  validate_cache(cache);
  if (physical_block < 0 || physical_block >= cache.num_blocks ||
      in_free_list(cache, physical_block))
    throw std::invalid_argument("Invalid block or double free");
  cache.free_blocks.push_back(physical_block);
}

void freeSequenceBlocks(PagedKVCache& cache, SequenceKVState& sequence) {
  validate_sequence_blocks(cache, sequence);
  for (int block : sequence.block_table) freePhysicalBlock(cache, block);
  sequence.block_table.clear();
  sequence.current_seq_len = 0;
}

void reserveSequenceBlocks(PagedKVCache& cache, SequenceKVState& sequence, int total_seq_len) {
  validate_sequence_blocks(cache, sequence);
  if (sequence.current_seq_len < 0 || total_seq_len < sequence.current_seq_len ||
      total_seq_len > cache.max_seq_len ||
      static_cast<size_t>(pages_for(sequence.current_seq_len)) > sequence.block_table.size())
    throw std::invalid_argument("Invalid sequence length or incomplete block table");
  const size_t needed = static_cast<size_t>(pages_for(total_seq_len));
  if (needed <= sequence.block_table.size()) return;
  if (needed - sequence.block_table.size() > cache.free_blocks.size())
    throw std::runtime_error("Insufficient free paged KV blocks");
  sequence.block_table.reserve(needed);
  while (sequence.block_table.size() < needed)
    sequence.block_table.push_back(allocatePhysicalBlock(cache));
}

void storePagedKV(PagedKVCache& cache, SequenceKVState& sequence, int layer, __nv_bfloat16* k,
                  const __nv_bfloat16* v, int num_tokens, bool apply_rope, __nv_bfloat16* rope_q,
                  cudaStream_t stream) {
  if (layer < 0 || layer >= cache.num_layers || num_tokens <= 0 || !k || !v ||
      sequence.current_seq_len < 0 || sequence.current_seq_len > cache.max_seq_len ||
      num_tokens > cache.max_seq_len - sequence.current_seq_len)
    throw std::invalid_argument("Invalid paged KV store");
  if (!cache.device_storage) throw std::invalid_argument("Paged cache has no device storage");
  reserveSequenceBlocks(cache, sequence, sequence.current_seq_len + num_tokens);
  const int pages = static_cast<int>(sequence.block_table.size());
  // One upload of [block table | token positions | token rows (all 0)]; the
  // whole prompt belongs to block-table row 0 of a one-row table.
  const size_t n = static_cast<size_t>(pages) + 2 * static_cast<size_t>(num_tokens);
  ensure_scratch(cache, n);
  std::vector<int> staging(n, 0);
  std::copy(sequence.block_table.begin(), sequence.block_table.end(), staging.begin());
  for (int i = 0; i < num_tokens; ++i) staging[pages + i] = sequence.current_seq_len + i;
  check_cuda(cudaMemcpyAsync(cache.d_scratch, staging.data(), n * sizeof(int),
                             cudaMemcpyHostToDevice, stream));
  // The staging vector is pageable: make sure the copy has consumed it.
  check_cuda(cudaStreamSynchronize(stream));
  int flags = 0;
  if (apply_rope) flags |= TVP_APPEND_ROPE_K | TVP_APPEND_WRITEBACK_K;
  if (apply_rope && rope_q) flags |= TVP_APPEND_ROPE_Q;
  check_rc(tvp_rope_append(
      reinterpret_cast<tvp_bf16*>(cache.k_blocks), reinterpret_cast<tvp_bf16*>(cache.v_blocks),
      cache.num_blocks, cache.num_layers, layer, cache.kv_heads, cache.d_scratch, pages,
      /*num_seqs=*/1, /*d_token_seq=*/cache.d_scratch + pages + num_tokens,
      cache.d_scratch + pages, num_tokens, reinterpret_cast<tvp_bf16*>(k),
      reinterpret_cast<const tvp_bf16*>(v), reinterpret_cast<tvp_bf16*>(rope_q), TVP_Q_HEADS,
      flags, cache.d_error, stream));
}

void createPagedBatch(PagedBatchMetadata& metadata, int max_batch, int table_stride) {
  if (max_batch <= 0 || table_stride <= 0 || metadata.block_tables)
    throw std::invalid_argument("Invalid paged batch capacity");
  PagedBatchMetadata m{};
  try {
    m.max_batch = max_batch;
    m.table_stride = table_stride;
    check_rc(tvp_device_sm_count(&m.num_ctas));
    const size_t table_ints = static_cast<size_t>(max_batch) * table_stride;
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&m.block_tables), table_ints * sizeof(int)));
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&m.positions), 2 * max_batch * sizeof(int)));
    m.lengths_dev = m.positions + max_batch;
    check_cuda(cudaMalloc(reinterpret_cast<void**>(&m.d_error), sizeof(int)));
    check_cuda(cudaMemset(m.d_error, 0, sizeof(int)));
    m.workspace_bytes = tvp_decode_workspace_bytes(max_batch, TVP_KV_HEADS, m.num_ctas);
    if (m.workspace_bytes == 0) throw std::runtime_error("workspace size query failed");
    check_cuda(cudaMalloc(&m.workspace, m.workspace_bytes));
    check_cuda(cudaMallocHost(reinterpret_cast<void**>(&m.h_staging),
                              (table_ints + 2 * max_batch) * sizeof(int)));
    check_cuda(cudaEventCreateWithFlags(&m.staged, cudaEventDisableTiming));
  } catch (...) {
    destroyPagedBatch(m);
    throw;
  }
  metadata = std::move(m);
}

void destroyPagedBatch(PagedBatchMetadata& metadata) {
  if (metadata.staged) cudaEventSynchronize(metadata.staged);
  cudaFree(metadata.block_tables);
  cudaFree(metadata.positions);
  cudaFree(metadata.d_error);
  cudaFree(metadata.workspace);
  if (metadata.h_staging) cudaFreeHost(metadata.h_staging);
  if (metadata.staged) cudaEventDestroy(metadata.staged);
  metadata = PagedBatchMetadata{};
}

void preparePagedBatch(PagedKVCache& cache, const std::vector<SequenceKVState*>& sequences,
                       PagedBatchMetadata& metadata, cudaStream_t stream) {
  validate_cache(cache);
  if (!cache.device_storage || !metadata.block_tables || sequences.empty() ||
      static_cast<int>(sequences.size()) > metadata.max_batch)
    throw std::invalid_argument("Invalid paged decode batch");
  // Validation before any mutation, as src/model/paged_attention.cu:41-58.
  size_t needed = 0;
  std::vector<int> owners(cache.num_blocks, -1);
  for (size_t row = 0; row < sequences.size(); ++row) {
    const SequenceKVState* sequence = sequences[row];
    if (!sequence || sequence->current_seq_len < 1 ||
        sequence->current_seq_len >= cache.max_seq_len)
      throw std::invalid_argument("Paged decode requires 1..max_seq_len-1 cached tokens");
    for (int block : sequence->block_table) {
      if (block < 0 || block >= cache.num_blocks || owners[block] != -1)
        throw std::invalid_argument("Paged decode sequences must own distinct blocks");
      owners[block] = static_cast<int>(row);
    }
    const size_t required = static_cast<size_t>((sequence->current_seq_len + BLOCK_SIZE) / BLOCK_SIZE);
    if (required > sequence->block_table.size()) needed += required - sequence->block_table.size();
  }
  if (needed > cache.free_blocks.size())
    throw std::runtime_error("Insufficient blocks for decode batch");
  const int batch = static_cast<int>(sequences.size());
  const int stride = metadata.table_stride;
  // The previous step's upload must have left the pinned staging buffer.
  check_cuda(cudaEventSynchronize(metadata.staged));
  int* tables = metadata.h_staging;
  int* positions = tables + static_cast<size_t>(metadata.max_batch) * stride;
  int* lengths = positions + metadata.max_batch;
  std::fill(tables, tables + static_cast<size_t>(batch) * stride, -1);
  metadata.lengths.clear();
  for (int row = 0; row < batch; ++row) {
    SequenceKVState& sequence = *sequences[row];
    reserveSequenceBlocks(cache, sequence, sequence.current_seq_len + 1);
    if (static_cast<int>(sequence.block_table.size()) > stride)
      throw std::invalid_argument("Paged block table exceeds context limit");
    std::copy(sequence.block_table.begin(), sequence.block_table.end(),
              tables + static_cast<size_t>(row) * stride);
    positions[row] = sequence.current_seq_len;
    lengths[row] = sequence.current_seq_len + 1;
    metadata.lengths.push_back(sequence.current_seq_len + 1);
  }
  metadata.batch_size = batch;
  check_cuda(cudaMemcpyAsync(metadata.block_tables, tables,
                             static_cast<size_t>(batch) * stride * sizeof(int),
                             cudaMemcpyHostToDevice, stream));
  check_cuda(cudaMemcpyAsync(metadata.positions, positions, batch * sizeof(int),
                             cudaMemcpyHostToDevice, stream));
  check_cuda(cudaMemcpyAsync(metadata.lengths_dev, lengths, batch * sizeof(int),
                             cudaMemcpyHostToDevice, stream));
  check_cuda(cudaEventRecord(metadata.staged, stream));
  check_rc(tvp_decode_plan(metadata.lengths_dev, batch, stride, TVP_KV_HEADS, metadata.num_ctas,
                           metadata.workspace, metadata.workspace_bytes, metadata.d_error, stream));
}

void storePagedKVBatch(PagedKVCache& cache, const PagedBatchMetadata& metadata, int layer,
                       __nv_bfloat16* q, __nv_bfloat16* k, const __nv_bfloat16* v,
                       cudaStream_t stream) {
  validate_cache(cache);
  if (!metadata.block_tables || metadata.batch_size < 1 || layer < 0 ||
      layer >= cache.num_layers || !k || !v)
    throw std::invalid_argument("Invalid paged attention arguments");
  int flags = TVP_APPEND_ROPE_K | TVP_APPEND_WRITEBACK_K;
  if (q) flags |= TVP_APPEND_ROPE_Q;
  check_rc(tvp_rope_append(reinterpret_cast<tvp_bf16*>(cache.k_blocks),
                           reinterpret_cast<tvp_bf16*>(cache.v_blocks), cache.num_blocks,
                           cache.num_layers, layer, cache.kv_heads, metadata.block_tables,
                           metadata.table_stride, metadata.batch_size, nullptr, metadata.positions,
                           metadata.batch_size, reinterpret_cast<tvp_bf16*>(k),
                           reinterpret_cast<const tvp_bf16*>(v), reinterpret_cast<tvp_bf16*>(q),
                           TVP_Q_HEADS, flags, metadata.d_error, stream));
}

void pagedDecodeAttention(const PagedKVCache& cache, PagedBatchMetadata& metadata, int layer,
                          const __nv_bfloat16* q, __nv_bfloat16* attention_output, int mode,
                          cudaStream_t stream) {
  validate_cache(cache);
  if (!metadata.block_tables || metadata.batch_size < 1 || layer < 0 ||
      layer >= cache.num_layers || !q || !attention_output)
    throw std::invalid_argument("Invalid paged attention arguments");
  check_rc(tvp_paged_decode_attention(
      reinterpret_cast<const tvp_bf16*>(q), reinterpret_cast<const tvp_bf16*>(cache.k_blocks),
      reinterpret_cast<const tvp_bf16*>(cache.v_blocks), cache.num_blocks, cache.num_layers,
      layer, cache.kv_heads, TVP_Q_HEADS, metadata.block_tables, metadata.table_stride,
      metadata.lengths_dev, metadata.batch_size, 0.125f, mode, metadata.num_ctas,
      metadata.workspace, metadata.workspace_bytes, reinterpret_cast<tvp_bf16*>(attention_output),
      metadata.d_error, stream));
}

int takePagedBatchError(PagedBatchMetadata& metadata, cudaStream_t stream) {
  int bits = 0;
  check_cuda(cudaStreamSynchronize(stream));
  check_cuda(cudaMemcpy(&bits, metadata.d_error, sizeof(int), cudaMemcpyDeviceToHost));
  check_cuda(cudaMemset(metadata.d_error, 0, sizeof(int)));
  return bits;
}

}  // namespace tvp

// ========================= C-ABI handle functions ==========================
struct tvp_cache {
  tvp::PagedKVCache impl;
};
struct tvp_seq {
  tvp::SequenceKVState impl;
};
struct tvp_batch {
  tvp::PagedBatchMetadata impl;
};

namespace {

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return TVP_OK;
  } catch (const std::invalid_argument&) {
    return TVP_ERR_INVALID_ARGUMENT;
  } catch (const std::bad_alloc&) {
    return TVP_ERR_RUNTIME;
  } catch (const std::runtime_error& e) {
    const std::string what = e.what();
    if (what.find("no free blocks") != std::string::npos ||
        what.find("Insufficient") != std::string::npos)
      return TVP_ERR_NO_FREE_BLOCKS;
    return TVP_ERR_RUNTIME;
  } catch (...) {
    return TVP_ERR_RUNTIME;
  }
}

}  // namespace

extern "C" {

int tvp_cache_create(int num_blocks, int num_layers, int kv_heads, int max_seq_len,
                     int device_storage, tvp_cache** out) {
  if (!out) return TVP_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (kv_heads != TVP_KV_HEADS) return TVP_ERR_UNSUPPORTED;
  tvp_cache* c = new (std::nothrow) tvp_cache();
  if (!c) return TVP_ERR_RUNTIME;
  const int rc = guarded([&] {
    tvp::allocatePagedKVCache(c->impl, num_blocks, num_layers, max_seq_len, device_storage != 0);
  });
  if (rc != TVP_OK) {
    delete c;
    return rc;
  }
  *out = c;
  return TVP_OK;
}

void tvp_cache_destroy(tvp_cache* cache) {
  if (!cache) return;
  tvp::freePagedKVCache(cache->impl);
  delete cache;
}

int tvp_cache_pools(const tvp_cache* cache, tvp_bf16** k_pool, tvp_bf16** v_pool, int* num_blocks) {
  if (!cache) return TVP_ERR_INVALID_ARGUMENT;
  if (k_pool) *k_pool = reinterpret_cast<tvp_bf16*>(cache->impl.k_blocks);
  if (v_pool) *v_pool = reinterpret_cast<tvp_bf16*>(cache->impl.v_blocks);
  if (num_blocks) *num_blocks = cache->impl.num_blocks;
  return TVP_OK;
}

int tvp_cache_free_count(const tvp_cache* cache) {
  return cache ? static_cast<int>(cache->impl.free_blocks.size()) : TVP_ERR_INVALID_ARGUMENT;
}

int tvp_cache_free_list(const tvp_cache* cache, int32_t* out, int capacity) {
  if (!cache || capacity < 0 || (capacity > 0 && !out)) return TVP_ERR_INVALID_ARGUMENT;
  const auto& f = cache->impl.free_blocks;
  const int n = static_cast<int>(f.size());
  for (int i = 0; i < n && i < capacity; ++i) out[i] = f[i];
  return n;
}

int tvp_cache_set_free_list(tvp_cache* cache, const int32_t* blocks, int count) {
  if (!cache || count < 0 || (count > 0 && !blocks) || count > cache->impl.num_blocks)
    return TVP_ERR_INVALID_ARGUMENT;
  std::vector<int> seen(cache->impl.num_blocks, 0);
  for (int i = 0; i < count; ++i) {
    if (blocks[i] < 0 || blocks[i] >= cache->impl.num_blocks || seen[blocks[i]]++)
      return TVP_ERR_INVALID_ARGUMENT;
  }
  cache->impl.free_blocks.assign(blocks, blocks + count);
  return TVP_OK;
}

int tvp_allocate_physical_block(tvp_cache* cache, int* out_block) {
  if (!cache || !out_block) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] { *out_block = tvp::allocatePhysicalBlock(cache->impl); });
}

int tvp_free_physical_block(tvp_cache* cache, int block) {
  if (!cache) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] { tvp::freePhysicalBlock(cache->impl, block); });
}

int tvp_seq_create(tvp_seq** out) {
  if (!out) return TVP_ERR_INVALID_ARGUMENT;
  *out = new (std::nothrow) tvp_seq();
  return *out ? TVP_OK : TVP_ERR_RUNTIME;
}

void tvp_seq_destroy(tvp_seq* seq) { delete seq; }

int tvp_seq_length(const tvp_seq* seq) {
  return seq ? seq->impl.current_seq_len : TVP_ERR_INVALID_ARGUMENT;
}

int tvp_seq_set_length(tvp_seq* seq, int current_seq_len) {
  if (!seq) return TVP_ERR_INVALID_ARGUMENT;
  seq->impl.current_seq_len = current_seq_len;
  return TVP_OK;
}

int tvp_seq_block_table(const tvp_seq* seq, int32_t* out, int capacity) {
  if (!seq || capacity < 0 || (capacity > 0 && !out)) return TVP_ERR_INVALID_ARGUMENT;
  const auto& t = seq->impl.block_table;
  const int n = static_cast<int>(t.size());
  for (int i = 0; i < n && i < capacity; ++i) out[i] = t[i];
  return n;
}

int tvp_reserve_sequence_blocks(tvp_cache* cache, tvp_seq* seq, int total_seq_len) {
  if (!cache || !seq) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] { tvp::reserveSequenceBlocks(cache->impl, seq->impl, total_seq_len); });
}

int tvp_free_sequence_blocks(tvp_cache* cache, tvp_seq* seq) {
  if (!cache || !seq) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] { tvp::freeSequenceBlocks(cache->impl, seq->impl); });
}

int tvp_store_paged_kv(tvp_cache* cache, tvp_seq* seq, int layer, tvp_bf16* k, const tvp_bf16* v,
                       int num_tokens, int apply_rope, tvp_bf16* rope_q, tvp_stream_t stream) {
  if (!cache || !seq) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] {
    tvp::storePagedKV(cache->impl, seq->impl, layer, reinterpret_cast<__nv_bfloat16*>(k),
                      reinterpret_cast<const __nv_bfloat16*>(v), num_tokens, apply_rope != 0,
                      reinterpret_cast<__nv_bfloat16*>(rope_q), static_cast<cudaStream_t>(stream));
  });
}

int tvp_batch_create(int max_batch, int max_pages_per_seq, tvp_batch** out) {
  if (!out) return TVP_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  tvp_batch* b = new (std::nothrow) tvp_batch();
  if (!b) return TVP_ERR_RUNTIME;
  const int rc = guarded([&] { tvp::createPagedBatch(b->impl, max_batch, max_pages_per_seq); });
  if (rc != TVP_OK) {
    delete b;
    return rc;
  }
  *out = b;
  return TVP_OK;
}

void tvp_batch_destroy(tvp_batch* batch) {
  if (!batch) return;
  tvp::destroyPagedBatch(batch->impl);
  delete batch;
}

int tvp_prepare_paged_batch(tvp_cache* cache, tvp_seq* const* seqs, int count, tvp_batch* batch,
                            tvp_stream_t stream) {
  if (!cache || !seqs || !batch || count <= 0) return TVP_ERR_INVALID_ARGUMENT;
  std::vector<tvp::SequenceKVState*> rows(count);
  for (int i = 0; i < count; ++i) rows[i] = seqs[i] ? &seqs[i]->impl : nullptr;
  return guarded([&] {
    tvp::preparePagedBatch(cache->impl, rows, batch->impl, static_cast<cudaStream_t>(stream));
  });
}

int tvp_batch_positions(const tvp_batch* batch, const int32_t** d_positions,
                        const int32_t** d_lengths, const int32_t** d_tables, int* table_stride) {
  if (!batch) return TVP_ERR_INVALID_ARGUMENT;
  if (d_positions) *d_positions = batch->impl.positions;
  if (d_lengths) *d_lengths = batch->impl.lengths_dev;
  if (d_tables) *d_tables = batch->impl.block_tables;
  if (table_stride) *table_stride = batch->impl.table_stride;
  return batch->impl.batch_size;
}

int tvp_store_paged_kv_batch(tvp_cache* cache, const tvp_batch* batch, int layer, tvp_bf16* q,
                             tvp_bf16* k, const tvp_bf16* v, tvp_stream_t stream) {
  if (!cache || !batch) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] {
    tvp::storePagedKVBatch(cache->impl, batch->impl, layer, reinterpret_cast<__nv_bfloat16*>(q),
                           reinterpret_cast<__nv_bfloat16*>(k),
                           reinterpret_cast<const __nv_bfloat16*>(v),
                           static_cast<cudaStream_t>(stream));
  });
}

int tvp_paged_attention(const tvp_cache* cache, tvp_batch* batch, int layer, const tvp_bf16* q,
                        tvp_bf16* out, int mode, tvp_stream_t stream) {
  if (!cache || !batch) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] {
    tvp::pagedDecodeAttention(cache->impl, batch->impl, layer,
                              reinterpret_cast<const __nv_bfloat16*>(q),
                              reinterpret_cast<__nv_bfloat16*>(out), mode,
                              static_cast<cudaStream_t>(stream));
  });
}

int tvp_batch_error(tvp_batch* batch, tvp_stream_t stream, int32_t* out_bits) {
  if (!batch || !out_bits) return TVP_ERR_INVALID_ARGUMENT;
  return guarded([&] {
    *out_bits = tvp::takePagedBatchError(batch->impl, static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
