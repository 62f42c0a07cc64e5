// KV-head-sharded decode with the all-gather fused into the decode kernel.
//
// The reference has no multi-GPU path; this is the KV-head-sharded variant of
// its decode block (src/model/paged_transformer.cu:85-94): GPU r of `world`
// holds KV heads [r K, (r + 1) K), K = 8 / world, of every page, computes
// query heads [4 r K, 4 (r + 1) K) and the [B][2048] attention rows are
// assembled on every GPU.  Instead of a decode followed by a collective, the
// decode kernel stores each finished output group straight into every rank's
// gathered rows (peer memory opened through CUDA IPC, plain stores over
// NVLink); its last CTA adds 1 to every rank's flag and waits, bounded, until
// every rank has signalled, so the launch ends with all ranks' rows in place.
//
// Per rank, one device allocation, exported once:
//   [flag 0 | flag 1 | done counter | pad to 256 B][rows 0][rows 1]
// rows b = [max_batch][2048] BF16 (two buffers, so that a rank can decode the
// next layer into one while its consumers still read the other).
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "tvp_params.cuh"

struct tvp_head_gather {
  int world = 0, rank = 0, kv_heads = 0, max_batch = 0, device = -1;
  char* base = nullptr;       // this rank's allocation
  size_t rows_bytes = 0, total = 0;
  std::vector<char*> peer_base;  // per rank: its allocation, opened here (own base at `rank`)
  void** d_table = nullptr;   // device: rows0[world], rows1[world], flag0[world], flag1[world]
  uint32_t epoch[2] = {0, 0}; // gather launches per buffer
  bool connected = false;
};

namespace tvp {
namespace {

constexpr size_t kGatherHeader = 256;
constexpr int kGatherRow = kMaxKvHeads * kGroup * kHeadDim;  // 2048 channels

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

int32_t* flag_of(char* base, int buffer) { return reinterpret_cast<int32_t*>(base) + buffer; }
int32_t* done_of(char* base) { return reinterpret_cast<int32_t*>(base) + 2; }
char* rows_of(char* base, size_t rows_bytes, int buffer) {
  return base + kGatherHeader + (size_t)buffer * rows_bytes;
}

bool on_device(const tvp_head_gather* g) {
  int dev = -1;
  return cudaGetDevice(&dev) == cudaSuccess && dev == g->device;
}

}  // namespace
}  // namespace tvp

using namespace tvp;

extern "C" {

int tvp_head_gather_create(int world, int rank, int kv_heads, int max_batch,
                           tvp_head_gather** out) {
  if (!out || max_batch <= 0 || rank < 0 || rank >= world) return TVP_ERR_INVALID_ARGUMENT;
  if (!(world == 2 || world == 4 || world == 8) || kv_heads * world != kMaxKvHeads)
    return TVP_ERR_UNSUPPORTED;
  auto* g = new (std::nothrow) tvp_head_gather();
  if (!g) return TVP_ERR_RUNTIME;
  g->world = world;
  g->rank = rank;
  g->kv_heads = kv_heads;
  g->max_batch = max_batch;
  g->rows_bytes = round_up((size_t)max_batch * kGatherRow * 2, 256);
  g->total = kGatherHeader + 2 * g->rows_bytes;
  bool ok = cudaGetDevice(&g->device) == cudaSuccess &&
            cudaMalloc(reinterpret_cast<void**>(&g->base), g->total) == cudaSuccess &&
            cudaMemset(g->base, 0, g->total) == cudaSuccess &&
            cudaMalloc(reinterpret_cast<void**>(&g->d_table), 4 * world * sizeof(void*)) ==
                cudaSuccess &&
            cudaDeviceSynchronize() == cudaSuccess;  // flags are zero before any peer sees them
  if (!ok) {
    if (g->base) cudaFree(g->base);
    if (g->d_table) cudaFree(g->d_table);
    delete g;
    return TVP_ERR_RUNTIME;
  }
  g->peer_base.assign(world, nullptr);
  g->peer_base[rank] = g->base;
  *out = g;
  return TVP_OK;
}

int tvp_head_gather_export(const tvp_head_gather* g, void* handle_out) {
  if (!g || !handle_out) return TVP_ERR_INVALID_ARGUMENT;
  if (!on_device(g)) return TVP_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, g->base) != cudaSuccess) return TVP_ERR_RUNTIME;
  static_assert(sizeof(cudaIpcMemHandle_t) <= TVP_IPC_HANDLE_BYTES, "IPC handle size");
  std::memset(handle_out, 0, TVP_IPC_HANDLE_BYTES);
  std::memcpy(handle_out, &h, sizeof(h));
  return TVP_OK;
}

int tvp_head_gather_connect(tvp_head_gather* g, const void* handles) {
  if (!g || !handles || g->connected) return TVP_ERR_INVALID_ARGUMENT;
  if (!on_device(g)) return TVP_ERR_INVALID_ARGUMENT;
  const char* hs = static_cast<const char*>(handles);
  for (int r = 0; r < g->world; ++r) {
    if (r == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + (size_t)r * TVP_IPC_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != g->rank && g->peer_base[q]) cudaIpcCloseMemHandle(g->peer_base[q]);
      std::fill(g->peer_base.begin(), g->peer_base.end(), nullptr);
      g->peer_base[g->rank] = g->base;
      return TVP_ERR_RUNTIME;
    }
    g->peer_base[r] = static_cast<char*>(ptr);
  }
  std::vector<void*> table(4 * g->world);
  for (int r = 0; r < g->world; ++r) {
    table[0 * g->world + r] = rows_of(g->peer_base[r], g->rows_bytes, 0);
    table[1 * g->world + r] = rows_of(g->peer_base[r], g->rows_bytes, 1);
    table[2 * g->world + r] = flag_of(g->peer_base[r], 0);
    table[3 * g->world + r] = flag_of(g->peer_base[r], 1);
  }
  if (cudaMemcpy(g->d_table, table.data(), table.size() * sizeof(void*), cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return TVP_ERR_RUNTIME;
  g->connected = true;
  return TVP_OK;
}

int tvp_head_gather_rows(const tvp_head_gather* g, int buffer, tvp_bf16** rows_out) {
  if (!g || !rows_out || buffer < 0 || buffer > 1) return TVP_ERR_INVALID_ARGUMENT;
  *rows_out = reinterpret_cast<tvp_bf16*>(rows_of(g->base, g->rows_bytes, buffer));
  return TVP_OK;
}

int tvp_paged_decode_attention_gather(const tvp_bf16* q, const tvp_bf16* k_pool,
                                      const tvp_bf16* v_pool, int num_pages, int num_layers,
                                      int layer, int kv_heads, int q_heads,
                                      const int32_t* d_block_tables, int table_stride,
                                      const int32_t* d_seq_lens, int batch, float scale,
                                      int num_ctas, void* d_workspace, size_t workspace_bytes,
                                      tvp_head_gather* g, int buffer, int32_t* d_error,
                                      tvp_stream_t stream) {
  if (!g || !g->connected || buffer < 0 || buffer > 1 || batch > g->max_batch ||
      kv_heads != g->kv_heads || !on_device(g))
    return TVP_ERR_INVALID_ARGUMENT;
  DecodeParams p;
  long long pool_rows = 0;
  int ctas = 0;
  const int rc = prepare_decode(q, k_pool, v_pool, num_pages, num_layers, layer, kv_heads, q_heads,
                                d_block_tables, table_stride, d_seq_lens, batch, scale, num_ctas,
                                d_workspace, workspace_bytes, d_error, &p, &pool_rows, &ctas);
  if (rc != TVP_OK) return rc;
  p.peer_rows = reinterpret_cast<__nv_bfloat16* const*>(g->d_table + (size_t)buffer * g->world);
  p.peer_flags = reinterpret_cast<int32_t* const*>(g->d_table + (size_t)(2 + buffer) * g->world);
  p.done_counter = done_of(g->base);
  p.world = g->world;
  p.rank = g->rank;
  p.flag_target = (int32_t)((g->epoch[buffer] + 1u) * (uint32_t)g->world);
  if (launch_paged_decode(p, pool_rows, ctas, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return TVP_ERR_RUNTIME;
  ++g->epoch[buffer];
  return TVP_OK;
}

int tvp_head_gather_disconnect(tvp_head_gather* g) {
  if (!g) return TVP_ERR_INVALID_ARGUMENT;
  int rc = TVP_OK;
  if (cudaDeviceSynchronize() != cudaSuccess) rc = TVP_ERR_RUNTIME;  // no launch still writes
  for (int r = 0; r < g->world; ++r)
    if (r != g->rank && g->peer_base[r]) {
      if (cudaIpcCloseMemHandle(g->peer_base[r]) != cudaSuccess) rc = TVP_ERR_RUNTIME;
      g->peer_base[r] = nullptr;
    }
  g->connected = false;
  return rc;
}

int tvp_head_gather_destroy(tvp_head_gather* g) {
  if (!g) return TVP_ERR_INVALID_ARGUMENT;
  int rc = g->connected ? tvp_head_gather_disconnect(g) : TVP_OK;
  if (g->d_table && cudaFree(g->d_table) != cudaSuccess) rc = TVP_ERR_RUNTIME;
  if (g->base && cudaFree(g->base) != cudaSuccess) rc = TVP_ERR_RUNTIME;
  delete g;
  return rc;
}

}  // extern "C"
