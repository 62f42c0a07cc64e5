// Decode attention for callers that cannot allocate device memory.
//
// tvp_paged_decode_attention needs a scratch workspace (plan header, page
// prefix sums, split-K counters and partial results) that the caller normally
// allocates once with cudaMalloc.  Some callers cannot do that: code running
// under an allocator that forbids raw cudaMalloc (a host framework that owns
// all device memory through its own pool), a plug-in loaded into a process
// whose memory budget is fixed up front, or a host thread that must never
// block on the device-wide synchronisation a cudaMalloc/cudaFree can imply.
// For them this file keeps the workspace in a fixed device array that is part
// of the library image itself, so the call below allocates nothing.
#include <mutex>

#include "tvp_common.cuh"
#include "tvp_params.cuh"

namespace {

// Largest workspace the no-allocation entry point can serve.  4 MiB covers a
// one-CTA-per-SM B200 grid (~2.5 MB of split-K partials) plus page prefix sums
// and counters for batches of up to 46,968 rows (8 KV heads, 148 CTAs).  Every GPU that loads
// this library keeps these 4 MiB resident until the process exits.
constexpr size_t kStaticWorkspaceBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

// Device address of g_static_workspace per device.  In host code the array's
// name is only a host-side stand-in: the address a kernel may use must come
// from cudaGetSymbolAddress, called with the device current.  It is resolved
// once per device, on the first call there, and kept for the life of the
// process: after cudaDeviceReset (or any teardown of the device's primary
// context) the library's module is loaded again and the array may move, so
// this entry point must not be used across a device reset.
void* g_workspace_ptr[64] = {};
std::mutex g_workspace_mutex;

int static_workspace(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TVP_ERR_RUNTIME;
  std::lock_guard<std::mutex> lock(g_workspace_mutex);
  if (!g_workspace_ptr[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_workspace) != cudaSuccess || !ptr)
      return TVP_ERR_RUNTIME;
    g_workspace_ptr[dev] = ptr;
  }
  *out = g_workspace_ptr[dev];
  return TVP_OK;
}

}  // namespace

extern "C" {

int tvp_paged_decode_attention_noalloc(const tvp_bf16* q, const tvp_bf16* k_pool,
                                       const tvp_bf16* v_pool, int num_pages, int num_layers,
                                       int layer, int kv_heads, int q_heads,
                                       const int32_t* d_block_tables, int table_stride,
                                       const int32_t* d_seq_lens, int batch, float scale,
                                       int num_ctas, tvp_bf16* out, int32_t* d_error,
                                       tvp_stream_t stream) {
  // Every argument check of the decode runs before anything is enqueued, so a
  // rejected call leaves the shared array and the error word untouched.
  const int arc = tvp::check_decode_args(q, k_pool, v_pool, out, num_pages, num_layers, layer,
                                         kv_heads, q_heads, d_block_tables, table_stride,
                                         d_seq_lens, batch, scale, TVP_MODE_FAST, num_ctas);
  if (arc != TVP_OK) return arc;
  const size_t need = tvp_decode_workspace_bytes(batch, kv_heads, num_ctas);
  if (need == 0)
    return (kv_heads == 1 || kv_heads == 2 || kv_heads == 4 || kv_heads == TVP_KV_HEADS)
               ? TVP_ERR_RUNTIME
               : TVP_ERR_UNSUPPORTED;
  if (need > kStaticWorkspaceBytes) return TVP_ERR_WORKSPACE;  // batch or grid too large
  void* ws = nullptr;
  const int rc = static_workspace(&ws);
  if (rc != TVP_OK) return rc;
  // The plan rewrites the header and prefix sums and zeroes the split-K
  // counters, so nothing left in the array by an earlier call is read.
  const int prc = tvp_decode_plan(d_seq_lens, batch, table_stride, kv_heads, num_ctas, ws,
                                  kStaticWorkspaceBytes, d_error, stream);
  if (prc != TVP_OK) return prc;
  return tvp_paged_decode_attention(q, k_pool, v_pool, num_pages, num_layers, layer, kv_heads,
                                    q_heads, d_block_tables, table_stride, d_seq_lens, batch,
                                    scale, TVP_MODE_FAST, num_ctas, ws, kStaticWorkspaceBytes, out,
                                    d_error, stream);
}

}  // extern "C"
