/*
 * tvp_paged.h — C-ABI of the B200 paged-KV hot path for the tiny-vLLM
 * Llama-3.2-1B engine (arpitsri28/vllm).
 *
 * Plain pointers and sizes only: no C++ types, no torch types.  Every entry
 * point returns 0 (TVP_OK) on success and a negative TVP_ERR_* code on
 * failure; nothing throws across this boundary.  The C++ host layer
 * (tvp_paged.hpp, namespace tvp) maps the codes back onto the reference's
 * exception types: TVP_ERR_INVALID_ARGUMENT -> std::invalid_argument,
 * everything else -> std::runtime_error.
 *
 * Geometry is the reference's hard-coded one (src/model/paged_kvcache.cu:10-11,
 * src/model/paged_attention.cu:10-12, src/model/RoPe.cu:7):
 *   head_dim 64, 16-token pages, 4 query heads per KV head (GQA),
 *   8 KV heads x 64 = 512 channels per cached token, 32 query heads.
 *
 * Pool layout (identical to the reference, src/model/paged_kvcache.cu:131):
 *   element (layer, page, slot, kv_head, d) of the K (or V) pool lives at
 *   ((layer * num_pages + page) * 16 + slot) * (kv_heads * 64) + kv_head * 64 + d
 * so a page of one layer is kv_heads * 2 KiB of contiguous BF16 per pool.
 *
 * "Device pointer" arguments (prefixed d_ or documented as such) must be CUDA
 * device memory of the current device.  "stream" is a cudaStream_t (NULL =
 * legacy default stream, as in the reference).  Kernels that detect a bad page
 * id, length or a stalled pipeline do not trap: they OR a TVP_DEVERR_* bit into
 * *d_error (optional, may be NULL) and skip the offending access.
 */
#ifndef TVP_PAGED_H
#define TVP_PAGED_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t tvp_bf16;   /* raw IEEE bfloat16 bits */
typedef void* tvp_stream_t;  /* cudaStream_t */

/* ---- return codes ----------------------------------------------------- */
#define TVP_OK 0
#define TVP_ERR_INVALID_ARGUMENT (-1) /* reference: std::invalid_argument          */
#define TVP_ERR_RUNTIME (-2)          /* reference: std::runtime_error (CUDA error)  */
#define TVP_ERR_NO_FREE_BLOCKS (-3)   /* reference: runtime_error, pool exhausted    */
#define TVP_ERR_UNSUPPORTED (-4)      /* geometry/mode this build does not provide   */
#define TVP_ERR_WORKSPACE (-5)        /* workspace missing or too small             */

/* ---- device error bits (written into *d_error by kernels) -------------- */
#define TVP_DEVERR_BAD_PAGE 1u     /* block-table entry outside [0, num_pages)   */
#define TVP_DEVERR_BAD_LENGTH 2u   /* sequence length < 0 or beyond its table    */
#define TVP_DEVERR_TIMEOUT 4u      /* a pipeline wait ran out its bound          */
#define TVP_DEVERR_BAD_PLAN 8u     /* workspace planned for another batch/grid   */
#define TVP_DEVERR_BAD_TOKEN 16u   /* append: token's sequence row or position invalid */
#define TVP_DEVERR_SMEM_ALIGN 32u  /* decode: shared window not 1 KiB aligned; nothing ran */
/* With TVP_DEVERR_TIMEOUT, which wait gave up: */
#define TVP_DEVERR_WAIT_FULL 0x100u   /* a consumer waiting for a stage's copies   */
#define TVP_DEVERR_WAIT_EMPTY 0x200u  /* the producer waiting for a free stage     */
#define TVP_DEVERR_WAIT_DRAIN 0x400u  /* the producer's wait for its last copies   */
#define TVP_DEVERR_WAIT_PEERS 0x800u  /* a gather waiting for the other ranks      */

/* ---- fixed geometry ---------------------------------------------------- */
#define TVP_HEAD_DIM 64
#define TVP_PAGE_TOKENS 16
#define TVP_GQA_GROUP 4
#define TVP_KV_HEADS 8
#define TVP_Q_HEADS 32

/* ---- decode attention numerics ----------------------------------------- */
/* FAST: one pass, FP32 online softmax (base-2 exponent), BF16 probabilities
 * into the P.V product, FP32 accumulation, BF16 output. */
#define TVP_MODE_FAST 0
/* COMPAT: the reference's rounding points (src/model/attention.cu:53-142,
 * src/model/softmax.cu:6-45): BF16 scores, exact max, expf, pairwise-tree sum,
 * BF16 probabilities, FP32 P.V, BF16 output.  Lengths up to 1,048,576. */
#define TVP_MODE_COMPAT 1

/* ---- flags of tvp_rope_append ------------------------------------------ */
#define TVP_APPEND_ROPE_K 1     /* apply llama3 RoPE to K before it is stored      */
#define TVP_APPEND_ROPE_Q 2     /* apply llama3 RoPE to q in place                  */
#define TVP_APPEND_WRITEBACK_K 4 /* also write the (RoPE'd) K back into k          */

const char* tvp_strerror(int code);
int tvp_version(void);

/* Number of SMs of the current device (the default decode grid size). */
int tvp_device_sm_count(int* out_sms);

/*
 * K1 — fused llama3 RoPE + paged KV append.
 *
 * Replaces, in one launch:
 *   rope(k)/ropeBatch(k)                 src/model/RoPe.cu:31-62 (K, in place)
 *   rope(q)/ropeBatch(q)                 src/model/RoPe.cu:31-62 (q, in place; optional)
 *   storePagedKV                         src/model/paged_kvcache.cu:119-139 (prefill)
 *   storePagedKVBatch / ...Kernel        src/model/paged_attention.cu:89-99,123-131 (decode)
 *
 * Token i (0 <= i < num_tokens) belongs to block-table row
 *   seq = d_token_seq ? d_token_seq[i] : i
 * and absolute position pos = d_token_pos[i]; it is written to slot pos % 16
 * of physical page d_block_tables[seq * table_stride + pos / 16].
 * k, v: [num_tokens][kv_heads * 64] BF16 (device).  q: [num_tokens][q_heads * 64]
 * (device, only with TVP_APPEND_ROPE_Q).  RoPE arithmetic is the reference
 * ropeKernel's, bit for bit.  Does not advance any sequence length.
 */
int tvp_rope_append(tvp_bf16* k_pool, tvp_bf16* v_pool, int num_pages, int num_layers,
                    int layer, int kv_heads, const int32_t* d_block_tables, int table_stride,
                    int num_seqs, const int32_t* d_token_seq, const int32_t* d_token_pos,
                    int num_tokens, tvp_bf16* k, const tvp_bf16* v, tvp_bf16* q, int q_heads,
                    int flags, int32_t* d_error, tvp_stream_t stream);

/*
 * Workspace of the decode path: plan header, per-sequence page prefix sums,
 * each CTA's first sequence, last-arriver counters and split-K partials for
 * `num_ctas` CTAs (0 = one per SM).  kv_heads is the number of KV heads the
 * pools hold: the model's 8, or 4, 2 or 1 for a GPU that holds a shard of the
 * heads (every page, only its heads' channels).  0 for any other value.
 */
size_t tvp_decode_workspace_bytes(int batch, int kv_heads, int num_ctas);

/*
 * Per-step plan (the device side of preparePagedBatch,
 * src/model/paged_attention.cu:30-87): page prefix sums over d_seq_lens, the
 * sequence holding each CTA's first page, and a reset of the split-K
 * counters.  One plan serves every layer of a decode step.
 * d_seq_lens[b] = attended length L (= current_seq_len + 1 after the append).
 */
int tvp_decode_plan(const int32_t* d_seq_lens, int batch, int table_stride, int kv_heads,
                    int num_ctas, void* d_workspace, size_t workspace_bytes, int32_t* d_error,
                    tvp_stream_t stream);

/*
 * K2 — fused GQA paged decode attention (+ split-K combine).
 *
 * Replaces src/model/paged_transformer.cu:85-94:
 *   computePagedAttentionScores (gather + 32*B cuBLAS GEMVs)  src/model/paged_attention.cu:133-146
 *   softmaxRows per (row, head)                               src/model/softmax.cu:47-72
 *   pagedAttentionScoresTimesV (gather + 32*B cuBLAS GEMVs)   src/model/paged_attention.cu:148-161
 * kv_heads: 8 (the model), or 4, 2, 1 for a KV-head shard; q_heads = 4 * kv_heads.
 * q:   [batch][q_heads * 64] BF16, already RoPE'd.
 * out: [batch][q_heads * 64] BF16, head-major (head h at h*64), as the reference.
 * out[b, h] = softmax(scale * q[b,h] . K[b, kv(h)]^T) . V[b, kv(h)] over the
 * first d_seq_lens[b] tokens of row b's pages, kv(h) = h / 4.
 * Pages are read in place.  The workspace must hold a plan made by
 * tvp_decode_plan with the same d_seq_lens contents, batch, kv_heads and
 * num_ctas.
 * With 8 KV heads in FAST mode the launch is a programmatic dependent launch:
 * when the kernel before it in the stream releases its dependents early, as
 * tvp_rope_append and tvp_decode_qkv_rope_append do, this kernel reads the
 * plan and the block tables while that kernel runs, and waits for it before
 * it reads q or any page.  So a kernel that releases its dependents early
 * must not write the plan, the workspace or the block tables when it runs
 * right before this call; after any other kernel (tvp_decode_plan included)
 * ordinary stream order holds.
 */
int tvp_paged_decode_attention(const tvp_bf16* q, const tvp_bf16* k_pool, const tvp_bf16* v_pool,
                               int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                               const int32_t* d_block_tables, int table_stride,
                               const int32_t* d_seq_lens, int batch, float scale, int mode,
                               int num_ctas, void* d_workspace, size_t workspace_bytes,
                               tvp_bf16* out, int32_t* d_error, tvp_stream_t stream);

/*
 * K3 — paged causal prefill attention, reading K and V from the pages.
 *
 * Replaces the prefill attention of src/model/paged_transformer.cu:37-40
 * (computeAttentionScores, causalMask, softmaxRows, attentionScoresTimesV over
 * the contiguous K/V, src/model/attention.cu:10-51,144-192,
 * src/model/causalMask.cu:7-38, src/model/softmax.cu:47-72), without its
 * 1024-token cap and without a score matrix in memory.
 * Queries are varlen: sequence s (row s of d_block_tables) owns query tokens
 * [d_cu_q[s], d_cu_q[s + 1]) at positions d_q_pos0[s], d_q_pos0[s] + 1, ...;
 * each attends the keys 0..its position already in the sequence's pages
 * (append them first with tvp_rope_append).  d_q_pos0[s] = 0 is a prompt;
 * d_q_pos0[s] = L0 > 0 a prefill chunk after L0 cached tokens.
 * q, out: [num_tokens][q_heads * 64] BF16, head-major as the reference,
 * 16-byte aligned; max_q_len >= the longest sequence's query count (at most
 * 65535 x 32 tokens: TVP_ERR_UNSUPPORTED beyond).  Scores are rounded to
 * BF16 where the reference rounds them, then an online softmax in base 2,
 * BF16 probabilities into P.V and FP32 accumulation.
 */
int tvp_paged_prefill_attention(const tvp_bf16* q, const tvp_bf16* k_pool, const tvp_bf16* v_pool,
                                int num_pages, int num_layers, int layer, int kv_heads, int q_heads,
                                const int32_t* d_block_tables, int table_stride,
                                const int32_t* d_cu_q, const int32_t* d_q_pos0, int num_seqs,
                                int max_q_len, float scale, tvp_bf16* out, int32_t* d_error,
                                tvp_stream_t stream);

/*
 * Greedy token selection for `rows` logit rows in one launch: replaces the
 * per-row argmaxLogits of the reference (src/model/argmax.cu:83-105; two
 * launches and a blocking copy per row) with the same selection rule
 * (src/model/argmax.cu:16-45): logits rounded to BF16, NaNs skipped, the
 * largest value wins with ties to the lowest index, and a row whose logit 0
 * is NaN selects 0.  d_logits: FP32 [rows][row_stride] (row_stride >= vocab);
 * d_tokens: int32 [rows], written on `stream`.  The workspace (at least
 * tvp_greedy_argmax_workspace_bytes(rows) bytes, 8-byte aligned, size a
 * multiple of 4) must be zeroed once before its first use; every call leaves
 * it zeroed, and one workspace serves calls of any row count up to what its
 * size allows (its per-row counters sit at fixed places from its end).  Calls
 * that share a workspace must not overlap on the GPU.
 */
size_t tvp_greedy_argmax_workspace_bytes(int rows);
int tvp_greedy_argmax(const float* d_logits, int rows, int vocab, long long row_stride,
                      int32_t* d_tokens, void* d_workspace, size_t workspace_bytes,
                      tvp_stream_t stream);

/*
 * K5 — the decode step's weight projections over 1-8 rows, several matrices
 * that share the input rows in one launch.
 *
 * Replaces the cublasGemmEx projections of the reference's decode step:
 * outputProjection / qProjection / kProjection / vProjection
 * (src/model/attention.cu:194-323), gateProjection / upProjection /
 * downProjection (src/model/mlp.cu:8-102) and lmHeadProjection
 * (src/model/lm_head.cu:8-36), called there once per row in decode.  Same
 * operands and math: for i < count,
 *     y[i][t][n] = sum_k w[i][n][k] x[t][k],   t < rows, n < n[i],
 * x: [rows][k] BF16; w[i]: [n[i]][k] BF16 (the reference's weight layout);
 * FP32 accumulation, the sum over k in a fixed order (results do not vary
 * from run to run).  `epilogue` says what is stored:
 *   TVP_PROJ_BF16      out[i] = bf16(y[i])                    [rows][n[i]] BF16
 *   TVP_PROJ_F32       out[i] = y[i]  (the LM head's logits)   [rows][n[i]] FP32
 *   TVP_PROJ_RESIDUAL  out[i] = out[i] + bf16(y[i]) as one BF16 add: the
 *                      projection followed by residualAdd
 *                      (src/model/resConnection.cu:6-17), bit for bit
 *   TVP_PROJ_SWIGLU    count = 2, n[0] = n[1]: out[0] =
 *                      bf16(g (1 / (1 + expf(-g))) u), g = bf16(y[0]),
 *                      u = bf16(y[1]): gate and up projections followed by
 *                      silu (src/model/SiLU.cu:5-16), bit for bit; out[1] is
 *                      not used (may be null)
 * w, n and out are HOST arrays of `count` (1..3) entries.  rows 1..8; k a
 * multiple of 256; every n[i] a multiple of 16; x and w[i] 16-byte aligned,
 * out[i] aligned to its element and not overlapping x.  No workspace, no
 * synchronisation: the launch goes on `stream`, as a programmatic dependent
 * launch that streams its first weights before it waits for the previous
 * kernel in the stream (it reads x and writes out only after that wait).
 */
#define TVP_PROJ_MAX 3
#define TVP_PROJ_BF16 0
#define TVP_PROJ_F32 1
#define TVP_PROJ_RESIDUAL 2
#define TVP_PROJ_SWIGLU 3
int tvp_decode_projections(const tvp_bf16* x, int rows, int k, int count, const tvp_bf16* const* w,
                           const int* n, void* const* out, int epilogue, tvp_stream_t stream);

/*
 * K5 with TVP_PROJ_RESIDUAL into the hidden rows, followed in the same launch
 * by the decode step's next RMSNorm: the O and down projections with their
 * residualAdd (src/model/resConnection.cu:6-17) and the rmsNormKernel launch
 * after each (src/model/paged_transformer.cu:68,103,116; src/model/rmsNorm.cu:
 * 3-22), bit for bit.  w: [2048][k]; hidden: [rows][2048] BF16 (updated in
 * place: hidden += bf16(w x)); then norm_out[t] = bf16((hidden[t] / r_t) g)
 * with r_t = sqrt(sum_i hidden[t][i]^2 / 2048 + 1e-5), the sum taken in the
 * reference kernel's order.  Each CTA sums the squares of its own features
 * as a subtree of the reference's tree and publishes it; once all 128 CTAs
 * have arrived, each normalises its own features.  d_scratch holds the
 * arrival counter (it grows by 128 per launch), an error word and the
 * subtree sums: TVP_NORM_SCRATCH_BYTES of device memory, 16-byte aligned,
 * zeroed once before first use.  The CTAs wait for one another, bounded by
 * 2 s, after which a CTA sets TVP_DEVERR_TIMEOUT in the error word (the int32
 * at d_scratch + 4) and leaves its norm outputs unwritten; on a device that
 * cannot hold all 128 CTAs at once the launch's last CTA computes the whole
 * norm instead.  rows 1..8, k a multiple of 256; x, w, hidden, norm_gain,
 * norm_out 16-byte aligned, norm_out and d_scratch overlapping none of x,
 * hidden, norm_gain.  Programmatic dependent launch, as
 * tvp_decode_projections.  Launches that share d_scratch must not overlap.
 */
#define TVP_NORM_SCRATCH_BYTES 4352
int tvp_decode_projection_residual_rmsnorm(const tvp_bf16* x, int rows, int k, const tvp_bf16* w,
                                           tvp_bf16* hidden, const tvp_bf16* norm_gain,
                                           tvp_bf16* norm_out, void* d_scratch,
                                           tvp_stream_t stream);

/*
 * K5's Q, K and V projections of one decode token per row, with K1's work in
 * the epilogue: the reference's qProjection, kProjection, vProjection
 * (src/model/attention.cu:194-323), ropeBatch of q and k (src/model/RoPe.cu:
 * 46-62) and storePagedKVBatch (src/model/paged_attention.cu:89-99,123-131)
 * in one launch, with tvp_rope_append's arithmetic bit for bit.  x: [rows][k]
 * BF16 (the normalised hidden rows); w_q [2048][k], w_k and w_v [512][k]
 * (32 query heads, 8 KV heads of 64).  Row t's token sits at position
 * d_positions[t] of block-table row t: q_out[t] gets its rotated q; its
 * rotated k and its v go into slot pos % 16 of page
 * d_block_tables[t * table_stride + pos / 16] of layer `layer` of the pools
 * (8 KV heads, the reference layout).  A bad position or page id sets
 * TVP_DEVERR_BAD_TOKEN / TVP_DEVERR_BAD_PAGE in *d_error and that store is
 * skipped.  rows 1..8, k a multiple of 256, x and weights 16-byte aligned.
 * Programmatic dependent launch, as tvp_decode_projections.
 */
int tvp_decode_qkv_rope_append(const tvp_bf16* x, int rows, int k, const tvp_bf16* w_q,
                               const tvp_bf16* w_k, const tvp_bf16* w_v, tvp_bf16* q_out,
                               tvp_bf16* k_pool, tvp_bf16* v_pool, int num_pages, int num_layers,
                               int layer, const int32_t* d_block_tables, int table_stride,
                               const int32_t* d_positions, int32_t* d_error, tvp_stream_t stream);

/*
 * tvp_decode_projection_residual_rmsnorm of the down projection followed by
 * tvp_decode_qkv_rope_append of the next layer, in one launch: the argument
 * groups are theirs (x, rows, k, w_down, hidden, norm_gain, norm_out,
 * d_scratch for the first; w_q, w_k, w_v, q_out, pools, layer, tables,
 * positions, d_error for the second, whose x is norm_out).  Every output has
 * the bits of the two launches.  After the grid-wide arrival of the norm
 * each CTA normalises all rows into shared memory, and its two halves of 8
 * warps run one Q/K/V item each, with weights loaded before the arrival.  k
 * a multiple of 512 above 4096 (the down projection's 8192), and a device
 * that holds all 128 CTAs of 16 warps at once (the spread norm); otherwise
 * TVP_ERR_UNSUPPORTED, and the caller makes the two launches.
 */
int tvp_decode_down_norm_qkv(const tvp_bf16* x, int rows, int k, const tvp_bf16* w_down,
                             tvp_bf16* hidden, const tvp_bf16* norm_gain, tvp_bf16* norm_out,
                             void* d_scratch, const tvp_bf16* w_q, const tvp_bf16* w_k,
                             const tvp_bf16* w_v, tvp_bf16* q_out, tvp_bf16* k_pool,
                             tvp_bf16* v_pool, int num_pages, int num_layers, int layer,
                             const int32_t* d_block_tables, int table_stride,
                             const int32_t* d_positions, int32_t* d_error, tvp_stream_t stream);

/*
 * K2 without any allocation.  This entry point has no counterpart in the
 * reference.  It is for callers that cannot call cudaMalloc: code whose
 * device memory is owned by a host framework's pool, plug-ins running under a
 * fixed memory budget, and threads that must not take the device-wide
 * synchronisation cudaMalloc/cudaFree can imply.  It runs tvp_decode_plan and
 * tvp_paged_decode_attention (FAST mode) on a workspace kept in a 4 MiB device
 * array inside this library; that array stays resident on every GPU that
 * loads the library until the process exits.  Inputs and outputs are the
 * caller's, exactly as for tvp_paged_decode_attention.
 *   - Returns TVP_ERR_WORKSPACE when batch and grid (num_ctas, 0 = one CTA per
 *     SM) need more than 4 MiB of workspace (with one CTA per SM of a B200:
 *     batches beyond 46,968 rows with 8 KV heads).
 *   - The first call on a device resolves the array's device address on that
 *     device (cudaGetSymbolAddress); make that first call before any stream
 *     capture.  The address is kept for the life of the process, so the entry
 *     point must not be used across cudaDeviceReset (the array may move).
 *   - Every argument check runs before anything is enqueued: a rejected call
 *     touches neither the array nor the error word.
 *   - Every call uses the same array: calls that can overlap on the GPU (other
 *     streams, other host threads on the same device) race and must be
 *     serialised by the caller.  Each call re-plans, so no state from an
 *     earlier call is read.
 */
int tvp_paged_decode_attention_noalloc(const tvp_bf16* q, const tvp_bf16* k_pool,
                                       const tvp_bf16* v_pool, int num_pages, int num_layers,
                                       int layer, int kv_heads, int q_heads,
                                       const int32_t* d_block_tables, int table_stride,
                                       const int32_t* d_seq_lens, int batch, float scale,
                                       int num_ctas, tvp_bf16* out, int32_t* d_error,
                                       tvp_stream_t stream);

/* ======================================================================= *
 * KV-head-sharded decode with the all-gather fused into the decode kernel.
 * No counterpart in the reference (its engine runs on one GPU); this is the
 * multi-GPU form of src/model/paged_transformer.cu:85-94 for long contexts:
 * GPU r of `world` (2, 4 or 8; one process per GPU) holds KV heads
 * [r K, (r + 1) K), K = 8 / world, of every page (pools of K x 64 channels,
 * the same block tables on every rank) and the [batch][2048] attention rows
 * end up on every rank.  The decode kernel stores each finished output group
 * straight into every rank's gathered rows over NVLink (peer memory opened
 * through CUDA IPC); its last CTA bumps every rank's flag and waits for all
 * ranks' signals.  Every rank makes the same calls in the same order (SPMD).
 * ======================================================================= */
#define TVP_IPC_HANDLE_BYTES 64
typedef struct tvp_head_gather tvp_head_gather;

/* This rank's gathered rows (two buffers of [max_batch][2048] BF16) and flag
 * words, zero-initialised, on the current device. */
int tvp_head_gather_create(int world, int rank, int kv_heads, int max_batch,
                           tvp_head_gather** out);
/* The IPC handle of this rank's allocation (TVP_IPC_HANDLE_BYTES bytes), to be
 * sent to every other rank (e.g. by an all-gather over the process group). */
int tvp_head_gather_export(const tvp_head_gather* g, void* handle_out);
/* Opens every other rank's allocation; handles = world x TVP_IPC_HANDLE_BYTES
 * in rank order (this rank's own entry is ignored).  Once per group. */
int tvp_head_gather_connect(tvp_head_gather* g, const void* handles);
/* Device address of this rank's gathered rows of buffer 0 or 1. */
int tvp_head_gather_rows(const tvp_head_gather* g, int buffer, tvp_bf16** rows_out);
/* FAST decode attention of this rank's heads (arguments as for
 * tvp_paged_decode_attention, kv_heads = 8 / world, no `out`), written into
 * every rank's gathered rows of `buffer`.  The launch ends once every rank's
 * rows of this call are in this rank's buffer: its last CTA waits for all
 * ranks' signals, bounded by 2 s, after which it sets TVP_DEVERR_TIMEOUT in
 * *d_error and ends (a rank that stopped never hangs the others; the group is
 * then unusable).  Alternate the buffers from one layer to the next: a rank
 * may start the next layer while another rank still reads this one's rows. */
int tvp_paged_decode_attention_gather(const tvp_bf16* q, const tvp_bf16* k_pool,
                                      const tvp_bf16* v_pool, int num_pages, int num_layers,
                                      int layer, int kv_heads, int q_heads,
                                      const int32_t* d_block_tables, int table_stride,
                                      const int32_t* d_seq_lens, int batch, float scale,
                                      int num_ctas, void* d_workspace, size_t workspace_bytes,
                                      tvp_head_gather* g, int buffer, int32_t* d_error,
                                      tvp_stream_t stream);
/* Teardown, in two steps on every rank: disconnect (waits for this device,
 * then closes the peers' allocations), a barrier across ranks, destroy (frees
 * this rank's allocation, which no peer maps any more).  Destroy alone also
 * disconnects, for a rank whose peers never connected. */
int tvp_head_gather_disconnect(tvp_head_gather* g);
int tvp_head_gather_destroy(tvp_head_gather* g);

/* ======================================================================= *
 * Host API mirror: PagedKVCache / SequenceKVState / PagedBatchMetadata.
 * Same allocator semantics as src/model/paged_kvcache.cu:37-117 (LIFO free
 * list seeded descending, lazy ceil(L/16) pages, exhaustion checked before
 * mutation, O(n) double-free rejection), with the 1024-token context cap
 * made a per-cache parameter (max_seq_len, 1024 reproduces the reference).
 * ======================================================================= */
typedef struct tvp_cache tvp_cache; /* PagedKVCache  (include/paged_kvcache.cuh:8-14) */
typedef struct tvp_seq tvp_seq;     /* SequenceKVState (include/paged_kvcache.cuh:16-19) */
typedef struct tvp_batch tvp_batch; /* PagedBatchMetadata (include/paged_attention.cuh:6-15) */

/* allocatePagedKVCache (src/model/paged_kvcache.cu:37-62).  device_storage=0
 * builds the allocator only (no pools), for host-side tests. */
int tvp_cache_create(int num_blocks, int num_layers, int kv_heads, int max_seq_len,
                     int device_storage, tvp_cache** out);
/* freePagedKVCache (src/model/paged_kvcache.cu:64-70). */
void tvp_cache_destroy(tvp_cache* cache);
int tvp_cache_pools(const tvp_cache* cache, tvp_bf16** k_pool, tvp_bf16** v_pool,
                    int* num_blocks);
int tvp_cache_free_count(const tvp_cache* cache);
/* Copies the free list (bottom..top of the LIFO stack); returns its length. */
int tvp_cache_free_list(const tvp_cache* cache, int32_t* out, int capacity);
/* Overwrites the free list (bottom..top); for seeded shuffled pools. */
int tvp_cache_set_free_list(tvp_cache* cache, const int32_t* blocks, int count);
/* allocatePhysicalBlock (src/model/paged_kvcache.cu:72-80). */
int tvp_allocate_physical_block(tvp_cache* cache, int* out_block);
/* freePhysicalBlock (src/model/paged_kvcache.cu:82-89). */
int tvp_free_physical_block(tvp_cache* cache, int block);

int tvp_seq_create(tvp_seq** out);
void tvp_seq_destroy(tvp_seq* seq);
int tvp_seq_length(const tvp_seq* seq);
int tvp_seq_set_length(tvp_seq* seq, int current_seq_len);
/* Copies the block table; returns its length. */
int tvp_seq_block_table(const tvp_seq* seq, int32_t* out, int capacity);
/* reserveSequenceBlocks (src/model/paged_kvcache.cu:100-117). */
int tvp_reserve_sequence_blocks(tvp_cache* cache, tvp_seq* seq, int total_seq_len);
/* freeSequenceBlocks (src/model/paged_kvcache.cu:91-98). */
int tvp_free_sequence_blocks(tvp_cache* cache, tvp_seq* seq);

/* storePagedKV (src/model/paged_kvcache.cu:119-139): reserve + append
 * num_tokens rows of k, v (device) at current_seq_len.. through K1; with
 * rope_q non-NULL the fused form also applies RoPE to k (in place) and q,
 * replacing rope(q), rope(k), storePagedKV of src/model/paged_transformer.cu:34-36. */
int tvp_store_paged_kv(tvp_cache* cache, tvp_seq* seq, int layer, tvp_bf16* k,
                       const tvp_bf16* v, int num_tokens, int apply_rope, tvp_bf16* rope_q,
                       tvp_stream_t stream);

/* PagedBatchMetadata with persistent device tables (no per-step malloc). */
int tvp_batch_create(int max_batch, int max_pages_per_seq, tvp_batch** out);
void tvp_batch_destroy(tvp_batch* batch);
/* preparePagedBatch (src/model/paged_attention.cu:30-87): validates the rows,
 * reserves the page of the new token, uploads tables / positions / lengths and
 * plans the decode grid. */
int tvp_prepare_paged_batch(tvp_cache* cache, tvp_seq* const* seqs, int count, tvp_batch* batch,
                            tvp_stream_t stream);
int tvp_batch_positions(const tvp_batch* batch, const int32_t** d_positions,
                        const int32_t** d_lengths, const int32_t** d_tables, int* table_stride);
/* ropeBatch(q) + ropeBatch(k) + storePagedKVBatch (src/model/paged_transformer.cu:80-84). */
int tvp_store_paged_kv_batch(tvp_cache* cache, const tvp_batch* batch, int layer, tvp_bf16* q,
                             tvp_bf16* k, const tvp_bf16* v, tvp_stream_t stream);
/* computePagedAttentionScores + softmaxRows + pagedAttentionScoresTimesV
 * (src/model/paged_transformer.cu:85-94) as one fused launch. */
int tvp_paged_attention(const tvp_cache* cache, tvp_batch* batch, int layer, const tvp_bf16* q,
                        tvp_bf16* out, int mode, tvp_stream_t stream);
/* Device error word of the batch's launches (synchronises the stream). */
int tvp_batch_error(tvp_batch* batch, tvp_stream_t stream, int32_t* out_bits);

#ifdef __cplusplus
}
#endif

#endif /* TVP_PAGED_H */
