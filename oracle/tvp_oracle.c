/*
 * tvp_oracle.c — TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * CPU restatement of the reference's paged-KV path, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg to check and to
 * time against; nothing in the vllm_b200 package links or calls it.
 *
 * Each function cites the reference code it restates (paths inside the
 * arpitsri28/vllm tree):
 *   orc_rope                 src/model/RoPe.cu:8-29 (ropeKernel), :31-62
 *   orc_store_paged          src/model/paged_kvcache.cu:119-139 (storePagedKV)
 *   orc_decode_attention     src/model/attention.cu:53-93 (scores), src/model/softmax.cu:6-45,
 *                            src/model/attention.cu:95-142 (P.V), driven as
 *                            src/model/paged_transformer.cu:85-94
 *   orc_decode_attention_f64 same maths in double without intermediate rounding
 *
 * Pinning: page placement is integer work and is exact.  RoPE calls the host
 * libm powf/cosf/sinf and is built with -ffp-contract=off, so it can differ
 * from the device kernel in the last FP32 bit and, rarely, by one BF16 ulp;
 * the tests bound that against golden vectors produced by the reference's own
 * kernel on a B200 (tests/golden/).  The FP32 dot products inside the cuBLAS
 * GEMVs of the reference have an unspecified order: here they are sequential.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_HEAD_DIM 64
#define ORC_PAGE 16
#define ORC_GROUP 4

float orc_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* float -> bfloat16, round to nearest even (NaN stays NaN). */
uint16_t orc_f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float round_bf16(float x) { return orc_bf16_to_f32(orc_f32_to_bf16(x)); }

void orc_f32_to_bf16_array(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_bf16(in[i]);
}

/* llama3-scaled inverse frequency, src/model/RoPe.cu:15-22. */
float orc_llama3_theta(int pair) {
  float theta = 1.0f / powf(500000.0f, (2.0f * pair) / ORC_HEAD_DIM);
  float wavelength = 6.283185307179586f / theta;
  if (wavelength > 8192.0f) {
    theta /= 32.0f;
  } else if (wavelength >= 2048.0f) {
    float smooth = (8192.0f / wavelength - 1.0f) / 3.0f;
    theta = (1.0f - smooth) * theta / 32.0f + smooth * theta;
  }
  return theta;
}

/* In-place RoPE of x[tokens][proj_dim]; token t sits at positions[t], or at
 * position_offset + t when positions is NULL (rope vs ropeBatch). */
void orc_rope(uint16_t* x, int tokens, int proj_dim, const int32_t* positions,
              int position_offset) {
  for (int t = 0; t < tokens; ++t) {
    const int position = positions ? positions[t] : position_offset + t;
    uint16_t* row = x + (size_t)t * proj_dim;
    for (int head = 0; head < proj_dim / ORC_HEAD_DIM; ++head) {
      for (int pair = 0; pair < ORC_HEAD_DIM / 2; ++pair) {
        const int xi = head * ORC_HEAD_DIM + pair, yi = xi + ORC_HEAD_DIM / 2;
        const float theta = orc_llama3_theta(pair);
        const float angle = position * theta;
        const float xf = orc_bf16_to_f32(row[xi]), yf = orc_bf16_to_f32(row[yi]);
        row[xi] = orc_f32_to_bf16(xf * cosf(angle) - yf * sinf(angle));
        row[yi] = orc_f32_to_bf16(xf * sinf(angle) + yf * cosf(angle));
      }
    }
  }
}

/* Element offset of (layer, physical page, slot) in a pool of rows of kv_dim,
 * src/model/paged_kvcache.cu:131. */
size_t orc_page_offset(int layer, int num_pages, int phys, int slot, int kv_dim) {
  return (((size_t)layer * num_pages + phys) * ORC_PAGE + slot) * (size_t)kv_dim;
}

/* storePagedKV: n rows of k, v appended from position `start` through `table`.
 * Returns -1 when a table entry is out of range (the reference throws). */
int orc_store_paged(uint16_t* k_pool, uint16_t* v_pool, int num_pages, int layer, int kv_dim,
                    const int32_t* table, int table_len, int start, int n, const uint16_t* k,
                    const uint16_t* v) {
  for (int token = 0; token < n; ++token) {
    const int pos = start + token;
    if (pos / ORC_PAGE >= table_len) return -1;
    const int phys = table[pos / ORC_PAGE];
    if (phys < 0 || phys >= num_pages) return -1;
    const size_t off = orc_page_offset(layer, num_pages, phys, pos % ORC_PAGE, kv_dim);
    memcpy(k_pool + off, k + (size_t)token * kv_dim, (size_t)kv_dim * 2);
    memcpy(v_pool + off, v + (size_t)token * kv_dim, (size_t)kv_dim * 2);
  }
  return 0;
}

/* One (row, KV head) of the reference decode attention.  s, e: scratch of 4*L. */
static void attend_group(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                         int num_pages, int layer, int kv_heads, const int32_t* table, int L,
                         float scale, int g, float* s, float* e, uint16_t* out) {
  const int kv_dim = kv_heads * ORC_HEAD_DIM;
  float qf[ORC_GROUP][ORC_HEAD_DIM];
  for (int h = 0; h < ORC_GROUP; ++h)
    for (int d = 0; d < ORC_HEAD_DIM; ++d)
      qf[h][d] = orc_bf16_to_f32(q[(g * ORC_GROUP + h) * ORC_HEAD_DIM + d]);
  /* scores, one page at a time, K transposed so the token loop vectorises
   * while each token keeps its sequential channel order */
  float kt[ORC_HEAD_DIM][ORC_PAGE];
  for (int t0 = 0; t0 < L; t0 += ORC_PAGE) {
    const int phys = table[t0 / ORC_PAGE];
    const int n = L - t0 < ORC_PAGE ? L - t0 : ORC_PAGE;
    for (int t = 0; t < ORC_PAGE; ++t)
      for (int d = 0; d < ORC_HEAD_DIM; ++d)
        kt[d][t] = t < n ? orc_bf16_to_f32(
                               k_pool[orc_page_offset(layer, num_pages, phys, t, kv_dim) +
                                      g * ORC_HEAD_DIM + d])
                         : 0.0f;
    for (int h = 0; h < ORC_GROUP; ++h) {
      float acc[ORC_PAGE];
      for (int t = 0; t < ORC_PAGE; ++t) acc[t] = 0.0f;
      for (int d = 0; d < ORC_HEAD_DIM; ++d)
        for (int t = 0; t < ORC_PAGE; ++t) acc[t] = acc[t] + qf[h][d] * kt[d][t];
      for (int t = 0; t < n; ++t) s[h * L + t0 + t] = round_bf16(scale * acc[t]);
    }
  }
  /* softmaxKernel per head row: exact max, expf, pairwise tree, BF16 output */
  for (int h = 0; h < ORC_GROUP; ++h) {
    float* sh = s + (size_t)h * L;
    float m = sh[0];
    for (int t = 1; t < L; ++t) m = fmaxf(m, sh[t]);
    for (int t = 0; t < L; ++t) e[t] = expf(sh[t] - m);
    for (int i = 1; i < L; i *= 2)
      for (int t = 0; t + i < L; t += 2 * i) e[t] = e[t] + e[t + i];
    const float sum = e[0];
    for (int t = 0; t < L; ++t) sh[t] = round_bf16(expf(sh[t] - m) / sum);
  }
  /* P.V with FP32 accumulation */
  for (int h = 0; h < ORC_GROUP; ++h) {
    float o[ORC_HEAD_DIM];
    for (int d = 0; d < ORC_HEAD_DIM; ++d) o[d] = 0.0f;
    for (int t = 0; t < L; ++t) {
      const float p = s[(size_t)h * L + t];
      const uint16_t* vrow = v_pool +
                             orc_page_offset(layer, num_pages, table[t / ORC_PAGE], t % ORC_PAGE,
                                             kv_dim) +
                             g * ORC_HEAD_DIM;
      for (int d = 0; d < ORC_HEAD_DIM; ++d) o[d] = o[d] + p * orc_bf16_to_f32(vrow[d]);
    }
    for (int d = 0; d < ORC_HEAD_DIM; ++d)
      out[(g * ORC_GROUP + h) * ORC_HEAD_DIM + d] = orc_f32_to_bf16(o[d]);
  }
}

/*
 * Reference decode attention for a batch: q [batch][kv_heads*4*64],
 * out [batch][kv_heads*4*64], tables [batch][table_stride], lens[b] = attended
 * length.  Rows with lens[b] <= 0 produce zeros.  threads <= 0: all cores.
 * Returns -1 on an out-of-range table entry.
 */
int orc_decode_attention(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                         int num_pages, int layer, int kv_heads, const int32_t* tables,
                         int table_stride, const int32_t* lens, int batch, float scale,
                         uint16_t* out, int threads) {
  const int qdim = kv_heads * ORC_GROUP * ORC_HEAD_DIM;
  for (int b = 0; b < batch; ++b) {
    if (lens[b] > table_stride * ORC_PAGE) return -1;
    for (int j = 0; j < (lens[b] + ORC_PAGE - 1) / ORC_PAGE; ++j) {
      const int phys = tables[(size_t)b * table_stride + j];
      if (phys < 0 || phys >= num_pages) return -1;
    }
  }
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(threads)
#endif
  for (int b = 0; b < batch; ++b) {
    for (int g = 0; g < kv_heads; ++g) {
      const int L = lens[b];
      uint16_t* o = out + (size_t)b * qdim;
      if (L <= 0) {
        memset(o + g * ORC_GROUP * ORC_HEAD_DIM, 0, ORC_GROUP * ORC_HEAD_DIM * 2);
        continue;
      }
      float* s = (float*)malloc(sizeof(float) * (size_t)ORC_GROUP * L);
      float* e = (float*)malloc(sizeof(float) * (size_t)L);
      attend_group(q + (size_t)b * qdim, k_pool, v_pool, num_pages, layer, kv_heads,
                   tables + (size_t)b * table_stride, L, scale, g, s, e, o);
      free(s);
      free(e);
    }
  }
  return 0;
}

/* Exact-arithmetic version: double throughout, no intermediate rounding; out in double. */
int orc_decode_attention_f64(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool,
                             int num_pages, int layer, int kv_heads, const int32_t* tables,
                             int table_stride, const int32_t* lens, int batch, double scale,
                             double* out, int threads) {
  const int kv_dim = kv_heads * ORC_HEAD_DIM;
  const int qdim = kv_heads * ORC_GROUP * ORC_HEAD_DIM;
  for (int b = 0; b < batch; ++b) {
    if (lens[b] > table_stride * ORC_PAGE) return -1;
    for (int j = 0; j < (lens[b] + ORC_PAGE - 1) / ORC_PAGE; ++j) {
      const int phys = tables[(size_t)b * table_stride + j];
      if (phys < 0 || phys >= num_pages) return -1;
    }
  }
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for collapse(2) schedule(dynamic, 1) num_threads(threads)
#endif
  for (int b = 0; b < batch; ++b) {
    for (int hq = 0; hq < kv_heads * ORC_GROUP; ++hq) {
      const int L = lens[b], g = hq / ORC_GROUP;
      double* o = out + (size_t)b * qdim + (size_t)hq * ORC_HEAD_DIM;
      for (int d = 0; d < ORC_HEAD_DIM; ++d) o[d] = 0.0;
      if (L <= 0) continue;
      const int32_t* table = tables + (size_t)b * table_stride;
      const uint16_t* qh = q + (size_t)b * qdim + (size_t)hq * ORC_HEAD_DIM;
      double* sc = (double*)malloc(sizeof(double) * (size_t)L);
      double m = -INFINITY;
      for (int t = 0; t < L; ++t) {
        const uint16_t* krow =
            k_pool + orc_page_offset(layer, num_pages, table[t / ORC_PAGE], t % ORC_PAGE, kv_dim) +
            g * ORC_HEAD_DIM;
        double acc = 0.0;
        for (int d = 0; d < ORC_HEAD_DIM; ++d)
          acc += (double)orc_bf16_to_f32(qh[d]) * (double)orc_bf16_to_f32(krow[d]);
        sc[t] = scale * acc;
        if (sc[t] > m) m = sc[t];
      }
      double sum = 0.0;
      for (int t = 0; t < L; ++t) {
        sc[t] = exp(sc[t] - m);
        sum += sc[t];
      }
      for (int t = 0; t < L; ++t) {
        const uint16_t* vrow =
            v_pool + orc_page_offset(layer, num_pages, table[t / ORC_PAGE], t % ORC_PAGE, kv_dim) +
            g * ORC_HEAD_DIM;
        const double p = sc[t] / sum;
        for (int d = 0; d < ORC_HEAD_DIM; ++d) o[d] += p * (double)orc_bf16_to_f32(vrow[d]);
      }
      free(sc);
    }
  }
  return 0;
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
