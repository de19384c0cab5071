/*
 * rpg_oracle.c -- CPU restatement of the RPGBarEngine token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * path: only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load it, and only to check or to time a CPU baseline.  Nothing in the
 * product (rpgbarengine_b200/) links, loads or calls it.
 *
 * What it restates, operation for operation, is the reference's SCALAR path
 * (the one the reference selects with RPGBAR_NO_SIMD=1):
 *   - fp16 <-> fp32                       src/dtypes.h:21-76
 *   - ggml block geometry                 src/quant.cc:29-45, 371-414
 *   - DequantizeRow (F32/F16/Q8_0/Q4_K/Q6_K)
 *                                         src/quant.cc:126-136, 207-217, 233-242,
 *                                         327-354, 396-429
 *   - DotRowQuantRef (4 strided partial sums, (s0+s1)+(s2+s3))
 *                                         src/matmul.cc:73-102
 *   - QuantMatrix::MatMulBatch (per (t,r) dot, scalar backend)
 *                                         src/model.cc:39-69
 *   - Dot / ArgMax / RmsNorm / SoftmaxInPlace / SiluInPlace / RopeInPlace
 *                                         src/kernels.h:26-120
 *   - BuildRopeTable                      src/model.cc:122-145
 *   - ForwardLayer / ForwardFull / CausalAttention / AttentionFromCache
 *                                         src/qwen3.cc:44-290
 *   - Generate                            src/qwen3.cc:302-355
 *   - SplitMix64 / CounterRng / CounterUniform / FilterToProbs / SampleToken
 *                                         src/sampler.cc:16-112
 *   - KvCache layout ((l*nkv+h)*max_seq+pos)*hd, fp32, zero-init
 *                                         src/kv_cache.h:35-82, src/kv_cache.cc:29-33
 *
 * Build rules that keep it bit-identical to the reference scalar path:
 * -O2 -ffp-contract=off, no -march/-mfma (the reference's non-AVX2 TUs are
 * built for baseline x86-64, so none of their float ops are contracted), and
 * the same float/double promotion points as the reference source.  OpenMP
 * only splits independent outputs (matrix rows, attention heads), so every
 * output keeps its serial accumulation order and results do not depend on
 * the thread count.
 *
 * One documented divergence: the reference's top-p sort is std::sort
 * (unstable), so among exactly-equal probabilities its order is unspecified;
 * here ties are broken by token index.  Only exact probability ties that
 * straddle the top-p cut can be affected.
 */
#include <math.h>
#include <stdio.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_F32 0u
#define ORC_F16 1u
#define ORC_Q8_0 8u
#define ORC_Q4_K 12u
#define ORC_Q6_K 14u

/* ------------------------------------------------------------------ dtypes */

/* src/dtypes.h:21-47: exact half -> float, subnormals normalised by hand. */
float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t out;
  if (exp == 0) {
    if (man == 0) {
      out = sign;
    } else {
      exp = 113; /* 127 - 15 + 1 */
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      man &= 0x3FFu;
      out = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    out = sign | 0x7F800000u | (man << 13);
  } else {
    out = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float v;
  memcpy(&v, &out, 4);
  return v;
}

/* src/dtypes.h:50-76: float -> half, round to nearest even. */
uint16_t orc_f32_to_f16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  const int32_t exp = (int32_t)((u >> 23) & 0xFFu) - 127 + 15;
  const uint32_t man = u & 0x7FFFFFu;
  if (((u >> 23) & 0xFFu) == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    uint32_t m = (man | 0x800000u) >> (1 - exp);
    m = (m + 0x1000u) >> 13;
    return (uint16_t)(sign | m);
  }
  uint32_t rounded = man + 0x1000u;
  uint32_t e = (uint32_t)exp;
  if (rounded & 0x800000u) {
    rounded = 0;
    ++e;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  }
  return (uint16_t)(sign | (e << 10) | (rounded >> 13));
}

static inline float half_at(const uint8_t* p) {
  uint16_t v;
  memcpy(&v, p, 2);
  return orc_f16_to_f32(v);
}

/* -------------------------------------------------------- block geometry */

/* src/quant.cc:29-45 (the in-scope rows of the type table). */
int orc_type_block(uint32_t type, int64_t* elems, int64_t* bytes) {
  switch (type) {
    case ORC_F32: *elems = 1; *bytes = 4; return 0;
    case ORC_F16: *elems = 1; *bytes = 2; return 0;
    case ORC_Q8_0: *elems = 32; *bytes = 34; return 0;
    case ORC_Q4_K: *elems = 256; *bytes = 144; return 0;
    case ORC_Q6_K: *elems = 256; *bytes = 210; return 0;
    default: return -1;
  }
}

/* src/quant.cc:405-414. Returns -1 when n is not a whole number of blocks. */
int64_t orc_row_bytes(uint32_t type, int64_t n) {
  int64_t be, bb;
  if (orc_type_block(type, &be, &bb) != 0) return -1;
  if (n % be != 0) return -1;
  return (n / be) * bb;
}

/* ------------------------------------------------------------- dequant */

/* src/quant.cc:233-242 (ggml get_scale_min_k4). */
static inline void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
  if (j < 4) {
    *d = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *d = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
    *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

/* src/quant.cc:207-217: y = q * d. */
static void deq_q8_0(const uint8_t* src, int64_t n, float* dst) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* p = src + b * 34;
    const float d = half_at(p);
    const int8_t* qs = (const int8_t*)(p + 2);
    for (int j = 0; j < 32; ++j) dst[b * 32 + j] = (float)qs[j] * d;
  }
}

/* src/quant.cc:327-354: per 64-group, y = (d*sc)*q - (dmin*m). */
static void deq_q4_k(const uint8_t* src, int64_t n, float* dst) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* p = src + b * 144;
    const float d = half_at(p + 0);
    const float dmin = half_at(p + 2);
    const uint8_t* scales = p + 4;
    const uint8_t* q = p + 16;
    float* y = dst + b * 256;
    for (int g = 0; g < 4; ++g) {
      uint8_t sc, m;
      scale_min_k4(2 * g, scales, &sc, &m);
      const float d1 = d * (float)sc;
      const float m1 = dmin * (float)m;
      scale_min_k4(2 * g + 1, scales, &sc, &m);
      const float d2 = d * (float)sc;
      const float m2 = dmin * (float)m;
      for (int l = 0; l < 32; ++l) *y++ = d1 * (float)(q[l] & 0x0F) - m1;
      for (int l = 0; l < 32; ++l) *y++ = d2 * (float)(q[l] >> 4) - m2;
      q += 32;
    }
  }
}

/* src/quant.cc:396-429: y = (d*sc[int8]) * (6-bit q - 32), 16-element scales. */
static void deq_q6_k(const uint8_t* src, int64_t n, float* dst) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* p = src + b * 210;
    const uint8_t* ql = p;
    const uint8_t* qh = p + 128;
    const int8_t* sc = (const int8_t*)(p + 192);
    const float d = half_at(p + 208);
    float* y = dst + b * 256;
    for (int half = 0; half < 2; ++half) {
      for (int l = 0; l < 32; ++l) {
        const int is = l / 16;
        const int q1 = (int)((ql[l] & 0x0F) | (((qh[l] >> 0) & 3) << 4)) - 32;
        const int q2 = (int)((ql[l + 32] & 0x0F) | (((qh[l] >> 2) & 3) << 4)) - 32;
        const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
        const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
        y[l + 0] = d * (float)sc[is + 0] * (float)q1;
        y[l + 32] = d * (float)sc[is + 2] * (float)q2;
        y[l + 64] = d * (float)sc[is + 4] * (float)q3;
        y[l + 96] = d * (float)sc[is + 6] * (float)q4;
      }
      y += 128;
      ql += 64;
      qh += 32;
      sc += 8;
    }
  }
}

/* src/quant.cc:416-436 (DequantizeRow). Returns -1 for unsupported types. */
int orc_dequantize_row(uint32_t type, const uint8_t* src, int64_t n, float* dst) {
  if (orc_row_bytes(type, n) < 0) return -1;
  switch (type) {
    case ORC_F32: memcpy(dst, src, (size_t)n * 4); return 0;
    case ORC_F16:
      for (int64_t i = 0; i < n; ++i) dst[i] = half_at(src + i * 2);
      return 0;
    case ORC_Q8_0: deq_q8_0(src, n, dst); return 0;
    case ORC_Q4_K: deq_q4_k(src, n, dst); return 0;
    case ORC_Q6_K: deq_q6_k(src, n, dst); return 0;
    default: return -1;
  }
}

/* ----------------------------------------------------------- dot / matmul */

/* src/matmul.cc:73-102: dequantise one block to the stack, 4 strided partial
 * sums over the block (tail into s0), result (s0+s1)+(s2+s3). */
float orc_dot_row(uint32_t type, const float* a, const uint8_t* w, int64_t k) {
  float tmp[256];
  int64_t be, bb;
  if (orc_type_block(type, &be, &bb) != 0 || k % be != 0) return NAN;
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  const int64_t nb = k / be;
  for (int64_t b = 0; b < nb; ++b) {
    orc_dequantize_row(type, w + b * bb, be, tmp);
    const float* ap = a + b * be;
    int64_t j = 0;
    const int64_t lim = be - 3;
    for (; j < lim; j += 4) {
      s0 += ap[j] * tmp[j];
      s1 += ap[j + 1] * tmp[j + 1];
      s2 += ap[j + 2] * tmp[j + 2];
      s3 += ap[j + 3] * tmp[j + 3];
    }
    for (; j < be; ++j) s0 += ap[j] * tmp[j];
  }
  return (s0 + s1) + (s2 + s3);
}

/* Float64 reference for the per-row error gate: returns sum(a*w) in double and
 * writes sum(|a*w|) (the gate's denominator) to *abs_sum. */
double orc_dot_row_f64(uint32_t type, const float* a, const uint8_t* w, int64_t k,
                       double* abs_sum) {
  float* tmp = (float*)malloc((size_t)k * sizeof(float));
  if (!tmp || orc_dequantize_row(type, w, k, tmp) != 0) {
    free(tmp);
    return NAN;
  }
  double s = 0.0, sa = 0.0;
  for (int64_t i = 0; i < k; ++i) {
    const double p = (double)a[i] * (double)tmp[i];
    s += p;
    sa += fabs(p);
  }
  free(tmp);
  if (abs_sum) *abs_sum = sa;
  return s;
}

/* src/model.cc:39-69 with the scalar backend: OUT[t*rows+r] = dot(X[t], W[r]).
 * Split over rows; each output keeps its serial order. */
int orc_matmul(uint32_t type, const uint8_t* w, int64_t rows, int64_t cols,
               const float* X, int64_t n, float* OUT) {
  const int64_t rb = orc_row_bytes(type, cols);
  if (rb < 0) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t t = 0; t < n; ++t) {
      OUT[t * rows + r] = orc_dot_row(type, X + t * cols, w + r * rb, cols);
    }
  }
  return 0;
}

/* ------------------------------------------------------------ vector ops */

/* src/kernels.h:26-38 */
static float dot4(const float* a, const float* b, int64_t n) {
  float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
  int64_t i = 0;
  const int64_t lim = n - 3;
  for (; i < lim; i += 4) {
    s0 += a[i] * b[i];
    s1 += a[i + 1] * b[i + 1];
    s2 += a[i + 2] * b[i + 2];
    s3 += a[i + 3] * b[i + 3];
  }
  for (; i < n; ++i) s0 += a[i] * b[i];
  return (s0 + s1) + (s2 + s3);
}

/* src/kernels.h:42-52: first index of the maximum (strict >). */
int32_t orc_argmax(const float* x, int64_t n) {
  int32_t best = 0;
  float bv = x[0];
  for (int64_t i = 1; i < n; ++i) {
    if (x[i] > bv) {
      bv = x[i];
      best = (int32_t)i;
    }
  }
  return best;
}

/* src/kernels.h:56-63: sum of squares in double, scale rounded to float,
 * out = (x*scale)*w.  In-place (out == x) is allowed. */
void orc_rmsnorm(const float* x, const float* w, int64_t n, float eps, float* out) {
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) sum += (double)x[i] * x[i];
  const double mean = sum / (double)n;
  const float scale = (float)(1.0 / sqrt(mean + eps));
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] * scale * w[i];
}

/* src/kernels.h:66-79: max-subtracted exp, double sum, float reciprocal. */
static void softmax_inplace(float* x, int64_t n) {
  if (n <= 0) return;
  float mx = x[0];
  for (int64_t i = 1; i < n; ++i)
    if (x[i] > mx) mx = x[i];
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const float e = expf(x[i] - mx);
    x[i] = e;
    sum += e;
  }
  const float inv = (float)(1.0 / sum);
  for (int64_t i = 0; i < n; ++i) x[i] *= inv;
}

/* src/kernels.h:108-120: half-split pairs (i, i+hd/2). */
static void rope_inplace(float* x, int32_t n_heads, int32_t hd, const float* c,
                         const float* s) {
  const int32_t half = hd / 2;
  for (int32_t h = 0; h < n_heads; ++h) {
    float* xh = x + (int64_t)h * hd;
    for (int32_t i = 0; i < half; ++i) {
      const float a = xh[i], b = xh[i + half];
      xh[i] = a * c[i] - b * s[i];
      xh[i + half] = b * c[i] + a * s[i];
    }
  }
}

/* -------------------------------------------------------------- sampler */

/* src/sampler.cc:16-22 */
uint64_t orc_splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

/* src/sampler.cc:24-34: u = top 24 bits of SplitMix64(seed + phi*counter). */
float orc_counter_uniform(uint64_t seed, uint64_t counter) {
  const uint32_t bits = (uint32_t)(orc_splitmix64(seed + 0x9E3779B97F4A7C15ull * counter) >> 40);
  return (float)bits * (1.0f / 16777216.0f);
}

static int cmp_desc_f32(const void* a, const void* b) {
  const float x = *(const float*)a, y = *(const float*)b;
  return (x < y) - (x > y);
}

static const float* g_sort_keys; /* only used under a single-threaded qsort */
static int cmp_asc_idx(const void* a, const void* b) {
  const int32_t i = *(const int32_t*)a, j = *(const int32_t*)b;
  const float x = g_sort_keys[i], y = g_sort_keys[j];
  if (x < y) return -1;
  if (x > y) return 1;
  return (i > j) - (i < j);
}

/* src/sampler.cc:36-94: temperature -> top-k (keep >= k-th, only when
 * 1 < k < n) -> softmax -> top-p (ascending double cumsum, zero while
 * cum <= 1-p, keep the largest) -> renormalise.  probs has n floats. */
int orc_filter_to_probs(const float* logits, int64_t n, float temperature, int32_t top_k,
                        float top_p, float* probs) {
  memcpy(probs, logits, (size_t)n * sizeof(float));
  float* s = probs;
  if (!(temperature > 0.0f)) {
    const int32_t best = orc_argmax(s, n);
    for (int64_t i = 0; i < n; ++i) s[i] = 0.0f;
    s[best] = 1.0f;
    return 0;
  }
  if (temperature != 1.0f) {
    const float inv = 1.0f / temperature;
    for (int64_t i = 0; i < n; ++i) s[i] *= inv;
  }
  if (top_k > 1 && top_k < n) {
    float* tmp = (float*)malloc((size_t)n * sizeof(float));
    if (!tmp) return -1;
    memcpy(tmp, s, (size_t)n * sizeof(float));
    qsort(tmp, (size_t)n, sizeof(float), cmp_desc_f32);
    const float kth = tmp[top_k - 1];
    free(tmp);
    for (int64_t i = 0; i < n; ++i)
      if (s[i] < kth) s[i] = -INFINITY;
  }
  softmax_inplace(s, n);
  if (top_p > 0.0f && top_p < 1.0f) {
    int32_t* asc = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    if (!asc) return -1;
    for (int64_t i = 0; i < n; ++i) asc[i] = (int32_t)i;
    g_sort_keys = s;
    qsort(asc, (size_t)n, sizeof(int32_t), cmp_asc_idx);
    const double threshold = 1.0 - (double)top_p;
    double cum = 0.0;
    for (int64_t j = 0; j < n; ++j) {
      cum += (double)s[asc[j]];
      if (cum <= threshold) s[asc[j]] = 0.0f;
    }
    if (n > 0 && s[asc[n - 1]] == 0.0f) s[asc[n - 1]] = 1.0f;
    free(asc);
    double sum = 0.0;
    for (int64_t i = 0; i < n; ++i) sum += (double)s[i];
    if (sum > 0.0) {
      const float inv = (float)(1.0 / sum);
      for (int64_t i = 0; i < n; ++i) s[i] *= inv;
    }
  }
  return 0;
}

/* src/sampler.cc:96-112: index-order inverse CDF with a double cumsum. */
int32_t orc_sample_token(const float* logits, int64_t n, float temperature, int32_t top_k,
                         float top_p, float u) {
  if (!(temperature > 0.0f)) return orc_argmax(logits, n);
  float* probs = (float*)malloc((size_t)n * sizeof(float));
  if (!probs) return -1;
  orc_filter_to_probs(logits, n, temperature, top_k, top_p, probs);
  double cum = 0.0;
  int32_t pick = -1;
  for (int64_t i = 0; i < n; ++i) {
    cum += (double)probs[i];
    if (cum > (double)u) {
      pick = (int32_t)i;
      break;
    }
  }
  if (pick < 0) pick = orc_argmax(probs, n);
  free(probs);
  return pick;
}

/* ----------------------------------------------------------------- model */

typedef struct {
  int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  int32_t context_length, max_pos;
  float rope_theta, rms_eps;
} orc_config;

/* One tensor of a GGUF-style table: dims[0] is the fastest axis. */
typedef struct {
  const char* name;
  uint32_t type;
  int32_t n_dims;
  int64_t dims[4];
  const void* data;
  int64_t n_bytes;
} orc_tensor;

typedef struct {
  uint32_t type;
  int64_t rows, cols;
  const uint8_t* data;
} orc_matrix;

typedef struct {
  const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
  orc_matrix q, k, v, o, gate, up, down;
} orc_layer;

typedef struct {
  orc_config c;
  orc_matrix token_embd, lm_head;
  const float* output_norm;
  orc_layer* layers;
  float* rope; /* [n_rope_pos][hd/2 cos | hd/2 sin] */
  int64_t n_rope_pos;
  float** owned_norms;
  int n_owned;
} orc_model;

typedef struct {
  int32_t n_layers, n_kv_heads, head_dim;
  int64_t max_seq, len;
  float* k;
  float* v;
} orc_kv;

static const orc_tensor* find_tensor(const orc_tensor* t, int n, const char* name) {
  for (int i = 0; i < n; ++i)
    if (strcmp(t[i].name, name) == 0) return &t[i];
  return NULL;
}

static int take_matrix(const orc_tensor* t, int64_t rows, int64_t cols, orc_matrix* m) {
  if (!t || t->n_dims != 2 || t->dims[1] != rows || t->dims[0] != cols) return -1;
  if (orc_row_bytes(t->type, cols) < 0) return -1;
  m->type = t->type;
  m->rows = rows;
  m->cols = cols;
  m->data = (const uint8_t*)t->data;
  return 0;
}

/* src/model.cc:99-120: norms become f32 copies (dequantised if needed). */
static const float* take_norm(orc_model* m, const orc_tensor* t, int64_t n) {
  if (!t || t->n_dims != 1 || t->dims[0] != n) return NULL;
  float* buf = (float*)malloc((size_t)n * sizeof(float));
  if (!buf) return NULL;
  if (orc_dequantize_row(t->type, (const uint8_t*)t->data, n, buf) != 0) {
    free(buf);
    return NULL;
  }
  m->owned_norms[m->n_owned++] = buf;
  return buf;
}

void orc_model_free(orc_model* m) {
  if (!m) return;
  for (int i = 0; i < m->n_owned; ++i) free(m->owned_norms[i]);
  free(m->owned_norms);
  free(m->layers);
  free(m->rope);
  free(m);
}

/* src/model.cc:122-145: angles in double, cos/sin rounded to float. */
static int build_rope(orc_model* m) {
  const int32_t hd = m->c.head_dim, half = hd / 2;
  int64_t np = m->c.max_pos > m->c.context_length ? m->c.context_length : m->c.max_pos;
  if (np <= 0) np = 1;
  m->n_rope_pos = np;
  m->rope = (float*)calloc((size_t)np * half * 2, sizeof(float));
  double* inv = (double*)malloc((size_t)half * sizeof(double));
  if (!m->rope || !inv) {
    free(inv);
    return -1;
  }
  for (int32_t i = 0; i < half; ++i)
    inv[i] = 1.0 / pow((double)m->c.rope_theta, (double)(2 * i) / (double)hd);
  for (int64_t p = 0; p < np; ++p) {
    float* row = m->rope + p * half * 2;
    for (int32_t i = 0; i < half; ++i) {
      const double ang = (double)p * inv[i];
      row[i] = (float)cos(ang);
      row[half + i] = (float)sin(ang);
    }
  }
  free(inv);
  return 0;
}

/* src/model.cc:147-281 minus the GGUF/tokenizer side: shape-checked views,
 * tied lm_head when output.weight is absent.  Tensor memory stays owned by the
 * caller.  Returns NULL on any missing tensor or shape mismatch. */
orc_model* orc_model_create(const orc_config* cfg, const orc_tensor* t, int n) {
  orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
  if (!m) return NULL;
  m->c = *cfg;
  const orc_config* c = &m->c;
  const int64_t qd = (int64_t)c->n_heads * c->head_dim, kvd = (int64_t)c->n_kv_heads * c->head_dim;
  m->owned_norms = (float**)calloc((size_t)(4 * c->n_layers + 1), sizeof(float*));
  m->layers = (orc_layer*)calloc((size_t)c->n_layers, sizeof(orc_layer));
  if (!m->owned_norms || !m->layers) goto fail;
  if (take_matrix(find_tensor(t, n, "token_embd.weight"), c->vocab, c->hidden, &m->token_embd))
    goto fail;
  {
    const orc_tensor* out = find_tensor(t, n, "output.weight");
    if (out) {
      if (take_matrix(out, c->vocab, c->hidden, &m->lm_head)) goto fail;
    } else {
      m->lm_head = m->token_embd;
    }
  }
  if (!(m->output_norm = take_norm(m, find_tensor(t, n, "output_norm.weight"), c->hidden)))
    goto fail;
  for (int32_t l = 0; l < c->n_layers; ++l) {
    orc_layer* w = &m->layers[l];
    char nm[96];
#define ORC_T(suffix) (snprintf(nm, sizeof(nm), "blk.%d.%s", l, suffix), find_tensor(t, n, nm))
    if (!(w->attn_norm = take_norm(m, ORC_T("attn_norm.weight"), c->hidden))) goto fail;
    if (!(w->ffn_norm = take_norm(m, ORC_T("ffn_norm.weight"), c->hidden))) goto fail;
    if (!(w->q_norm = take_norm(m, ORC_T("attn_q_norm.weight"), c->head_dim))) goto fail;
    if (!(w->k_norm = take_norm(m, ORC_T("attn_k_norm.weight"), c->head_dim))) goto fail;
    if (take_matrix(ORC_T("attn_q.weight"), qd, c->hidden, &w->q)) goto fail;
    if (take_matrix(ORC_T("attn_k.weight"), kvd, c->hidden, &w->k)) goto fail;
    if (take_matrix(ORC_T("attn_v.weight"), kvd, c->hidden, &w->v)) goto fail;
    if (take_matrix(ORC_T("attn_output.weight"), c->hidden, qd, &w->o)) goto fail;
    if (take_matrix(ORC_T("ffn_gate.weight"), c->intermediate, c->hidden, &w->gate)) goto fail;
    if (take_matrix(ORC_T("ffn_up.weight"), c->intermediate, c->hidden, &w->up)) goto fail;
    if (take_matrix(ORC_T("ffn_down.weight"), c->hidden, c->intermediate, &w->down)) goto fail;
#undef ORC_T
  }
  if (build_rope(m)) goto fail;
  return m;
fail:
  orc_model_free(m);
  return NULL;
}

int64_t orc_model_rope_positions(const orc_model* m) { return m->n_rope_pos; }
const float* orc_model_rope_table(const orc_model* m) { return m->rope; }

/* src/kv_cache.cc:5-27: zero-initialised fp32 K and V. */
orc_kv* orc_kv_create(const orc_model* m, int64_t max_seq) {
  orc_kv* kv = (orc_kv*)calloc(1, sizeof(orc_kv));
  if (!kv || max_seq <= 0) {
    free(kv);
    return NULL;
  }
  kv->n_layers = m->c.n_layers;
  kv->n_kv_heads = m->c.n_kv_heads;
  kv->head_dim = m->c.head_dim;
  kv->max_seq = max_seq;
  const size_t per = (size_t)kv->n_layers * kv->n_kv_heads * (size_t)max_seq * kv->head_dim;
  kv->k = (float*)calloc(per, sizeof(float));
  kv->v = (float*)calloc(per, sizeof(float));
  if (!kv->k || !kv->v) {
    free(kv->k);
    free(kv->v);
    free(kv);
    return NULL;
  }
  return kv;
}

void orc_kv_free(orc_kv* kv) {
  if (!kv) return;
  free(kv->k);
  free(kv->v);
  free(kv);
}

int64_t orc_kv_len(const orc_kv* kv) { return kv->len; }
int orc_kv_set_len(orc_kv* kv, int64_t n) {
  if (n < 0 || n > kv->max_seq) return -1;
  kv->len = n;
  return 0;
}
/* Raw cache views for tests: [n_layers][n_kv][max_seq][hd]. */
const float* orc_kv_k(const orc_kv* kv) { return kv->k; }
const float* orc_kv_v(const orc_kv* kv) { return kv->v; }

static inline int64_t kv_off(const orc_kv* kv, int32_t l, int32_t h, int64_t pos) {
  return (((int64_t)l * kv->n_kv_heads + h) * kv->max_seq + pos) * kv->head_dim;
}

typedef struct {
  float *x, *h, *q, *k, *v, *attn, *proj, *gate, *up;
} scratch_t;

/* src/qwen3.cc:44-77 (no cache) and :79-117 (from cache).  Heads are
 * independent, so they are split across threads. */
static void attention(const orc_config* c, const float* q, int64_t seq, int64_t pos0,
                      const float* kseq, const float* vseq, const orc_kv* kv, int32_t layer,
                      float* out) {
  const int32_t nh = c->n_heads, nkv = c->n_kv_heads, hd = c->head_dim;
  const int32_t group = nh / nkv;
  const float scale = 1.0f / sqrtf((float)hd);
  const int64_t q_stride = (int64_t)nh * hd, kv_stride = (int64_t)nkv * hd;
  const int64_t max_len = pos0 + seq;
  memset(out, 0, (size_t)seq * q_stride * sizeof(float));
#pragma omp parallel for schedule(dynamic)
  for (int32_t h = 0; h < nh; ++h) {
    float* scores = (float*)malloc((size_t)max_len * sizeof(float));
    const int32_t kh = h / group;
    for (int64_t t = 0; t < seq; ++t) {
      const int64_t pos = pos0 + t;
      const float* qt = q + t * q_stride + (int64_t)h * hd;
      for (int64_t s = 0; s <= pos; ++s) {
        const float* ks = kv ? kv->k + kv_off(kv, layer, kh, s) : kseq + s * kv_stride + (int64_t)kh * hd;
        scores[s] = dot4(qt, ks, hd) * scale;
      }
      softmax_inplace(scores, pos + 1);
      float* ot = out + t * q_stride + (int64_t)h * hd;
      for (int64_t s = 0; s <= pos; ++s) {
        const float* vs = kv ? kv->v + kv_off(kv, layer, kh, s) : vseq + s * kv_stride + (int64_t)kh * hd;
        const float p = scores[s];
        for (int32_t d = 0; d < hd; ++d) ot[d] += p * vs[d];
      }
    }
    free(scores);
  }
}

/* src/qwen3.cc:79-117 for one query token at position pos over one layer's
 * cache [nkv][max_seq][hd]: scores = dot(q, K[s]) * (1/sqrt(hd)) for s <= pos,
 * softmax (double sum), out = sum_s p_s V[s] accumulated in float. */
int orc_attention_one(const float* q, const float* kc, const float* vc, int64_t max_seq,
                      int32_t nh, int32_t nkv, int32_t hd, int64_t pos, float* out) {
  if (nh <= 0 || nkv <= 0 || nh % nkv || pos < 0 || pos >= max_seq) return -1;
  const int32_t group = nh / nkv;
  const float scale = 1.0f / sqrtf((float)hd);
  float* scores = (float*)malloc((size_t)(pos + 1) * sizeof(float));
  if (!scores) return -1;
  for (int32_t h = 0; h < nh; ++h) {
    const float* kb = kc + (int64_t)(h / group) * max_seq * hd;
    const float* vb = vc + (int64_t)(h / group) * max_seq * hd;
    const float* qh = q + (int64_t)h * hd;
    for (int64_t s = 0; s <= pos; ++s) scores[s] = dot4(qh, kb + s * hd, hd) * scale;
    softmax_inplace(scores, pos + 1);
    float* oh = out + (int64_t)h * hd;
    for (int32_t d = 0; d < hd; ++d) oh[d] = 0.0f;
    for (int64_t s = 0; s <= pos; ++s) {
      const float p = scores[s];
      for (int32_t d = 0; d < hd; ++d) oh[d] += p * vb[s * hd + d];
    }
  }
  free(scores);
  return 0;
}

/* src/qwen3.cc:119-206 */
static void forward_layer(const orc_model* m, const orc_layer* w, int32_t layer, int64_t pos0,
                          scratch_t* s, int64_t seq, orc_kv* kv) {
  const orc_config* c = &m->c;
  const int64_t H = c->hidden, F = c->intermediate;
  const int32_t hd = c->head_dim, half = hd / 2;
  const int64_t qd = (int64_t)c->n_heads * hd, kvd = (int64_t)c->n_kv_heads * hd;
  for (int64_t t = 0; t < seq; ++t) orc_rmsnorm(s->x + t * H, w->attn_norm, H, c->rms_eps, s->h + t * H);
  orc_matmul(w->q.type, w->q.data, w->q.rows, w->q.cols, s->h, seq, s->q);
  orc_matmul(w->k.type, w->k.data, w->k.rows, w->k.cols, s->h, seq, s->k);
  orc_matmul(w->v.type, w->v.data, w->v.rows, w->v.cols, s->h, seq, s->v);
  for (int64_t t = 0; t < seq; ++t) {
    for (int32_t h = 0; h < c->n_heads; ++h) {
      float* p = s->q + t * qd + (int64_t)h * hd;
      orc_rmsnorm(p, w->q_norm, hd, c->rms_eps, p);
    }
    for (int32_t h = 0; h < c->n_kv_heads; ++h) {
      float* p = s->k + t * kvd + (int64_t)h * hd;
      orc_rmsnorm(p, w->k_norm, hd, c->rms_eps, p);
    }
  }
  for (int64_t t = 0; t < seq; ++t) {
    const float* ct = m->rope + (pos0 + t) * half * 2;
    rope_inplace(s->q + t * qd, c->n_heads, hd, ct, ct + half);
    rope_inplace(s->k + t * kvd, c->n_kv_heads, hd, ct, ct + half);
  }
  if (kv) {
    for (int64_t t = 0; t < seq; ++t) {
      for (int32_t h = 0; h < c->n_kv_heads; ++h) {
        memcpy(kv->k + kv_off(kv, layer, h, pos0 + t), s->k + t * kvd + (int64_t)h * hd,
               (size_t)hd * sizeof(float));
        memcpy(kv->v + kv_off(kv, layer, h, pos0 + t), s->v + t * kvd + (int64_t)h * hd,
               (size_t)hd * sizeof(float));
      }
    }
  }
  attention(c, s->q, seq, kv ? pos0 : 0, s->k, s->v, kv, layer, s->attn);
  orc_matmul(w->o.type, w->o.data, w->o.rows, w->o.cols, s->attn, seq, s->proj);
  for (int64_t i = 0; i < seq * H; ++i) s->x[i] += s->proj[i];
  for (int64_t t = 0; t < seq; ++t) orc_rmsnorm(s->x + t * H, w->ffn_norm, H, c->rms_eps, s->h + t * H);
  orc_matmul(w->gate.type, w->gate.data, w->gate.rows, w->gate.cols, s->h, seq, s->gate);
  orc_matmul(w->up.type, w->up.data, w->up.rows, w->up.cols, s->h, seq, s->up);
  for (int64_t i = 0; i < seq * F; ++i) {
    const float v = s->gate[i];
    s->gate[i] = v / (1.0f + expf(-v));
  }
  for (int64_t i = 0; i < seq * F; ++i) s->gate[i] *= s->up[i];
  orc_matmul(w->down.type, w->down.data, w->down.rows, w->down.cols, s->gate, seq, s->proj);
  for (int64_t i = 0; i < seq * H; ++i) s->x[i] += s->proj[i];
}

/* src/qwen3.cc:208-290 (ForwardFull).  logits receives seq*vocab floats when
 * all_rows != 0, otherwise only the last row (vocab floats) -- the last row is
 * computed exactly as the reference computes it.  Returns 0, or -1 on a bad
 * argument (bounds mirror src/qwen3.cc:215-232). */
int orc_forward(const orc_model* m, orc_kv* kv, const int32_t* ids, int64_t seq, float* logits,
                int all_rows) {
  const orc_config* c = &m->c;
  const int64_t H = c->hidden, F = c->intermediate;
  const int64_t qd = (int64_t)c->n_heads * c->head_dim, kvd = (int64_t)c->n_kv_heads * c->head_dim;
  if (seq <= 0) return -1;
  const int64_t pos0 = kv ? kv->len : 0;
  if (pos0 + seq > m->n_rope_pos) return -1;
  if (kv && pos0 + seq > kv->max_seq) return -1;
  for (int64_t t = 0; t < seq; ++t)
    if (ids[t] < 0 || ids[t] >= c->vocab) return -1;
  scratch_t s;
  s.x = (float*)malloc((size_t)seq * H * 4);
  s.h = (float*)malloc((size_t)seq * H * 4);
  s.q = (float*)malloc((size_t)seq * qd * 4);
  s.k = (float*)malloc((size_t)seq * kvd * 4);
  s.v = (float*)malloc((size_t)seq * kvd * 4);
  s.attn = (float*)malloc((size_t)seq * qd * 4);
  s.proj = (float*)malloc((size_t)seq * H * 4);
  s.gate = (float*)malloc((size_t)seq * F * 4);
  s.up = (float*)malloc((size_t)seq * F * 4);
  const int64_t erb = orc_row_bytes(m->token_embd.type, H);
  for (int64_t t = 0; t < seq; ++t)
    orc_dequantize_row(m->token_embd.type, m->token_embd.data + ids[t] * erb, H, s.x + t * H);
  for (int32_t l = 0; l < c->n_layers; ++l) forward_layer(m, &m->layers[l], l, pos0, &s, seq, kv);
  if (kv) kv->len = pos0 + seq;
  const int64_t t0 = all_rows ? 0 : seq - 1;
  for (int64_t t = t0; t < seq; ++t) orc_rmsnorm(s.x + t * H, m->output_norm, H, c->rms_eps, s.h + t * H);
  orc_matmul(m->lm_head.type, m->lm_head.data, m->lm_head.rows, m->lm_head.cols, s.h + t0 * H,
             seq - t0, logits);
  free(s.x); free(s.h); free(s.q); free(s.k); free(s.v);
  free(s.attn); free(s.proj); free(s.gate); free(s.up);
  return 0;
}

typedef struct {
  int32_t max_tokens;
  const int32_t* stop_ids;
  int32_t n_stop;
  float temperature;
  int32_t top_k;
  float top_p;
  uint64_t seed;
} orc_gen_opts;

/* src/qwen3.cc:302-355 (Generate).  out receives up to max_tokens ids;
 * step_logits (optional, max_tokens*vocab) receives the logits each token was
 * picked from.  Returns 0, -1 on a bad argument, -2 when the context filled
 * up (the reference throws there; out/n_out hold what was produced). */
int orc_generate(const orc_model* m, orc_kv* kv, const float* first_logits,
                 const orc_gen_opts* o, int32_t* out, int32_t* n_out, float* step_logits) {
  const int64_t V = m->c.vocab;
  *n_out = 0;
  if (!kv || !first_logits || o->max_tokens <= 0) return -1;
  float* logits = (float*)malloc((size_t)V * sizeof(float));
  memcpy(logits, first_logits, (size_t)V * sizeof(float));
  const int greedy = !(o->temperature > 0.0f);
  int rc = 0;
  for (int32_t i = 0; i < o->max_tokens; ++i) {
    if (step_logits) memcpy(step_logits + (int64_t)i * V, logits, (size_t)V * sizeof(float));
    int32_t next;
    if (greedy) {
      next = orc_argmax(logits, V);
    } else {
      const float u = orc_counter_uniform(o->seed, (uint64_t)kv->len);
      next = orc_sample_token(logits, V, o->temperature, o->top_k, o->top_p, u);
    }
    out[(*n_out)++] = next;
    int stop = 0;
    for (int32_t j = 0; j < o->n_stop; ++j)
      if (o->stop_ids[j] == next) stop = 1;
    if (!(kv->len < kv->max_seq)) {
      rc = -2;
      break;
    }
    if (orc_forward(m, kv, &next, 1, logits, 0) != 0) {
      rc = -1;
      break;
    }
    if (stop) break;
  }
  free(logits);
  return rc;
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
