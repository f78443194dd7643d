/*
 * tg_oracle.c -- CPU parity oracle (test infrastructure only; see
 * tg_oracle.h).  A plain-C restatement of the reference's CPU hot path:
 *   RoPE            tmac_gguf.cpp:990-1016   (apply_rope)
 *   cache-write     tmac_gguf.cpp:1090-1091
 *   GQA attention   tmac_gguf.cpp:1093-1128
 *   Q/K/V projection f16_to_f32 :220-232, dequant_q8_0 :240-248,
 *                   dequant_q5_0 :311-328, read_tensor :402-415, matmul's
 *                   CPU loop :508-512, bias adds :1067-1081
 *   attn_output     matmul + residual add :1129-1140
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, no -march=native).
 */
#include "tg_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ */
/* seeded inputs                                                       */
/* ------------------------------------------------------------------ */

uint64_t tgo_splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ULL);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

void tgo_fill_normal(uint64_t seed, float *out, size_t n) {
  uint64_t s = seed;
  const double two_pi = 6.283185307179586476925286766559;
  const double inv53 = 1.0 / 9007199254740992.0; /* 2^-53 */
  size_t i = 0;
  while (i < n) {
    uint64_t a = tgo_splitmix64(&s);
    uint64_t b = tgo_splitmix64(&s);
    double u1 = ((double)(a >> 11) + 1.0) * inv53; /* (0, 1] */
    double u2 = (double)(b >> 11) * inv53;         /* [0, 1) */
    double r = sqrt(-2.0 * log(u1));
    out[i++] = (float)(r * cos(two_pi * u2));
    if (i < n) out[i++] = (float)(r * sin(two_pi * u2));
  }
}

uint16_t tgo_f32_to_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  }
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

float tgo_bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void tgo_round_bf16_inplace(float *x, size_t n) {
  for (size_t i = 0; i < n; i++) x[i] = tgo_bf16_to_f32(tgo_f32_to_bf16(x[i]));
}

void tgo_pack_bf16(const float *x, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = tgo_f32_to_bf16(x[i]);
}

void tgo_fill_normal_bf16(uint64_t seed, float *out, size_t n) {
  tgo_fill_normal(seed, out, n);
  tgo_round_bf16_inplace(out, n);
}

/* ------------------------------------------------------------------ */
/* RoPE -- tmac_gguf.cpp:990-1016                                      */
/* ------------------------------------------------------------------ */

void tgo_rope_cos_sin(int head_dim, int pos, float base, float *cs) {
  for (int d = 0; d < head_dim; d += 2) {
    /* :993 theta = 1/powf(base, (float)d / HEAD_DIM); :994 freq = pos*theta */
    float theta = 1.0f / powf(base, (float)d / head_dim);
    float freq = pos * theta;
    cs[d] = cosf(freq);     /* :995 */
    cs[d + 1] = sinf(freq); /* :996 */
  }
}

void tgo_rope_heads(float *x, int n_heads, int head_dim, int pos, float base) {
  for (int h = 0; h < n_heads; h++) {
    for (int d = 0; d < head_dim; d += 2) {
      float theta = 1.0f / powf(base, (float)d / head_dim);
      float freq = pos * theta;
      float cos_val = cosf(freq);
      float sin_val = sinf(freq);
      int idx = h * head_dim + d;
      float x0 = x[idx], x1 = x[idx + 1];
      /* :999-1000, two roundings per output (no contraction) */
      x[idx] = x0 * cos_val - x1 * sin_val;
      x[idx + 1] = x0 * sin_val + x1 * cos_val;
    }
  }
}

void tgo_apply_rope(float *q, float *k, int n_head, int n_kv_head,
                    int head_dim, int pos, float base) {
  tgo_rope_heads(q, n_head, head_dim, pos, base);    /* :992-1002 */
  tgo_rope_heads(k, n_kv_head, head_dim, pos, base); /* :1003-1015 */
}

/* ------------------------------------------------------------------ */
/* cache-write -- tmac_gguf.cpp:1090-1091                              */
/* ------------------------------------------------------------------ */

void tgo_cache_write(float *k_cache, float *v_cache, const float *k_new,
                     const float *v_new, int n_kv_head, int head_dim,
                     int pos) {
  const int kdim = n_kv_head * head_dim;
  for (int i = 0; i < kdim; i++) k_cache[(size_t)pos * kdim + i] = k_new[i];
  for (int i = 0; i < kdim; i++) v_cache[(size_t)pos * kdim + i] = v_new[i];
}

/* ------------------------------------------------------------------ */
/* attention -- tmac_gguf.cpp:1093-1128                                */
/* ------------------------------------------------------------------ */

void tgo_attention_head(const float *q, const float *k_cache,
                        const float *v_cache, float *ctx_h, int qh,
                        int n_head, int n_kv_head, int head_dim, int pos,
                        float *scores) {
  const int kdim = n_kv_head * head_dim;
  const int q_per_kv = n_head / n_kv_head; /* :1096 */
  const int kv = qh / q_per_kv;            /* :1099 */
  const float *qh_data = q + qh * head_dim;

  /* :1103-1110 -- d outer, p inner */
  for (int p = 0; p <= pos; p++) scores[p] = 0;
  for (int d = 0; d < head_dim; d++) {
    float q_val = qh_data[d];
    for (int p = 0; p <= pos; p++) {
      const float *k_cached = k_cache + (size_t)p * kdim + kv * head_dim;
      scores[p] += q_val * k_cached[d];
    }
  }
  /* :1111 */
  for (int p = 0; p <= pos; p++) scores[p] /= sqrtf((float)head_dim);

  /* :1113-1117 */
  float max_score = scores[0];
  for (int p = 1; p <= pos; p++)
    if (scores[p] > max_score) max_score = scores[p];
  float exp_sum = 0;
  for (int p = 0; p <= pos; p++) exp_sum += expf(scores[p] - max_score);
  float log_sum = logf(exp_sum) + max_score;

  /* :1119-1125 -- p outer, d inner, context starts at zero (:1095) */
  for (int d = 0; d < head_dim; d++) ctx_h[d] = 0;
  for (int p = 0; p <= pos; p++) {
    const float *v_cached = v_cache + (size_t)p * kdim + kv * head_dim;
    float exp_score = expf(scores[p] - log_sum);
    for (int d = 0; d < head_dim; d++) ctx_h[d] += exp_score * v_cached[d];
  }
}

void tgo_attention(const float *q, const float *k_cache, const float *v_cache,
                   float *context, int n_head, int n_kv_head, int head_dim,
                   int pos, float *scores_buf) {
  for (int qh = 0; qh < n_head; qh++)
    tgo_attention_head(q, k_cache, v_cache, context + qh * head_dim, qh,
                       n_head, n_kv_head, head_dim, pos, scores_buf);
}

void tgo_decode_step(float *q, float *k_new, const float *v_new,
                     float *k_cache, float *v_cache, float *context,
                     int n_head, int n_kv_head, int head_dim, int pos,
                     float base, float *scores_buf) {
  tgo_apply_rope(q, k_new, n_head, n_kv_head, head_dim, pos, base); /* :1087 */
  tgo_cache_write(k_cache, v_cache, k_new, v_new, n_kv_head, head_dim,
                  pos);                                          /* :1090 */
  tgo_attention(q, k_cache, v_cache, context, n_head, n_kv_head, head_dim,
                pos, scores_buf);                                /* :1093 */
}

void tgo_prefill_causal(const float *q, const float *k, const float *v,
                        float *out, int S, int n_head, int n_kv_head,
                        int head_dim, int t_begin, int t_end) {
  (void)S;
  float *scores = (float *)malloc(sizeof(float) * (size_t)(t_end > 0 ? t_end : 1));
  const size_t qdim = (size_t)n_head * head_dim;
  for (int t = t_begin; t < t_end; t++)
    tgo_attention(q + (size_t)t * qdim, k, v, out + (size_t)t * qdim, n_head,
                  n_kv_head, head_dim, t, scores);
  free(scores);
}

/* ------------------------------------------------------------------ */
/* multi-threaded baseline                                             */
/* ------------------------------------------------------------------ */

typedef struct {
  int n_units, n_head, n_kv_head, head_dim;
  const float *q;
  size_t q_stride;
  const float *const *k_ptrs;
  const float *const *v_ptrs;
  const int *pos;
  float *out;
  int max_pos;
  int thread_idx, n_threads;
} mt_job;

static void *mt_worker(void *arg) {
  mt_job *j = (mt_job *)arg;
  float *scores = (float *)malloc(sizeof(float) * (size_t)(j->max_pos + 1));
  if (!scores) return (void *)1;
  const long total = (long)j->n_units * j->n_head;
  for (long w = j->thread_idx; w < total; w += j->n_threads) {
    int u = (int)(w / j->n_head), qh = (int)(w % j->n_head);
    tgo_attention_head(j->q + (size_t)u * j->q_stride, j->k_ptrs[u],
                       j->v_ptrs[u],
                       j->out + (size_t)u * j->q_stride + (size_t)qh * j->head_dim,
                       qh, j->n_head, j->n_kv_head, j->head_dim, j->pos[u],
                       scores);
  }
  free(scores);
  return NULL;
}

int tgo_attention_units_mt(int n_units, const float *q, size_t q_stride,
                           const float *const *k_ptrs,
                           const float *const *v_ptrs, const int *pos,
                           float *out, int n_head, int n_kv_head,
                           int head_dim, int n_threads) {
  if (n_threads < 1) n_threads = 1;
  int max_pos = 0;
  for (int u = 0; u < n_units; u++)
    if (pos[u] > max_pos) max_pos = pos[u];
  mt_job *jobs = (mt_job *)calloc((size_t)n_threads, sizeof(mt_job));
  pthread_t *th = (pthread_t *)calloc((size_t)n_threads, sizeof(pthread_t));
  if (!jobs || !th) {
    free(jobs);
    free(th);
    return 1;
  }
  int rc = 0;
  for (int t = 0; t < n_threads; t++) {
    mt_job j = {n_units, n_head, n_kv_head, head_dim, q, q_stride, k_ptrs,
                v_ptrs, pos, out, max_pos, t, n_threads};
    jobs[t] = j;
  }
  int started = 0;
  for (int t = 1; t < n_threads; t++) {
    if (pthread_create(&th[t], NULL, mt_worker, &jobs[t]) != 0) {
      rc = 1;
      break;
    }
    started = t;
  }
  if (mt_worker(&jobs[0]) != NULL) rc = 1;
  for (int t = 1; t <= started; t++) {
    void *ret = NULL;
    pthread_join(th[t], &ret);
    if (ret != NULL) rc = 1;
  }
  free(jobs);
  free(th);
  return rc;
}

/* ------------------------------------------------------------------ */
/* split-KV helpers (not in the reference)                             */
/* ------------------------------------------------------------------ */

void tgo_partial_head(const float *q, const float *k_cache,
                      const float *v_cache, int qh, int n_head,
                      int n_kv_head, int head_dim, int p0, int p1, float *m,
                      float *l, float *o, float *scores) {
  const int kdim = n_kv_head * head_dim;
  const int kv = qh / (n_head / n_kv_head);
  const float *qh_data = q + qh * head_dim;
  for (int p = p0; p < p1; p++) scores[p - p0] = 0;
  for (int d = 0; d < head_dim; d++) {
    float q_val = qh_data[d];
    for (int p = p0; p < p1; p++)
      scores[p - p0] += q_val * k_cache[(size_t)p * kdim + kv * head_dim + d];
  }
  for (int p = p0; p < p1; p++) scores[p - p0] /= sqrtf((float)head_dim);
  float mx = -INFINITY;
  for (int p = p0; p < p1; p++)
    if (scores[p - p0] > mx) mx = scores[p - p0];
  float sum = 0;
  for (int d = 0; d < head_dim; d++) o[d] = 0;
  for (int p = p0; p < p1; p++) {
    float e = expf(scores[p - p0] - mx);
    sum += e;
    const float *vr = v_cache + (size_t)p * kdim + kv * head_dim;
    for (int d = 0; d < head_dim; d++) o[d] += e * vr[d];
  }
  *m = mx;
  *l = sum;
}

void tgo_merge_partials(int n_parts, const float *m, const float *l,
                        const float *o, int head_dim, float *out) {
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; i++)
    if (m[i] > mx) mx = m[i];
  float lsum = 0;
  for (int d = 0; d < head_dim; d++) out[d] = 0;
  for (int i = 0; i < n_parts; i++) {
    if (l[i] == 0.0f) continue;
    float w = expf(m[i] - mx);
    lsum += l[i] * w;
    for (int d = 0; d < head_dim; d++) out[d] += o[(size_t)i * head_dim + d] * w;
  }
  for (int d = 0; d < head_dim; d++) out[d] /= lsum;
}

/* ------------------------------------------------------------------ */
/* quantized Q/K/V projection                                          */
/* ------------------------------------------------------------------ */

size_t tgo_qrow_bytes(int type, int cols) {
  if (type == TGO_TYPE_F32) return (size_t)cols * 4;
  if (type == TGO_TYPE_Q5_0) return (size_t)(cols / 32) * 22;
  if (type == TGO_TYPE_Q8_0) return (size_t)(cols / 32) * 34;
  return 0;
}

/* f16_to_f32 (tmac_gguf.cpp:220-232) widens exactly: a zero of either sign
 * becomes +0 (:225), subnormals mant*2^-24 (:226), Inf keeps its sign and
 * every NaN becomes the NAN macro (:228), normals rebias the exponent
 * (:230).  Restated with the bit pattern built directly. */
float tgo_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t u;
  if (e == 0) {
    if (m == 0) return 0.0f;
    const float f = (float)m * 0x1p-24f; /* exact: m < 2^10 */
    return sign ? -f : f;
  }
  if (e == 0x1fu) {
    if (m) return NAN;
    u = sign | 0x7f800000u;
  } else {
    u = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

float tgo_dequant(int type, const uint8_t *w, uint64_t idx) {
  if (type == TGO_TYPE_F32) {
    float f;
    memcpy(&f, w + idx * 4, 4);
    return f;
  }
  const uint64_t blk = idx / 32, j = idx % 32;
  if (type == TGO_TYPE_Q8_0) {
    /* :243-247: d at bytes 0-1 (little endian), int8 values from byte 2. */
    const uint8_t *b = w + blk * 34;
    const float d = tgo_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    return (float)(int8_t)b[2 + j] * d;
  }
  if (type == TGO_TYPE_Q5_0) {
    /* :314-327: d, then the 32 high bits, then 16 bytes holding elements
     * j (low nibble) and j+16 (high nibble). */
    const uint8_t *b = w + blk * 22;
    const float d = tgo_f16_to_f32((uint16_t)(b[0] | (b[1] << 8)));
    const uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) |
                        ((uint32_t)b[5] << 24);
    const uint8_t byte = b[6 + (j < 16 ? j : j - 16)];
    const uint32_t lo = j < 16 ? (byte & 0xfu) : (byte >> 4);
    const int q = (int)((((qh >> j) & 1u) << 4) | lo) - 16;
    return d * (float)q;
  }
  return 0.0f;
}

void tgo_matmul_q(int type, const uint8_t *w, const float *x, float *y, int rows, int cols) {
  for (int i = 0; i < rows; i++) {
    float sum = 0.0f;
    for (int j = 0; j < cols; j++)
      sum += tgo_dequant(type, w, (uint64_t)j + (uint64_t)i * (uint64_t)cols) * x[j];
    y[i] = sum;
  }
}

void tgo_qkv_step(int q_type, const uint8_t *wq, int k_type, const uint8_t *wk, int v_type,
                  const uint8_t *wv, const float *bq, const float *bk, const float *bv,
                  const float *x, float *q, float *k, float *v, int n_head, int n_kv_head,
                  int head_dim, int cols, int pos, float base, float *k_cache,
                  float *v_cache) {
  const int qd = n_head * head_dim, kd = n_kv_head * head_dim;
  /* :1046-1064 the three projections of the same input */
  tgo_matmul_q(q_type, wq, x, q, qd, cols);
  tgo_matmul_q(k_type, wk, x, k, kd, cols);
  tgo_matmul_q(v_type, wv, x, v, kd, cols);
  /* :1067-1081 bias adds, each present bias added element by element */
  if (bq)
    for (int i = 0; i < qd; i++) q[i] += bq[i];
  if (bk)
    for (int i = 0; i < kd; i++) k[i] += bk[i];
  if (bv)
    for (int i = 0; i < kd; i++) v[i] += bv[i];
  /* :1085-1088 RoPE; :1090-1091 cache-write */
  tgo_apply_rope(q, k, n_head, n_kv_head, head_dim, pos, base);
  if (k_cache && v_cache) tgo_cache_write(k_cache, v_cache, k, v, n_kv_head, head_dim, pos);
}

void tgo_attn_output(int o_type, const uint8_t *wo, const float *context,
                     const float *original_hidden, float *hidden, int rows, int cols,
                     float *attn_out) {
  float *tmp = attn_out ? attn_out : (float *)malloc((size_t)rows * sizeof(float));
  if (!tmp) return;
  tgo_matmul_q(o_type, wo, context, tmp, rows, cols);                    /* :1135 */
  for (int i = 0; i < rows; i++) hidden[i] = original_hidden[i] + tmp[i]; /* :1140 */
  if (!attn_out) free(tmp);
}

/* Round a positive or negative binary32 in the half normal range to an
 * IEEE half (nearest even); out-of-range magnitudes clamp to the smallest
 * or largest normal half.  Used only to make synthetic scales. */
static uint16_t f32_to_f16_clamped(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  const uint32_t sign = (u >> 16) & 0x8000u;
  int32_t e = (int32_t)((u >> 23) & 0xffu) - 127 + 15;
  const uint32_t m = u & 0x7fffffu;
  if (e <= 0) return (uint16_t)(sign | 0x0400u);
  if (e >= 31) return (uint16_t)(sign | 0x7bffu);
  uint32_t r = m >> 13;
  const uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) {
    if (++r == 0x400u) {
      r = 0;
      if (++e >= 31) return (uint16_t)(sign | 0x7bffu);
    }
  }
  return (uint16_t)(sign | ((uint32_t)e << 10) | r);
}

void tgo_fill_qblocks(int type, uint64_t seed, uint8_t *out, size_t n_blocks, float d_scale) {
  uint64_t s = seed;
  const size_t bs = type == TGO_TYPE_Q5_0 ? 22 : 34;
  for (size_t b = 0; b < n_blocks; b++) {
    uint8_t *blk = out + b * bs;
    const uint64_t a = tgo_splitmix64(&s);
    const double u = (double)(a >> 11) * (1.0 / 9007199254740992.0);
    float d = (float)((double)d_scale * (0.5 + u));
    if (a & 1u) d = -d;
    const uint16_t h = f32_to_f16_clamped(d);
    blk[0] = (uint8_t)(h & 0xffu);
    blk[1] = (uint8_t)(h >> 8);
    for (size_t i = 2; i < bs; i += 8) {
      uint64_t r = tgo_splitmix64(&s);
      for (size_t k = 0; k < 8 && i + k < bs; k++, r >>= 8) blk[i + k] = (uint8_t)(r & 0xffu);
    }
  }
}
