/*
 * tg_oracle.h -- CPU parity oracle for the decode-attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: it restates, in
 * plain C, the reference's CPU algorithm for RoPE, the KV cache-write and
 * the GQA decode attention of tmac_gguf.cpp, so that the CUDA product can be
 * compared against it on identical seeded inputs.  Only tests/, the smoke
 * check in __graft_entry__.py and bench.py's cpu_baseline / reference arm
 * may load it.  The product library never links or calls it.
 *
 * Parity pin: every routine here is checked bit-for-bit against the
 * reference's own code (tmac_gguf.cpp:990-1016 and :1090-1128, compiled
 * from the reference source tree by oracle/Makefile into oracle/_ref/) and
 * against the golden fixtures in tests/golden/ that the reference code
 * produced (tests/golden/make_golden.py).
 *
 * Floating-point contract: compiled with -O2 -ffp-contract=off and without
 * -march=native, so every product and sum is one IEEE binary32 operation
 * with round-to-nearest-even, exactly as written.
 */
#ifndef TG_ORACLE_H
#define TG_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (splitmix64 + Box-Muller, N(0,1)) ---- */

/* One splitmix64 step; *state advances by the golden-gamma constant. */
uint64_t tgo_splitmix64(uint64_t *state);

/* Fill out[0..n) with N(0,1) binary32 values from `seed`.  Pairs of
 * splitmix64 draws feed one Box-Muller transform evaluated in binary64
 * and rounded once to binary32.  The stream depends only on (seed, n). */
void tgo_fill_normal(uint64_t seed, float *out, size_t n);

/* Same stream, rounded to bfloat16 (round-to-nearest-even) and widened
 * back to binary32: the "bf16 KV ~ N(0,1) rounded to bf16" inputs. */
void tgo_fill_normal_bf16(uint64_t seed, float *out, size_t n);

/* Round a binary32 value to bfloat16 with round-to-nearest-even; NaN stays
 * a quiet NaN.  Returns the 16-bit pattern. */
uint16_t tgo_f32_to_bf16(float x);
float tgo_bf16_to_f32(uint16_t h);
/* In-place: x[i] = widen(round_bf16(x[i])). */
void tgo_round_bf16_inplace(float *x, size_t n);
/* Pack x[0..n) into bf16 bit patterns (RNE). */
void tgo_pack_bf16(const float *x, uint16_t *out, size_t n);

/* ---- RoPE (tmac_gguf.cpp:990-1016) ---- */

/* Rotate adjacent pairs (2i, 2i+1) of n_heads heads of head_dim values in
 * place at position pos.  theta = 1/powf(base, d/head_dim), angle =
 * pos*theta, cosf/sinf from the host libm.  The reference hard-codes
 * base = 1e6, 14 query heads and 2 KV heads of 64; this takes them as
 * arguments and applies the same per-head loop. */
void tgo_rope_heads(float *x, int n_heads, int head_dim, int pos, float base);

/* apply_rope(q, k, pos) with the reference's shape: q has n_head heads, k
 * has n_kv_head heads (tmac_gguf.cpp:990-1016, base 1e6 at :991). */
void tgo_apply_rope(float *q, float *k, int n_head, int n_kv_head,
                    int head_dim, int pos, float base);

/* The cos/sin values the reference computes for (pos, pair i):
 * cs[2*i] = cosf(pos*theta_i), cs[2*i+1] = sinf(pos*theta_i). */
void tgo_rope_cos_sin(int head_dim, int pos, float base, float *cs);

/* ---- cache-write (tmac_gguf.cpp:1090-1091) ---- */

/* k_cache/v_cache are one layer's cache, position-major, row stride
 * n_kv_head*head_dim floats (g_k_cache[layer][pos][K_DIM], :200-201). */
void tgo_cache_write(float *k_cache, float *v_cache, const float *k_new,
                     const float *v_new, int n_kv_head, int head_dim,
                     int pos);

/* ---- GQA decode attention (tmac_gguf.cpp:1093-1128) ---- */

/* context[h*head_dim + d] for h < n_head, over cache rows p = 0..pos.
 * Loop order, the /sqrtf(head_dim) scaling, the max / exp_sum / log_sum
 * softmax and the p-outer accumulation follow the reference line by line.
 * scores_buf must hold pos+1 floats (the reference's scores[MAX_SEQ_LEN]). */
void tgo_attention(const float *q, const float *k_cache, const float *v_cache,
                   float *context, int n_head, int n_kv_head, int head_dim,
                   int pos, float *scores_buf);

/* One query head of the above (the unit the multi-threaded baseline fans
 * out over).  ctx_h receives head_dim values. */
void tgo_attention_head(const float *q, const float *k_cache,
                        const float *v_cache, float *ctx_h, int qh,
                        int n_head, int n_kv_head, int head_dim, int pos,
                        float *scores_buf);

/* The full per-(sequence, layer) hot path of forward_layer_with_cache
 * (tmac_gguf.cpp:1087-1128): RoPE on q/k_new at pos, write the roped k and
 * v rows at pos, attend over 0..pos.  q and k_new are rotated in place. */
void tgo_decode_step(float *q, float *k_new, const float *v_new,
                     float *k_cache, float *v_cache, float *context,
                     int n_head, int n_kv_head, int head_dim, int pos,
                     float base, float *scores_buf);

/* Causal prefill as the reference runs it: token by token
 * (process_prompt, tmac_gguf.cpp:1621-1644, one decode step per token).
 * q: [S][n_head*hd], k/v: [S][n_kv*hd] (already roped, already rounded as
 * the caller wants), out: [S][n_head*hd].  Rows are attended over the
 * prefix 0..t of k/v, which play the role of the filled cache. */
void tgo_prefill_causal(const float *q, const float *k, const float *v,
                        float *out, int S, int n_head, int n_kv_head,
                        int head_dim, int t_begin, int t_end);

/* ---- quantized Q/K/V projection (tmac_gguf.cpp:220-248, 311-328,
 *      402-415, 476-513 and the layer step :1046-1091) ---- */

/* Weight types (tmac_gguf.cpp:177-182) and their 32-element blocks:
 * Q8_0 = fp16 d + 32 int8 (34 bytes), value d*q;
 * Q5_0 = fp16 d + 32 high bits + 16 bytes of nibbles (22 bytes), value
 * d*(((hi<<4)|lo) - 16), element j < 16 in the low nibble of byte j,
 * element j >= 16 in the high nibble of byte j-16. */
#define TGO_TYPE_F32 0
#define TGO_TYPE_Q5_0 6
#define TGO_TYPE_Q8_0 8

/* Bytes of one row of `cols` elements (cols a multiple of 32); 0 for an
 * unknown type. */
size_t tgo_qrow_bytes(int type, int cols);

/* f16_to_f32 (tmac_gguf.cpp:220-232): exact widening of an IEEE half. */
float tgo_f16_to_f32(uint16_t h);

/* dequant_q8_0 / dequant_q5_0 (tmac_gguf.cpp:240-248, :311-328): element
 * idx of a row-major block array. */
float tgo_dequant(int type, const uint8_t *w, uint64_t idx);

/* matmul's CPU loop (tmac_gguf.cpp:508-512 with read_tensor :402-415):
 * y[i] = sum over j of dequant(w, j + i*cols) * x[j], summed in j order in
 * binary32. */
void tgo_matmul_q(int type, const uint8_t *w, const float *x, float *y,
                  int rows, int cols);

/* The layer step from the normed hidden state to the cache
 * (forward_layer_with_cache, tmac_gguf.cpp:1046-1091): q/k/v = W x
 * (q rows n_head*head_dim, k/v rows n_kv_head*head_dim, `cols` inputs),
 * + bias (skipped where the bias pointer is NULL), RoPE of q and k at pos,
 * then the k and v rows written at row pos of k_cache / v_cache (skipped
 * when the caches are NULL).  q, k, v receive the final vectors. */
void tgo_qkv_step(int q_type, const uint8_t *wq, int k_type,
                  const uint8_t *wk, int v_type, const uint8_t *wv,
                  const float *bq, const float *bk, const float *bv,
                  const float *x, float *q, float *k, float *v, int n_head,
                  int n_kv_head, int head_dim, int cols, int pos, float base,
                  float *k_cache, float *v_cache);

/* The attn_output matvec and the residual add of forward_layer_with_cache
 * (tmac_gguf.cpp:1129-1140): attn_out = W_o context (matmul's CPU loop),
 * then hidden[i] = original_hidden[i] + attn_out[i].  attn_out may be NULL
 * when the caller does not need it (a rows-long scratch is used). */
void tgo_attn_output(int o_type, const uint8_t *wo, const float *context,
                     const float *original_hidden, float *hidden, int rows,
                     int cols, float *attn_out);

/* Synthetic weight blocks from `seed`: scales d = fp16(d_scale * (0.5 +
 * u)), u uniform in [0, 1); the quant bytes uniform.  n_blocks blocks of
 * `type` are written to out. */
void tgo_fill_qblocks(int type, uint64_t seed, uint8_t *out, size_t n_blocks,
                      float d_scale);

/* ---- multi-threaded CPU baseline (not in the reference) ---- */

/* Attention for n_units independent (sequence, layer) units, fanned out
 * over n_threads POSIX threads at (unit, head) granularity.  Unit u reads
 * q + u*q_stride, k/v caches at k_ptrs[u]/v_ptrs[u] and attends over
 * positions 0..pos[u]; output to out + u*q_stride.  Each (unit, head) runs
 * tgo_attention_head, so results are bit-identical to the serial oracle.
 * Returns 0 on success. */
int tgo_attention_units_mt(int n_units, const float *q, size_t q_stride,
                           const float *const *k_ptrs,
                           const float *const *v_ptrs, const int *pos,
                           float *out, int n_head, int n_kv_head,
                           int head_dim, int n_threads);

/* Split-KV merge restated on the host: combine n_parts partial softmax
 * states (m in natural-log units, l = sum of exp(s - m), o = unnormalised
 * sum of exp(s - m)*V) of one head into the normalised output. */
void tgo_merge_partials(int n_parts, const float *m, const float *l,
                        const float *o, int head_dim, float *out);

/* Partial softmax state of one head over cache rows [p0, p1) in the
 * oracle's own arithmetic (scores as in tgo_attention_head). */
void tgo_partial_head(const float *q, const float *k_cache,
                      const float *v_cache, int qh, int n_head,
                      int n_kv_head, int head_dim, int p0, int p1, float *m,
                      float *l, float *o, float *scores_buf);

#ifdef __cplusplus
}
#endif
#endif /* TG_ORACLE_H */
