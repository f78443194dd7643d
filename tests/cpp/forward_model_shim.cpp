// The decode step of the reference's forward loop (tmac_gguf.cpp:1453-1516,
// forward_all_layers_fused) on Linux with this library as the backend of its
// Metal ops: per layer RMSNorm -> fused_qkv_op (Q5_0 q/k, Q8_0 v) and the
// three bias adds (elem_op 0) -> rope_op x2 -> elem_op(2) x2 (cache-write)
// -> attention_op -> matmul_q5_0 (attn_output) -> elem_op(0) residual, all
// inside metal_batch_begin / metal_batch_end, as :1468-1499 encodes them ->
// RMSNorm -> gate/up -> SiLU -> down -> residual.  The ops go through
// cuda_backend.hpp with the reference's arguments and host arrays; the
// norms and the FFN (not on this path) are host-side fp32 stubs.  Weights
// are seeded blocks of Qwen2-0.5B's shapes (one weight set shared by all
// layers, to keep the program small), registered once as device-owned.
// The same loop is run a second time with the CPU oracle in place of the
// backend (tg_oracle.c: the restatements of matmul's CPU loop
// :476-513 with dequant_q5_0 / dequant_q8_0, the bias adds :1067-1081 and
// the decode step :990-1016, :1090-1128, attn_output + residual
// :1129-1140), and the hidden states after every
// token are compared.  Prints PASS / FAIL.
//
// usage: forward_model_shim <n_tokens> <device_owned 0|1>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "cuda_backend.hpp"
#include "tg_oracle.h"

namespace {
constexpr int NUM_LAYERS = 24, NUM_HEADS = 14, NUM_KV_HEADS = 2, HEAD_DIM = 64;
constexpr int HIDDEN_DIM = NUM_HEADS * HEAD_DIM, K_DIM = NUM_KV_HEADS * HEAD_DIM;
constexpr int INTER_DIM = 4864, MAX_SEQ_LEN = 64;
constexpr float ROPE_BASE = 1000000.0f, RMS_EPS = 1e-6f;

// The reference's static caches (tmac_gguf.cpp:200-201): one pair driven by
// the backend, one by the oracle.
float g_k_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float g_v_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float o_k_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float o_v_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];

struct Weights {
  std::vector<uint8_t> wq, wk, wv, wo;  // GGML blocks: Q5_0 (q, k, o), Q8_0 (v)
  std::vector<float> bq, bk, bv, gate, up, down;
};

void fill_blocks(std::vector<uint8_t>& w, int type, int rows, int cols, uint64_t seed,
                 float d_scale) {
  const size_t nb = (size_t)rows * (cols / 32);
  w.resize(nb * (type == TGO_TYPE_Q5_0 ? 22 : 34));
  tgo_fill_qblocks(type, seed, w.data(), nb, d_scale);
}

void fill(std::vector<float>& w, size_t n, uint64_t seed, float scale) {
  w.resize(n);
  tgo_fill_normal(seed, w.data(), (int)n);
  for (float& x : w) x *= scale;
}

void matvec(const std::vector<float>& w, const float* x, float* y, int rows, int cols) {
  for (int r = 0; r < rows; ++r) {
    const float* wr = w.data() + (size_t)r * cols;
    double acc = 0.0;
    for (int c = 0; c < cols; ++c) acc += (double)wr[c] * x[c];
    y[r] = (float)acc;
  }
}

void rmsnorm(float* x, int n) {
  double ss = 0.0;
  for (int i = 0; i < n; ++i) ss += (double)x[i] * x[i];
  const float inv = 1.0f / std::sqrt((float)(ss / n) + RMS_EPS);
  for (int i = 0; i < n; ++i) x[i] *= inv;
}

// One decode step of all layers.  `backend` selects the attention path:
// cuda_backend ops, or the oracle's decode step on the CPU.
bool forward(cuda_backend::Context* ctx, const Weights& W, float* hidden, int pos,
             float (*kc)[MAX_SEQ_LEN][K_DIM], float (*vc)[MAX_SEQ_LEN][K_DIM],
             std::vector<float>& scores) {
  static float scratch[HIDDEN_DIM], q[HIDDEN_DIM], k[K_DIM], v[K_DIM], context[HIDDEN_DIM];
  static float attn_out[HIDDEN_DIM], gate[INTER_DIM], up[INTER_DIM], ffn_out[HIDDEN_DIM];
  for (int layer = 0; layer < NUM_LAYERS; ++layer) {
    std::memcpy(scratch, hidden, sizeof(scratch));
    rmsnorm(scratch, HIDDEN_DIM);
    if (ctx) {
      cuda_backend::metal_batch_begin(*ctx);
      cuda_backend::fused_qkv_op(*ctx, W.wq.data(), W.wk.data(), W.wv.data(), scratch, q, k, v,
                                 HIDDEN_DIM, K_DIM, K_DIM, HIDDEN_DIM, true);
      cuda_backend::elem_op(*ctx, 0, q, W.bq.data(), HIDDEN_DIM);
      cuda_backend::elem_op(*ctx, 0, k, W.bk.data(), K_DIM);
      cuda_backend::elem_op(*ctx, 0, v, W.bv.data(), K_DIM);
      cuda_backend::rope_op(*ctx, q, NUM_HEADS, HEAD_DIM, pos, ROPE_BASE);
      cuda_backend::rope_op(*ctx, k, NUM_KV_HEADS, HEAD_DIM, pos, ROPE_BASE);
      cuda_backend::elem_op(*ctx, 2, &kc[layer][pos][0], k, K_DIM);
      cuda_backend::elem_op(*ctx, 2, &vc[layer][pos][0], v, K_DIM);
      cuda_backend::attention_op(*ctx, q, &kc[layer][0][0], &vc[layer][0][0], context,
                                 NUM_HEADS, NUM_KV_HEADS, HEAD_DIM, pos);
      cuda_backend::matmul_q5_0(*ctx, HIDDEN_DIM, HIDDEN_DIM, W.wo.data(), context, attn_out);
      cuda_backend::elem_op(*ctx, 0, hidden, attn_out, HIDDEN_DIM);  // residual1, :1499
      cuda_backend::metal_batch_end();  // hidden valid on the host
      if (ctx->last_status != TG_OK) return false;
    } else {
      tgo_matmul_q(TGO_TYPE_Q5_0, W.wq.data(), scratch, q, HIDDEN_DIM, HIDDEN_DIM);
      tgo_matmul_q(TGO_TYPE_Q5_0, W.wk.data(), scratch, k, K_DIM, HIDDEN_DIM);
      tgo_matmul_q(TGO_TYPE_Q8_0, W.wv.data(), scratch, v, K_DIM, HIDDEN_DIM);
      for (int i = 0; i < HIDDEN_DIM; ++i) q[i] += W.bq[i];
      for (int i = 0; i < K_DIM; ++i) k[i] += W.bk[i], v[i] += W.bv[i];
      tgo_decode_step(q, k, v, &kc[layer][0][0], &vc[layer][0][0], context, NUM_HEADS,
                      NUM_KV_HEADS, HEAD_DIM, pos, ROPE_BASE, scores.data());
      tgo_attn_output(TGO_TYPE_Q5_0, W.wo.data(), context, hidden, hidden, HIDDEN_DIM,
                      HIDDEN_DIM, attn_out);
    }
    std::memcpy(scratch, hidden, sizeof(scratch));
    rmsnorm(scratch, HIDDEN_DIM);
    matvec(W.gate, scratch, gate, INTER_DIM, HIDDEN_DIM);
    matvec(W.up, scratch, up, INTER_DIM, HIDDEN_DIM);
    for (int i = 0; i < INTER_DIM; ++i) gate[i] = gate[i] / (1.0f + std::exp(-gate[i])) * up[i];
    matvec(W.down, gate, ffn_out, HIDDEN_DIM, INTER_DIM);
    for (int i = 0; i < HIDDEN_DIM; ++i) hidden[i] += ffn_out[i];
  }
  return true;
}
}  // namespace

int main(int argc, char** argv) {
  const int n_tok = argc > 1 ? std::atoi(argv[1]) : 8;
  const bool owned = argc > 2 && std::atoi(argv[2]) != 0;
  if (n_tok < 1 || n_tok > MAX_SEQ_LEN) return 2;
  Weights W;
  const float sh = 1.0f / std::sqrt((float)HIDDEN_DIM), si = 1.0f / std::sqrt((float)INTER_DIM);
  // Block scales so that a row's dot product with a unit-RMS input is O(1).
  fill_blocks(W.wq, TGO_TYPE_Q5_0, HIDDEN_DIM, HIDDEN_DIM, 11, 0.004f);
  fill_blocks(W.wk, TGO_TYPE_Q5_0, K_DIM, HIDDEN_DIM, 12, 0.004f);
  fill_blocks(W.wv, TGO_TYPE_Q8_0, K_DIM, HIDDEN_DIM, 13, 0.0005f);
  fill_blocks(W.wo, TGO_TYPE_Q5_0, HIDDEN_DIM, HIDDEN_DIM, 17, 0.004f);
  fill(W.bq, HIDDEN_DIM, 14, 0.1f);
  fill(W.bk, K_DIM, 15, 0.1f);
  fill(W.bv, K_DIM, 16, 0.1f);
  fill(W.gate, (size_t)INTER_DIM * HIDDEN_DIM, 18, sh);
  fill(W.up, (size_t)INTER_DIM * HIDDEN_DIM, 19, sh);
  fill(W.down, (size_t)HIDDEN_DIM * INTER_DIM, 20, si);

  cuda_backend::Context g_ctx;
  if (!cuda_backend::init(g_ctx)) {
    std::printf("FAIL: init\n");
    return 1;
  }
  if (owned) {
    cuda_backend::register_device_owned(g_ctx, g_k_cache, sizeof(g_k_cache));
    cuda_backend::register_device_owned(g_ctx, g_v_cache, sizeof(g_v_cache));
  }
  // The model's weights: uploaded once (the reference wraps the mapped
  // model file with no-copy buffers, metal_backend.hpp:52-65).
  for (std::vector<uint8_t>* w : {&W.wq, &W.wk, &W.wv, &W.wo})
    cuda_backend::register_device_owned(g_ctx, w->data(), w->size());
  std::vector<float> scores(MAX_SEQ_LEN);
  std::vector<float> hid_gpu(HIDDEN_DIM), hid_cpu(HIDDEN_DIM);
  double worst = 0.0;
  for (int pos = 0; pos < n_tok; ++pos) {
    // Token embedding stub: a seeded vector per position, the same for both.
    tgo_fill_normal(0xE000ULL + pos, hid_gpu.data(), HIDDEN_DIM);
    std::memcpy(hid_cpu.data(), hid_gpu.data(), HIDDEN_DIM * sizeof(float));
    if (!forward(&g_ctx, W, hid_gpu.data(), pos, g_k_cache, g_v_cache, scores)) {
      std::printf("FAIL: backend status %d at pos %d\n", g_ctx.last_status, pos);
      return 1;
    }
    forward(nullptr, W, hid_cpu.data(), pos, o_k_cache, o_v_cache, scores);
    double scale = 0.0, diff = 0.0;
    for (int i = 0; i < HIDDEN_DIM; ++i) {
      scale = std::fmax(scale, std::fabs((double)hid_cpu[i]));
      diff = std::fmax(diff, std::fabs((double)hid_gpu[i] - hid_cpu[i]));
    }
    worst = std::fmax(worst, diff / scale);
  }
  cuda_backend::shutdown(g_ctx);
  // Each layer's attention agrees with the oracle to ~1e-6 relative; 24
  // layers of residual updates keep the hidden state within 1e-4 of it.
  const bool ok = worst <= 1e-4;
  std::printf("%s: %d tokens x %d layers through the backend, max |hidden - oracle loop| / "
              "max |hidden| = %.3g\n",
              ok ? "PASS" : "FAIL", n_tok, NUM_LAYERS, worst);
  return ok ? 0 : 1;
}
