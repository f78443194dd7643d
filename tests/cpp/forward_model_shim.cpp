// The decode step of the reference's forward loop (tmac_gguf.cpp:1453-1516,
// forward_all_layers_fused) on Linux with this library as the attention
// backend: per layer RMSNorm -> Q/K/V matvecs + biases -> RoPE -> cache-write
// -> attention -> output matvec -> residual -> RMSNorm -> gate/up -> SiLU ->
// down -> residual.  The attention-path ops (rope_op, elem_op(2),
// attention_op inside metal_batch_begin / metal_batch_end) go through
// cuda_backend.hpp with the reference's arguments and host arrays; the
// weight matvecs, norms and SiLU are host-side fp32 stubs with seeded
// weights of Qwen2-0.5B's shapes (one weight set shared by all layers, to
// keep the program small).  The same loop is run a second time with the
// CPU oracle's decode step (tg_oracle.c, the restatement of
// tmac_gguf.cpp:990-1016 and :1090-1128) in place of the backend, and the
// hidden states after every token are compared.  Prints PASS / FAIL.
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
  std::vector<float> wq, wk, wv, bq, bk, bv, wo, gate, up, down;
};

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
    matvec(W.wq, scratch, q, HIDDEN_DIM, HIDDEN_DIM);
    matvec(W.wk, scratch, k, K_DIM, HIDDEN_DIM);
    matvec(W.wv, scratch, v, K_DIM, HIDDEN_DIM);
    for (int i = 0; i < HIDDEN_DIM; ++i) q[i] += W.bq[i];
    for (int i = 0; i < K_DIM; ++i) k[i] += W.bk[i], v[i] += W.bv[i];
    if (ctx) {
      cuda_backend::metal_batch_begin(*ctx);
      cuda_backend::rope_op(*ctx, q, NUM_HEADS, HEAD_DIM, pos, ROPE_BASE);
      cuda_backend::rope_op(*ctx, k, NUM_KV_HEADS, HEAD_DIM, pos, ROPE_BASE);
      cuda_backend::elem_op(*ctx, 2, &kc[layer][pos][0], k, K_DIM);
      cuda_backend::elem_op(*ctx, 2, &vc[layer][pos][0], v, K_DIM);
      cuda_backend::attention_op(*ctx, q, &kc[layer][0][0], &vc[layer][0][0], context,
                                 NUM_HEADS, NUM_KV_HEADS, HEAD_DIM, pos);
      cuda_backend::metal_batch_end();  // context valid on the host
      if (ctx->last_status != TG_OK) return false;
    } else {
      tgo_decode_step(q, k, v, &kc[layer][0][0], &vc[layer][0][0], context, NUM_HEADS,
                      NUM_KV_HEADS, HEAD_DIM, pos, ROPE_BASE, scores.data());
    }
    matvec(W.wo, context, attn_out, HIDDEN_DIM, HIDDEN_DIM);
    for (int i = 0; i < HIDDEN_DIM; ++i) hidden[i] += attn_out[i];
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
  fill(W.wq, (size_t)HIDDEN_DIM * HIDDEN_DIM, 11, sh);
  fill(W.wk, (size_t)K_DIM * HIDDEN_DIM, 12, sh);
  fill(W.wv, (size_t)K_DIM * HIDDEN_DIM, 13, sh);
  fill(W.bq, HIDDEN_DIM, 14, 0.1f);
  fill(W.bk, K_DIM, 15, 0.1f);
  fill(W.bv, K_DIM, 16, 0.1f);
  fill(W.wo, (size_t)HIDDEN_DIM * HIDDEN_DIM, 17, sh);
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
