// Drives the attention part of the reference's fused forward loop
// (tmac_gguf.cpp:1490-1496 / :1562-1568) through cuda_backend.hpp -- the
// same calls, argument order and host arrays the reference passes to
// metal_backend -- and checks every layer's context against the CPU oracle
// (tg_oracle.c, the restatement of tmac_gguf.cpp:990-1016 and :1090-1128).
// Prints PASS / FAIL like the reference's standalone test programs.
//
// usage: forward_loop_shim <n_tokens> <device_owned 0|1>
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
constexpr int MAX_SEQ_LEN = 256;
// The reference's static caches (tmac_gguf.cpp:200-201) and an oracle copy.
float g_k_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float g_v_cache[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float ref_k[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
float ref_v[NUM_LAYERS][MAX_SEQ_LEN][K_DIM];
// Per-layer vectors: the CPU fills them before the batch (in the reference
// the fused QKV kernel produces them inside the command buffer).
float q_vec[NUM_LAYERS][HIDDEN_DIM], k_new[NUM_LAYERS][K_DIM], v_new[NUM_LAYERS][K_DIM];
float context[NUM_LAYERS][HIDDEN_DIM];
}  // namespace

int main(int argc, char** argv) {
  const int n_tok = argc > 1 ? std::atoi(argv[1]) : 40;
  const bool owned = argc > 2 && std::atoi(argv[2]) != 0;
  if (n_tok < 1 || n_tok > MAX_SEQ_LEN) return 2;
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
  double worst = 0.0;
  long bad_bits = 0;
  for (int pos = 0; pos < n_tok; ++pos) {
    std::vector<float> exp_ctx(NUM_LAYERS * HIDDEN_DIM), exp_q(NUM_LAYERS * HIDDEN_DIM);
    for (int layer = 0; layer < NUM_LAYERS; ++layer) {
      const uint64_t s = 0x1234ULL ^ ((uint64_t)layer << 32) ^ ((uint64_t)pos << 8);
      tgo_fill_normal(s ^ (1ULL << 56), q_vec[layer], HIDDEN_DIM);
      tgo_fill_normal(s ^ (2ULL << 56), k_new[layer], K_DIM);
      tgo_fill_normal(s ^ (3ULL << 56), v_new[layer], K_DIM);
      float q[HIDDEN_DIM], k[K_DIM];
      std::memcpy(q, q_vec[layer], sizeof(q));
      std::memcpy(k, k_new[layer], sizeof(k));
      tgo_decode_step(q, k, v_new[layer], &ref_k[layer][0][0], &ref_v[layer][0][0],
                      &exp_ctx[layer * HIDDEN_DIM], NUM_HEADS, NUM_KV_HEADS, HEAD_DIM, pos,
                      1000000.0f, scores.data());
      std::memcpy(&exp_q[layer * HIDDEN_DIM], q, sizeof(q));
    }
    cuda_backend::metal_batch_begin(g_ctx);
    for (int layer = 0; layer < NUM_LAYERS; ++layer) {
      cuda_backend::rope_op(g_ctx, q_vec[layer], NUM_HEADS, HEAD_DIM, pos, 1000000.0f);
      cuda_backend::rope_op(g_ctx, k_new[layer], NUM_KV_HEADS, HEAD_DIM, pos, 1000000.0f);
      cuda_backend::elem_op(g_ctx, 2, &g_k_cache[layer][pos][0], k_new[layer], K_DIM);
      cuda_backend::elem_op(g_ctx, 2, &g_v_cache[layer][pos][0], v_new[layer], K_DIM);
      cuda_backend::attention_op(g_ctx, q_vec[layer], &g_k_cache[layer][0][0],
                                 &g_v_cache[layer][0][0], context[layer], NUM_HEADS,
                                 NUM_KV_HEADS, HEAD_DIM, pos);
    }
    cuda_backend::metal_batch_end();
    if (g_ctx.last_status != TG_OK) {
      std::printf("FAIL: status %d at pos %d\n", g_ctx.last_status, pos);
      return 1;
    }
    for (int layer = 0; layer < NUM_LAYERS; ++layer) {
      for (int i = 0; i < HIDDEN_DIM; ++i) {
        const double e = std::fabs((double)context[layer][i] - exp_ctx[layer * HIDDEN_DIM + i]);
        if (e > worst) worst = e;
        if (std::memcmp(&q_vec[layer][i], &exp_q[layer * HIDDEN_DIM + i], 4)) ++bad_bits;
      }
    }
  }
  if (owned) {
    cuda_backend::download(g_ctx, g_k_cache, sizeof(g_k_cache));
    cuda_backend::download(g_ctx, g_v_cache, sizeof(g_v_cache));
  }
  if (std::memcmp(g_k_cache, ref_k, sizeof(g_k_cache)) ||
      std::memcmp(g_v_cache, ref_v, sizeof(g_v_cache)))
    ++bad_bits;
  cuda_backend::shutdown(g_ctx);
  const bool ok = worst <= 1e-4 && bad_bits == 0;
  std::printf("%s: %d tokens x %d layers, max|ctx - oracle| = %.3g, rope/cache bit mismatches = %ld\n",
              ok ? "PASS" : "FAIL", n_tok, NUM_LAYERS, worst, bad_bits);
  return ok ? 0 : 1;
}
