// cuda_backend.hpp -- C++ mirror of the reference's metal_backend operator
// surface for the attention hot path, over the C ABI of tg_cuda_backend.h.
//
// tmac_gguf.cpp drives the Q/K/V projection, RoPE, the KV cache-write and
// decode attention through metal_backend::{init, shutdown,
// metal_batch_begin, metal_batch_end, fused_qkv_op, matmul_q5_0,
// matmul_q8_0, rope_op, elem_op, attention_op} (metal_backend.hpp:114-191,
// :320-338, :354-489, :519-520).  This header offers the same functions, with the same names,
// argument order and meaning, in namespace cuda_backend, so the forward loop
// (tmac_gguf.cpp:1490-1496, :1562-1568) switches backend with a namespace
// alias.  Error behaviour follows the reference: init returns bool and
// prints on failure, the dispatch helpers return void; in addition each
// call's status is kept in Context::last_status and printed as an [ERROR]
// line, where the Metal helpers fail silently.
//
// Host arrays behave as with Metal's no-copy buffers: results written by
// ops are valid in host memory after metal_batch_end().  Arrays only GPU
// ops write (g_k_cache / g_v_cache in the fused path) can be registered as
// device-owned with register_device_owned() so they are not copied back and
// forth every batch.
#pragma once

#include <cstdio>

#include "tg_cuda_backend.h"

namespace cuda_backend {

struct Context {
  tg_context* tg = nullptr;
  int device = 0;
  int last_status = TG_OK;
  bool initialized = false;
};

namespace detail {
inline Context*& current() {
  static thread_local Context* c = nullptr;  // the batch opened on this thread
  return c;
}
inline void report(Context& ctx, int st, const char* what) {
  ctx.last_status = st;
  if (st != TG_OK)
    std::fprintf(stderr, "[ERROR] cuda_backend::%s: %s (%s)\n", what, tg_status_string(st),
                 tg_last_error());
}
}  // namespace detail

// metal_backend::init (metal_backend.cpp:21-89).
inline bool init(Context& ctx, int device = 0) {
  if (ctx.initialized) return true;
  int st = tg_init(device, &ctx.tg);
  detail::report(ctx, st, "init");
  if (st != TG_OK) return false;
  ctx.device = device;
  ctx.initialized = true;
  std::printf("[CUDA] backend %s on device %d\n", tg_version(), device);
  return true;
}

// metal_backend::shutdown.
inline void shutdown(Context& ctx) {
  if (!ctx.initialized) return;
  tg_shutdown(ctx.tg);
  ctx.tg = nullptr;
  ctx.initialized = false;
}

// metal_batch_begin (metal_backend.hpp:114).
inline void metal_batch_begin(Context& ctx, bool reset_offset = true) {
  (void)reset_offset;
  detail::current() = &ctx;
  detail::report(ctx, tg_batch_begin(ctx.tg), "metal_batch_begin");
}

// metal_batch_end (metal_backend.hpp:176): wait, copy results to host arrays.
inline void metal_batch_end() {
  Context* c = detail::current();
  if (!c) return;
  detail::report(*c, tg_batch_end(c->tg), "metal_batch_end");
  detail::current() = nullptr;
}

// rope_op (metal_backend.hpp:381).
inline void rope_op(Context& ctx, float* data, int n_heads, int head_dim, int pos, float base) {
  detail::report(ctx, tg_rope_op(ctx.tg, data, n_heads, head_dim, pos, base), "rope_op");
}

// elem_op (metal_backend.hpp:354): op 0 add, op 2 copy (the cache-write).
inline void elem_op(Context& ctx, int op, float* data, const float* aux, int dim) {
  detail::report(ctx, tg_elem_op(ctx.tg, op, data, aux, dim), "elem_op");
}

// attention_op (metal_backend.hpp:413).
inline void attention_op(Context& ctx, const float* Q, const float* K_cache,
                         const float* V_cache, float* output, int n_head, int n_kv_head,
                         int head_dim, int past_len) {
  detail::report(ctx,
                 tg_attention_op(ctx.tg, Q, K_cache, V_cache, output, n_head, n_kv_head,
                                 head_dim, past_len),
                 "attention_op");
}

// fused_qkv_op (metal_backend.hpp:456): y_q = W_q x, y_k = W_k x, y_v = W_v x
// with W_q / W_k in Q5_0 and W_v in Q5_0 or Q8_0 blocks.
inline void fused_qkv_op(Context& ctx, const uint8_t* W_q, const uint8_t* W_k,
                         const uint8_t* W_v, const float* x, float* y_q, float* y_k, float* y_v,
                         int q_rows, int k_rows, int v_rows, int cols, bool v_is_q8) {
  detail::report(ctx,
                 tg_fused_qkv_op(ctx.tg, W_q, W_k, W_v, x, y_q, y_k, y_v, q_rows, k_rows,
                                 v_rows, cols, v_is_q8 ? 1 : 0),
                 "fused_qkv_op");
}

// matmul_q5_0 / matmul_q8_0 (metal_backend.hpp:320-338): y = W x.
inline void matmul_q5_0(Context& ctx, int rows, int cols, const uint8_t* w, const float* x,
                        float* y) {
  detail::report(ctx, tg_matmul_q(ctx.tg, TG_WTYPE_Q5_0, rows, cols, w, x, y), "matmul_q5_0");
}
inline void matmul_q8_0(Context& ctx, int rows, int cols, const uint8_t* w, const float* x,
                        float* y) {
  detail::report(ctx, tg_matmul_q(ctx.tg, TG_WTYPE_Q8_0, rows, cols, w, x, y), "matmul_q8_0");
}

// Mark a host array (e.g. the static g_k_cache) as written only by GPU ops.
inline void register_device_owned(Context& ctx, void* host_ptr, size_t bytes) {
  detail::report(ctx, tg_register_host(ctx.tg, host_ptr, bytes, TG_REGION_DEVICE_OWNED),
                 "register_device_owned");
}

// Copy a device-owned array (or part of it) back to host memory.
inline void download(Context& ctx, void* host_ptr, size_t bytes) {
  detail::report(ctx, tg_region_sync(ctx.tg, host_ptr, bytes, 0), "download");
}

}  // namespace cuda_backend
