/*
 * tg_cuda_backend.h -- C ABI of the B200 (sm_100a) decode-attention backend.
 *
 * Drop-in for the attention hot path of tmac_gguf.cpp: the reference's
 * forward loop (tmac_gguf.cpp:1490-1496, :1562-1568) drives RoPE, the KV
 * cache-write and GQA decode attention through metal_backend::{rope_op,
 * elem_op, attention_op, metal_batch_begin, metal_batch_end}; each of those
 * has an entry point here with the same argument order and meaning.  On top
 * of that surface the library adds what the reference does not have:
 * device-resident KV caches, batched variable-length decode, bf16 caches
 * and split-KV decode across GPUs.
 *
 * Conventions
 *  - Every function returns an int status: TG_OK (0) or a TG_ERR_* code;
 *    tg_last_error() gives a message for the calling thread.  (The reference
 *    dispatch helpers return void and report nothing.)
 *  - A tg_context binds one CUDA device and one stream.  It is not
 *    thread-safe: use one context per host thread.
 *  - Pointers may be CUDA device (or managed) pointers, used in place, or
 *    host pointers, which the library stages through device memory.  A call
 *    that reads or writes host memory returns when its host outputs are
 *    valid (or, inside a batch, at tg_batch_end); a call on device pointers
 *    only is stream-ordered and asynchronous, and errors that kernels
 *    detect surface at the next tg_synchronize or tg_batch_end.  For
 *    the reference-compatible ops (tg_rope_op, tg_elem_op, tg_attention_op)
 *    host arrays get persistent device mirrors, like the reference's buffer
 *    wrapper cache (metal_backend.hpp:44-65); results in host arrays are
 *    valid after tg_batch_end (or on return when no batch is open), exactly
 *    when Metal results are valid after metal_batch_end.  Host buffers that
 *    a call inside a batch writes (outputs, in-place q / k) must stay
 *    allocated until tg_batch_end: page-locked ones are written there.
 *    Host inputs are read at the call and may be reused at once.
 *  - Shapes: head_dim even and <= 128, n_head a multiple of n_kv_head,
 *    n_head*head_dim <= 4096.  The tensor-core path serves bf16 caches with
 *    head_dim 64, n_kv_head in {1,2,4} and n_head/n_kv_head <= 8 (Qwen2-0.5B:
 *    14 / 2 / 64); other shapes run on the CUDA-core kernel.
 */
#ifndef TG_CUDA_BACKEND_H
#define TG_CUDA_BACKEND_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TG_API __attribute__((visibility("default")))
#else
#define TG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define TG_OK 0
#define TG_ERR_INVALID_ARG 1   /* bad shape, null pointer, out-of-range pos */
#define TG_ERR_CUDA 2          /* a CUDA runtime call failed */
#define TG_ERR_NO_DEVICE 3
#define TG_ERR_OUT_OF_MEMORY 4
#define TG_ERR_UNSUPPORTED 5   /* e.g. elem_op op 1 (SiLU*up): not this path */
#define TG_ERR_DEVICE 6        /* a kernel reported an error (bad position,
                                  a bounded wait expired) */
#define TG_ERR_COMM 7          /* NCCL unavailable or failed */
#define TG_ERR_STATE 8         /* call order (batch_end without begin, ...) */

/* KV cache element types */
#define TG_DTYPE_F32 0
#define TG_DTYPE_BF16 1

/* tg_register_host flags */
#define TG_REGION_MIRROR 0        /* host copy is authoritative */
#define TG_REGION_DEVICE_OWNED 1  /* device copy is authoritative */

typedef struct tg_context tg_context;
typedef struct tg_kv_cache tg_kv_cache;
typedef struct tg_graph tg_graph;

TG_API const char* tg_status_string(int status);
/* Message of the last failing call on this thread ("" if none). */
TG_API const char* tg_last_error(void);
/* Library version string. */
TG_API const char* tg_version(void);

/* ------------------------------------------------------ context / batches */

/* metal_backend::init (metal_backend.hpp:519, metal_backend.cpp:21-89).
 * Binds `device`, creates a stream and the device error word. */
TG_API int tg_init(int device, tg_context** out_ctx);
/* metal_backend::shutdown (metal_backend.hpp:520).  Synchronises, frees
 * everything the context owns. */
TG_API int tg_shutdown(tg_context* ctx);
/* Use an existing cudaStream_t (e.g. a framework's stream) for all work. */
TG_API int tg_set_stream(tg_context* ctx, void* cuda_stream);
TG_API int tg_get_stream(tg_context* ctx, void** cuda_stream);
/* Number of SMs of the bound device. */
TG_API int tg_device_sms(tg_context* ctx, int* out_sms);

/* metal_batch_begin (metal_backend.hpp:114-122): subsequent ops are queued
 * on the context stream and host-array results are deferred. */
TG_API int tg_batch_begin(tg_context* ctx);
/* metal_batch_end (metal_backend.hpp:176-191): copies back host arrays the
 * batch wrote, waits for the stream and reports device errors. */
TG_API int tg_batch_end(tg_context* ctx);
/* Wait for the stream and report device errors (no batch semantics). */
TG_API int tg_synchronize(tg_context* ctx);

/* CUDA-graph capture of a sequence of calls on device pointers -- the
 * B200 counterpart of encoding a whole forward pass into one Metal command
 * buffer (tmac_gguf.cpp:1468-1515).  Between tg_graph_begin and
 * tg_graph_end, calls are recorded instead of run; host pointers are
 * rejected and scratch must already be sized (run the same calls once
 * before capturing).  NCCL collectives of split-KV calls are captured too.
 * A graph replays its recorded kernels on the context stream. */
TG_API int tg_graph_begin(tg_context* ctx);
TG_API int tg_graph_end(tg_context* ctx, tg_graph** out);
TG_API int tg_graph_launch(tg_context* ctx, tg_graph* g);
TG_API int tg_graph_destroy(tg_graph* g);

/* Device mirror of a host array, the explicit form of wrap_buffer
 * (metal_backend.hpp:52-65).  TG_REGION_DEVICE_OWNED marks arrays only GPU
 * ops write, such as the reference's g_k_cache / g_v_cache
 * (tmac_gguf.cpp:200-201) in the fused path: they are uploaded once here
 * and never copied automatically again. */
TG_API int tg_register_host(tg_context* ctx, void* host_ptr, size_t bytes, int flags);
TG_API int tg_unregister_host(tg_context* ctx, void* host_ptr);
/* Copy [host_ptr, host_ptr+bytes) of a registered array device -> host
 * (or host -> device with to_device = 1). */
TG_API int tg_region_sync(tg_context* ctx, void* host_ptr, size_t bytes, int to_device);

/* ------------------------------------------- reference-compatible ops */

/* rope_op (metal_backend.hpp:381-396; kernel_rope.metal:5-22; CPU
 * apply_rope tmac_gguf.cpp:990-1016): rotate adjacent pairs of n_heads
 * heads of `data` in place at position pos.  Results are bit-identical to
 * the reference CPU code (host-libm cos/sin table, one rounding per
 * product and sum). */
TG_API int tg_rope_op(tg_context* ctx, float* data, int n_heads, int head_dim,
               int pos, float base);

/* elem_op (metal_backend.hpp:354-379; kernel_elem.metal:6-21) for op 0
 * (data += aux) and op 2 (data = aux, the cache-write of
 * tmac_gguf.cpp:1492-1493).  op 1 (SiLU x up, FFN) is not on this path and
 * returns TG_ERR_UNSUPPORTED. */
TG_API int tg_elem_op(tg_context* ctx, int op, float* data, const float* aux, int dim);

/* attention_op (metal_backend.hpp:413-453; kernels kernel_flash_attn.metal /
 * kernel_attn.metal; CPU tmac_gguf.cpp:1093-1128): one query token, n_head
 * query heads over n_kv_head KV heads, fp32 K/V caches laid out
 * [pos][n_kv_head*head_dim] from the layer base, attending rows
 * 0..past_len.  output[h*head_dim + d]. */
TG_API int tg_attention_op(tg_context* ctx, const float* Q, const float* K_cache,
                    const float* V_cache, float* output, int n_head,
                    int n_kv_head, int head_dim, int past_len);

/* ------------------------------------------------- Q/K/V projection */

/* Weight block types (tmac_gguf.cpp:177-182), GGML's 32-element blocks:
 * Q5_0 = fp16 d, 32 high bits, 16 bytes of nibbles (22 bytes); element j
 * < 16 in the low nibble of byte j, j >= 16 in the high nibble of byte
 * j-16; value d*(((hi<<4)|lo) - 16) (dequant_q5_0, :311-328).  Q8_0 =
 * fp16 d, 32 int8 (34 bytes); value d*q (dequant_q8_0, :240-248).  Rows
 * are row-major runs of cols/32 blocks (read_tensor, :402-415). */
#define TG_WTYPE_Q5_0 6
#define TG_WTYPE_Q8_0 8

/* fused_qkv_op (metal_backend.hpp:456-489; kernel_fused_qkv.metal:8-70):
 * y_q = W_q x, y_k = W_k x, y_v = W_v x for one input vector of `cols`
 * values (a multiple of 32); W_q / W_k are Q5_0, W_v is Q5_0 or Q8_0
 * (v_is_q8).  Host or device pointers, weights at least 2-byte aligned;
 * host weight arrays are best registered (tg_register_host,
 * TG_REGION_DEVICE_OWNED) so that they are uploaded once.  The kernel
 * reads the weights before it waits for the kernel launched just before
 * it on the stream, which therefore must not write them. */
TG_API int tg_fused_qkv_op(tg_context* ctx, const uint8_t* W_q, const uint8_t* W_k,
                           const uint8_t* W_v, const float* x, float* y_q, float* y_k,
                           float* y_v, int q_rows, int k_rows, int v_rows, int cols,
                           int v_is_q8);

/* matmul_q5_0 / matmul_q8_0 (metal_backend.hpp:320-338; the CPU path
 * matmul, tmac_gguf.cpp:476-513): y = W x for a rows x cols weight of
 * wtype (TG_WTYPE_*).  Pointer rules as tg_fused_qkv_op. */
TG_API int tg_matmul_q(tg_context* ctx, int wtype, int rows, int cols, const uint8_t* w,
                       const float* x, float* y);

/* The attn_output matvec and its residual add (tmac_gguf.cpp:1497-1499:
 * matmul of blk.N.attn_output.weight, then elem_op(0, hidden, attn_out)):
 * hidden[s] += W_o context[s] for n_seqs sequences, W_o `rows` x `cols` in
 * wtype blocks (Q5_0 or Q8_0: a 896-wide row is not a multiple of the 256
 * values of a K-quant super-block).  The product sum is rounded once, then
 * the add, as the reference does.  context [n_seqs][cols], hidden
 * [n_seqs][rows]; pointer rules as tg_fused_qkv_op. */
TG_API int tg_attn_output(tg_context* ctx, int n_seqs, int wtype, const void* w_o, int rows,
                          int cols, const float* context, float* hidden);

/* Tuning: projections of 9+ sequences run on the tensor cores in clusters
 * of 1 to 8 CTAs that split the columns (chosen per launch from the
 * device's resident-cluster count).  split 1-8 fixes the width for later
 * launches of every context (clamped to cols / 32), 0 restores the
 * automatic choice; other values give TG_ERR_INVALID_ARG.  Results differ
 * between widths only by the order of the fp32 partial sums. */
TG_API int tg_set_projection_split(int split);

/* Tuning of the bf16 decode kernel (no reference counterpart: the
 * reference's attention_op, metal_backend.hpp:413-453, has no knobs).
 * ring_kb: K/V ring per CTA, 128 or 192 KB (0, the default: 128).
 * preload: 1 lets the kernel load its first tiles before its
 * grid-dependency wait on short shards (at most 16 tiles of 64 rows per SM)
 * when the library knows that no kernel still running writes those cache
 * rows; 0 (the default) never.  Both measured slower on B200 at 4 x 131072
 * rows on 1 and 8 GPUs and are kept as tuning knobs.  Applies to later
 * launches of every context; results do not depend on either.  Other
 * values give TG_ERR_INVALID_ARG. */
TG_API int tg_set_decode_tuning(int ring_kb, int preload);

/* One layer's projection weights: W_q has n_head*head_dim rows, W_k and
 * W_v n_kv_head*head_dim rows of `cols` inputs.  Device pointers or
 * registered host arrays; a NULL bias is a bias the model does not have. */
typedef struct tg_qkv_weights {
  int q_type, k_type, v_type; /* TG_WTYPE_* */
  int cols;
  const void* w_q;
  const void* w_k;
  const void* w_v;
  const float* b_q;
  const float* b_k;
  const float* b_v;
} tg_qkv_weights;

/* ------------------------------------------------- model files */

/* A TMAC model file (scripts/extract_tmac.py:6-23: "TMAC", uint64 count,
 * then per tensor uint64 name_len, name, uint64 rows, uint64 cols, uint32
 * GGUF type, uint64 n_bytes, data) loaded into device memory -- load_tmac
 * (tmac_gguf.cpp:1372-1425) with the reference's 512 MB host region
 * replaced by one device allocation (tensors at 256-byte aligned offsets).
 * The table keeps what load_tmac keeps: names cut to 127 characters, rows
 * (outputs), cols (inputs), type and size; the magic is read, not checked,
 * as there.  A truncated file or an unreadable path gives
 * TG_ERR_INVALID_ARG. */
typedef struct tg_model tg_model;
typedef struct tg_tensor_info {
  const char* name;   /* NULL when tg_model_find does not find the name */
  uint64_t rows, cols, n_bytes;
  uint32_t type;      /* GGUF type code: 0 F32, 6 Q5_0, 8 Q8_0, ... */
  const void* data;   /* device address */
} tg_tensor_info;

TG_API int tg_model_load_tmac(tg_context* ctx, const char* path, tg_model** out);
TG_API int tg_model_destroy(tg_model* m);
TG_API int tg_model_count(tg_model* m, int* n_tensors);
TG_API int tg_model_tensor_at(tg_model* m, int index, tg_tensor_info* out);
/* get_tensor_info (tmac_gguf.cpp:417-422): the first tensor of that name;
 * out->name == NULL (status TG_OK) when there is none. */
TG_API int tg_model_find(tg_model* m, const char* name, tg_tensor_info* out);
/* Copy the first `bytes` of tensor `index` to host memory. */
TG_API int tg_model_read(tg_model* m, int index, void* dst, size_t bytes);
/* One layer's attention weights, blk.<layer>.attn_{q,k,v}.weight, the fp32
 * biases blk.<layer>.attn_{q,k,v}.bias (NULL when absent) and
 * blk.<layer>.attn_output.weight (*w_o NULL and *o_type -1 when absent),
 * ready for tg_decode_layer_x / tg_attention_block. */
TG_API int tg_model_layer_attention(tg_model* m, int layer, tg_qkv_weights* w,
                                    const void** w_o, int* o_type);

/* ------------------------------------------------- device KV caches */

/* A device-resident cache replacing the static g_k_cache / g_v_cache
 * (tmac_gguf.cpp:200-201), for n_seqs sequences: K and V are each laid out
 * [n_layers][n_seqs][max_ctx][n_kv_head*head_dim] of `dtype`.  The cache
 * holds global positions [shard_start, shard_start + max_ctx) (shard_start
 * 0 for a whole cache; > 0 for one GPU's shard in split-KV decode).
 * Zero-initialised. */
typedef struct tg_kv_desc {
  int n_layers, n_seqs, max_ctx, n_head, n_kv_head, head_dim, dtype;
  int shard_start;
  int global_ctx;  /* positions over all shards; 0 means shard_start+max_ctx.
                      RoPE accepts positions 0..global_ctx-1. */
  float rope_base; /* RoPE base for this model (1e6 for Qwen2) */
} tg_kv_desc;

TG_API int tg_kv_create(tg_context* ctx, const tg_kv_desc* desc, tg_kv_cache** out);
/* Destroy before tg_shutdown of its context; tg_shutdown frees caches that
 * are still alive, after which their handles must not be used. */
TG_API int tg_kv_destroy(tg_kv_cache* kv);
/* reset_cache (tmac_gguf.cpp:1430-1434): zero both caches. */
TG_API int tg_kv_reset(tg_kv_cache* kv);
/* Device pointers to layer `layer` of K and V ([n_seqs][max_ctx][row]). */
TG_API int tg_kv_layer_ptrs(tg_kv_cache* kv, int layer, void** k, void** v);
/* Fill K and V with synthetic N(0,1) values rounded to the cache type. */
TG_API int tg_kv_fill_normal(tg_kv_cache* kv, uint64_t seed);
/* Write n_rows fp32 rows (host or device) at local rows row0.. of one
 * sequence/layer, converted to the cache type (RNE for bf16). */
TG_API int tg_kv_write_rows(tg_kv_cache* kv, int layer, int seq, int row0,
                     int n_rows, const float* k_rows, const float* v_rows);
/* Read n_rows raw rows (cache type) into host or device memory. */
TG_API int tg_kv_read_rows(tg_kv_cache* kv, int layer, int seq, int row0,
                    int n_rows, void* k_out, void* v_out);

/* ------------------------------------------------- batched decode */

/* RoPE + cache-write for n_seqs sequences (tmac_gguf.cpp:1087-1091; the
 * rope_op x2 + elem_op(2) x2 of :1490-1493 fused into one launch).
 * q [n_seqs][n_head*head_dim] and k_new [n_seqs][n_kv*head_dim] are rotated
 * in place; the rotated k row and v_new are written at each sequence's
 * position pos[s] (global) when this cache holds it. */
TG_API int tg_rope_cache_write(tg_context* ctx, tg_kv_cache* kv, int layer,
                        int n_seqs, float* q, float* k_new,
                        const float* v_new, const int32_t* pos);

/* Decode attention for n_seqs sequences of one layer: sequence s attends
 * rows 0..past_len[s] of its cache (tmac_gguf.cpp:1093-1128 per sequence).
 * q: [n_seqs][n_head*head_dim] (rotated), out: same shape. */
TG_API int tg_attention_batched(tg_context* ctx, tg_kv_cache* kv, int layer,
                         int n_seqs, const float* q, const int32_t* past_len,
                         float* out);

/* The whole per-layer decode step: tg_rope_cache_write then
 * tg_attention_batched with past_len = pos. */
TG_API int tg_decode_layer(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                    float* q, float* k_new, const float* v_new,
                    const int32_t* pos, float* out);

/* The layer step from the normed hidden state to the cache
 * (forward_layer_with_cache, tmac_gguf.cpp:1046-1091; the fused_qkv_op +
 * elem_op(0) x3 + rope_op x2 + elem_op(2) x2 of :1479-1493) in one launch:
 * q/k/v = W x + bias, RoPE of q and k at pos[s], the k and v rows written
 * into the cache at pos[s] (when this cache or shard holds it), rotated q
 * to q_out [n_seqs][n_head*head_dim].  x [n_seqs][w->cols]. */
TG_API int tg_qkv_rope_cache_write(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                                   const tg_qkv_weights* w, const float* x,
                                   const int32_t* pos, float* q_out);

/* tg_qkv_rope_cache_write followed by decode attention over rows
 * 0..pos[s]: the layer from x to the attention context out
 * [n_seqs][n_head*head_dim] (tmac_gguf.cpp:1046-1128), two kernels chained
 * by programmatic dependent launch plus the split-sequence merge. */
TG_API int tg_decode_layer_x(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                             const tg_qkv_weights* w, const float* x, const int32_t* pos,
                             float* out);

/* The attention block of a decode layer, from the normed hidden state x to
 * the residual stream (tmac_gguf.cpp:1479-1499): tg_qkv_rope_cache_write,
 * attention over rows 0..pos[s], then hidden[s] += W_o context[s]
 * (tg_attn_output, o_type blocks; W_o square of n_head*head_dim).  The
 * context stays on the device; hidden [n_seqs][n_head*head_dim] is read and
 * written.  Four kernels chained by programmatic dependent launch. */
TG_API int tg_attention_block(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                              const tg_qkv_weights* w, int o_type, const void* w_o,
                              const float* x, const int32_t* pos, float* hidden);

/* ------------------------------------------------- prefill */

/* Causal prefill of one layer for n_seqs prompts of S tokens (positions
 * 0..S-1).  The reference runs a prompt token by token (process_prompt,
 * tmac_gguf.cpp:1621-1658: one decode step per position); this computes the
 * same attention for all S positions at once on the tcgen05 tensor cores.
 * q [n_seqs][S][n_head*head_dim], k/v [n_seqs][S][n_kv*head_dim] are fp32
 * and un-rotated; RoPE is applied in fp32 exactly as apply_rope
 * (tmac_gguf.cpp:990-1016) and the rotated q, k and v are rounded to bf16.
 * The k and v rows are written to the cache (rows 0..S-1 of each
 * sequence), so decode can continue from position S.  out
 * [n_seqs][S][n_head*head_dim] fp32.  Needs a bf16 cache with head_dim 64
 * that is not a split-KV shard, and S <= max_ctx. */
TG_API int tg_prefill_layer(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, int S,
                            const float* q, const float* k, const float* v, float* out);

/* ------------------------------------------------- split-KV across GPUs */

/* NCCL unique id (128 bytes) for tg_comm_init; call on one rank and share
 * it out of band. */
TG_API int tg_comm_unique_id(void* id_out, size_t id_bytes);
/* Join a world of `world` ranks (one per GPU).  timeout_ms bounds the
 * initialisation and every later collective wait on this context. */
TG_API int tg_comm_init(tg_context* ctx, const void* id, int rank, int world,
                 int timeout_ms);
TG_API int tg_comm_destroy(tg_context* ctx);

/* How the ranks exchange their softmax records in the split-KV calls. */
#define TG_EXCHANGE_AUTO 0  /* peer memory when every GPU maps every other's, else NCCL */
#define TG_EXCHANGE_PEER 1  /* NVLink peer stores of epoch-tagged words in the merge kernel */
#define TG_EXCHANGE_NCCL 2  /* ncclAllGather of the records, then a merge kernel */
/* Bound, in milliseconds (default 5000), of the merge kernel's wait for the
 * other GPUs' softmax records in the peer exchange.  A wait that runs out
 * ends the kernel with device error 0x105, reported as TG_ERR_DEVICE at the
 * next synchronisation; then destroy and create the communicator again (the
 * ranks' exchange epochs may differ).  No counterpart in the reference
 * (metal_backend.cpp:23-27 only prints). */
TG_API int tg_comm_set_wait_limit_ms(tg_context* ctx, int ms);
/* Choose the exchange (collective: every rank passes the same value before
 * its next split-KV call).  TG_EXCHANGE_PEER fails with TG_ERR_UNSUPPORTED
 * at the next call if peer memory cannot be set up on some rank. */
TG_API int tg_comm_set_exchange(tg_context* ctx, int exchange);
/* The exchange the last split-KV call used: TG_EXCHANGE_PEER,
 * TG_EXCHANGE_NCCL, or TG_EXCHANGE_AUTO before the first call. */
TG_API int tg_comm_exchange(tg_context* ctx, int* exchange);

/* Split-KV (flash-decoding) step across the world: each rank holds a shard
 * of every sequence's positions (its kv cache's [shard_start,
 * shard_start+max_ctx)), computes the softmax partials of its shard, the
 * ranks exchange them (peer memory or NCCL, see above) and every rank
 * merges the same result into out.  Inputs and outputs are replicated on
 * all ranks. */
TG_API int tg_attention_splitkv(tg_context* ctx, tg_kv_cache* shard, int layer,
                         int n_seqs, const float* q, const int32_t* past_len,
                         float* out);

/* The two halves of tg_attention_splitkv, for callers that move the
 * partials themselves.  tg_attention_records writes, per sequence, the
 * softmax record of this cache's shard: records[s] = { o[n_head][head_dim]
 * (un-normalised), m[n_head] (running max, log2 units), l[n_head] } --
 * n_head*(head_dim+2) floats.  tg_merge_records combines n_parts such
 * record arrays, laid out [n_parts][n_seqs][record], into out. */
TG_API int tg_attention_records(tg_context* ctx, tg_kv_cache* shard, int layer,
                                int n_seqs, const float* q,
                                const int32_t* past_len, float* records);
TG_API int tg_merge_records(tg_context* ctx, int n_parts, int n_seqs,
                            int n_head, int head_dim, const float* records,
                            float* out);

/* RoPE + owner cache-write + split-KV attention, one layer. */
TG_API int tg_decode_layer_splitkv(tg_context* ctx, tg_kv_cache* shard, int layer,
                            int n_seqs, float* q, float* k_new,
                            const float* v_new, const int32_t* pos,
                            float* out);

/* tg_decode_layer_x on a split-KV shard: every rank projects the replicated
 * q from x (same weights and x on every rank), the rank whose shard holds
 * pos[s] writes the k / v row, then the split-KV attention, exchange and
 * merge of tg_decode_layer_splitkv give every rank the full output. */
TG_API int tg_decode_layer_splitkv_x(tg_context* ctx, tg_kv_cache* shard, int layer,
                                     int n_seqs, const tg_qkv_weights* w, const float* x,
                                     const int32_t* pos, float* out);

/* tg_attention_block on a split-KV shard: the attention as
 * tg_decode_layer_splitkv_x, then every rank applies the attn_output
 * matvec to the replicated context (identical hidden on every rank). */
TG_API int tg_attention_block_splitkv(tg_context* ctx, tg_kv_cache* shard, int layer,
                                      int n_seqs, const tg_qkv_weights* w, int o_type,
                                      const void* w_o, const float* x, const int32_t* pos,
                                      float* hidden);

/* ------------------------------------------------- allocation-free decode */

/* No counterpart in the reference.  Decode attention for callers that cannot
 * allocate device memory when they run it: code recording a CUDA graph in
 * global capture mode (allocation calls are refused there), runtimes that
 * own a fixed memory pool and forbid the driver allocator after start-up,
 * or an allocator hook that must not re-enter itself.  It calls no
 * cudaMalloc / cudaFree: the split-KV scratch (partial softmax records, tile
 * schedule, error word) is one fixed device array of
 * TG_NOALLOC_SCRATCH_BYTES inside the library, held by every GPU that loads
 * the library until the process exits.  It works on the calling thread's
 * current device; if that device's primary context is not yet set up, the
 * first call sets it up (as any CUDA runtime call does), so make the first
 * call before any stream capture.
 *
 * Same work as tg_attention_batched on one layer: sequence s attends rows
 * 0..past_len[s] of its cache rows [s][max_ctx][n_kv_head*head_dim] of
 * `dtype`.  All pointers are device memory; the work is queued on
 * cuda_stream (a cudaStream_t, 0 = legacy default stream) and the call does
 * not wait.  n_seqs may be at most TG_NOALLOC_MAX_SEQS; larger batches are
 * refused with TG_ERR_INVALID_ARG.  If device_status is not null, the
 * kernels' error word (0, or 0x103 for a position outside the cache) is
 * copied there once the work has run.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current and raises the
 * shared-memory limit of every kernel variant it can launch; make it before
 * any stream capture.  bf16 caches with head_dim 64 take the tensor-core
 * kernel when both caches are 16-byte aligned, else the CUDA-core kernel.
 * All calls share the array and it keeps the last call's contents, so calls
 * whose GPU work overlaps (other streams or threads) race: serialise them. */
#define TG_NOALLOC_MAX_SEQS 4096
#define TG_NOALLOC_SCRATCH_BYTES ((4u << 20) + 16896u)
TG_API int tg_attention_noalloc(void* cuda_stream, const float* q, const void* k_cache,
                                const void* v_cache, int dtype, int n_seqs, int max_ctx,
                                int n_head, int n_kv_head, int head_dim,
                                const int32_t* past_len, float* out, int* device_status);

/* ------------------------------------------------- introspection */

/* Kernel launches this context has issued since creation (all kinds). */
TG_API int tg_launch_count(tg_context* ctx, long long* out);
/* CUDA-event timing of kernel launches on the context stream (events
 * recorded just before and after each launch, also into a graph being
 * captured, so that replays re-record them).  `on` selects the kernels: a
 * mask of TG_PROFILE_ATTENTION (the decode / prefill attention kernels; 1,
 * so that a true value keeps its meaning) and TG_PROFILE_PROJECTION (the
 * Q/K/V projection kernel); 0 stops recording.  Enabling resets the
 * record; tg_profile_read waits for the stream and returns the summed time
 * of the recorded launches (for a graph: of its latest replay) and their
 * number. */
#define TG_PROFILE_ATTENTION 1
#define TG_PROFILE_PROJECTION 2
/* TG_PROFILE_STAMPS: the CTAs of each bf16 decode step record %globaltimer
 * values (ns) -- decode CTAs: start, grid dependency released, tile loop
 * done, end; merge CTAs: start, grid dependency released, first record
 * slice stored to the peers (split-KV), end.
 * Unlike events this keeps the launches' programmatic overlap, so it times
 * the kernels as they run inside a step.  Up to TG_STAMP_LAUNCHES decode
 * steps are recorded after enabling (also into a graph being captured;
 * each replay rewrites them). */
#define TG_PROFILE_STAMPS 4
#define TG_STAMP_LAUNCHES 1024
TG_API int tg_profile_enable(tg_context* ctx, int on);
TG_API int tg_profile_read(tg_context* ctx, double* total_ms, long long* launches);
/* Waits for the stream and copies the stamps into out (at most cap_words
 * values): [step][row][4], steps in enqueue order, rows = 3 x the SM count
 * (*rows): decode CTA c in row c, merge CTA m in row SMs + m, absent CTAs
 * 0.  *n_launches: the recorded steps. */
TG_API int tg_profile_read_stamps(tg_context* ctx, unsigned long long* out, size_t cap_words,
                                  int* n_launches, int* rows);
/* 1 if the next batched decode on `kv` uses the tensor-core kernel. */
TG_API int tg_kv_uses_tensor_cores(tg_kv_cache* kv, int* out);

#ifdef __cplusplus
}
#endif
#endif /* TG_CUDA_BACKEND_H */
