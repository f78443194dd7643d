// tg_qkv.cu -- the Q/K/V projection of a decode step (sm_100a: CUDA cores for
// small batches and very wide rows, tcgen05 tensor cores for batches).
//
//   qkv_kernel   y_m = W_m x for the layer's three projection matrices and B
//                input vectors, weights in the model file's 32-element
//                blocks (GGML Q5_0 / Q8_0, tmac_gguf.cpp:240-248, :311-328;
//                kernel_fused_qkv.metal:8-70).  Mode 0 writes y_m as
//                fused_qkv_op / matmul_q5_0 / matmul_q8_0 do
//                (metal_backend.hpp:320-338, :456-489); mode 2 adds W x to
//                y in place, the attn_output matvec with its residual add
//                (tmac_gguf.cpp:1497-1499).  Mode 1 fuses the
//                rest of the layer step up to attention
//                (tmac_gguf.cpp:1067-1091): the bias adds, RoPE of q and k
//                at each sequence's position (cos/sin from the host-libm
//                table, one rounding per product and sum), the k / v rows
//                written into the cache and the rotated q written out for
//                the attention kernel.
//
// Decomposition: CTA (c, g) takes kQkvRows = 8 consecutive rows of one matrix
// and kQkvSeqs = 64 sequences (grid.y = ceil(B / 64)).  It copies the rows'
// raw blocks into shared memory with 16-byte loads (all of a thread's loads
// issued before any store).  Warp w then owns row w and lane l its 32-element
// block l: the lane decodes the block once into 32 registers (exact: an fp16
// scale times a small integer) and, per sequence, multiplies it with the
// matching 32 inputs (eight float4 loads issued together), two sequences at a
// time; a shuffle reduction over the lanes finishes each sum.  Rows longer
// than 32 blocks loop over groups of 32 blocks and decode per sequence.  The
// epilogue runs over (sequence, row pair).
//
//   qkv_tc_kernel  the same contract for batches of kQkvGemmMinB or more
//                sequences with rows of up to qkv_tc_max_cols() inputs, on
//                the tensor cores (3xTF32 products accumulated in TMEM,
//                clusters of 1-8 CTAs splitting the columns; described at
//                the kernel).
//
//   qkv_gemm_kernel  the same contract for such batches whose rows are
//                wider than the tensor-core kernel takes: a CTA covers
//                kQkvGemmRows = 16 rows x 64
//                sequences.  The rows are decoded once into a K-major fp32
//                tile in shared memory, x is staged transposed 32 columns
//                at a time (double-buffered through registers), and every
//                thread accumulates a 4-row x 2-sequence register tile over
//                K (one broadcast LDS.128 of weights and one LDS.64 of inputs
//                feed 8 FMAs), so no sum needs a cross-lane reduction and
//                each x value is read from memory once per CTA.  The
//                epilogue works from registers (a RoPE pair is two of the
//                thread's rows).
//
// PDL: the weight copy and decode come before griddepcontrol.wait, so they
// overlap the previous kernel on the stream (weights are constants of the
// model; the C ABI requires that the kernel launched just before a
// projection does not write its weights).  x, the outputs and the caches are
// touched only after the wait.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "tg_device.cuh"
#include "tg_tc.cuh"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace tg {

namespace cg = cooperative_groups;

namespace {

constexpr int QKV_THREADS = kQkvRows * 32;

struct QkvSmem {
  int raw_bytes;   // staged blocks of kQkvRows rows (16-byte multiple)
  int y_off;       // dot products [kQkvSeqs][kQkvRows]
  int total;
};

__host__ __device__ inline QkvSmem qkv_smem_layout(int cols) {
  QkvSmem L;
  const int max_row = (cols / 32) * 34;  // the larger block type
  L.raw_bytes = ((kQkvRows * max_row) + 15) & ~15;
  L.y_off = L.raw_bytes;
  L.total = L.y_off + kQkvSeqs * kQkvRows * 4;
  return L;
}

// f16_to_f32 of tmac_gguf.cpp:220-232: the exact widening, except that a
// zero of either sign becomes +0 (:225).
__device__ __forceinline__ float f16_scale(uint16_t h) {
  if ((h & 0x7fffu) == 0) return 0.0f;
  return __half2float(__ushort_as_half(h));
}

// The 32 values of one block, decoded exactly as dequant_q5_0 /
// dequant_q8_0 (tmac_gguf.cpp:311-328, :240-248).  blk is 2-byte aligned.
__device__ __forceinline__ void decode_block(const uint8_t* blk, int type, float (&w)[32]) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(blk);
  const float d = f16_scale(h[0]);
  if (type == kWTypeQ5_0) {
    // qh: bit j is the high bit of element j; byte j of qs holds element j
    // (low nibble) and element j + 16 (high nibble).
    const uint32_t qh = (uint32_t)h[1] | ((uint32_t)h[2] << 16);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t two = h[3 + k];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int j = 2 * k + t;
        const uint32_t byte = (two >> (8 * t)) & 0xffu;
        w[j] = d * (float)((int)((((qh >> j) & 1u) << 4) | (byte & 0xfu)) - 16);
        w[j + 16] = d * (float)((int)((((qh >> (j + 16)) & 1u) << 4) | (byte >> 4)) - 16);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t two = h[1 + k];
      w[2 * k] = (float)(int8_t)(two & 0xffu) * d;
      w[2 * k + 1] = (float)(int8_t)(two >> 8) * d;
    }
  }
}

// The 32 inputs of block `blk` of one x row: eight 16-byte loads (vec) or
// 32 scalar loads, all issued before use.
__device__ __forceinline__ void load_x32(const float* x, bool vec, float (&v)[32]) {
  if (vec) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(x) + k);
      v[4 * k] = f.x;
      v[4 * k + 1] = f.y;
      v[4 * k + 2] = f.z;
      v[4 * k + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __ldg(x + k);
  }
}

__device__ __forceinline__ float dot32(const float (&w)[32], const float (&v)[32]) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int k = 0; k < 32; k += 4) {
    a0 = fmaf(w[k], v[k], a0);
    a1 = fmaf(w[k + 1], v[k + 1], a1);
    a2 = fmaf(w[k + 2], v[k + 2], a2);
    a3 = fmaf(w[k + 3], v[k + 3], a3);
  }
  return (a0 + a1) + (a2 + a3);
}

// Elements 16h..16h+15 of one block (h = 0 or 1), decoded as decode_block.
__device__ __forceinline__ void decode_half(const uint8_t* blk, int type, int h, float (&w)[16]) {
  const uint16_t* hw = reinterpret_cast<const uint16_t*>(blk);
  const float d = f16_scale(hw[0]);
  if (type == kWTypeQ5_0) {
    const uint32_t qh = ((uint32_t)hw[1] | ((uint32_t)hw[2] << 16)) >> (16 * h);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t two = hw[3 + k];
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int j = 2 * k + t;
        const uint32_t byte = (two >> (8 * t)) & 0xffu;
        const uint32_t lo = h ? (byte >> 4) : (byte & 0xfu);
        w[j] = d * (float)((int)((((qh >> j) & 1u) << 4) | lo) - 16);
      }
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t two = hw[1 + 8 * h + k];
      w[2 * k] = (float)(int8_t)(two & 0xffu) * d;
      w[2 * k + 1] = (float)(int8_t)(two >> 8) * d;
    }
  }
}

// Cache element write: fp32, or bf16 rounded to nearest even.
__device__ __forceinline__ void cache_store(void* base, size_t off, int dtype, float v) {
  if (dtype == 0)
    static_cast<float*>(base)[off] = v;
  else
    static_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(v);
}

}  // namespace

__global__ void __launch_bounds__(QKV_THREADS) qkv_kernel(const QkvParams p) {
  extern __shared__ __align__(16) unsigned char qsm[];
  griddep_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cols = p.cols;
  const QkvSmem L = qkv_smem_layout(cols);
  uint8_t* raw = qsm;
  float* ys = reinterpret_cast<float*>(qsm + L.y_off);

  // This CTA's matrix and rows.
  int b = blockIdx.x, m = 0;
  while (m < 2 && b >= p.tiles[m]) {
    b -= p.tiles[m];
    ++m;
  }
  const int rows = p.rows[m], r0 = b * kQkvRows, nr = min(kQkvRows, rows - r0);
  const int type = p.wtype[m], bs = wtype_block_bytes(type);
  const size_t row_bytes = (size_t)(cols >> 5) * bs;
  const uint8_t* src = p.w[m] + (size_t)r0 * row_bytes;
  const size_t bytes = (size_t)nr * row_bytes;

  const int s_begin = blockIdx.y * kQkvSeqs, ns = min(kQkvSeqs, p.B - s_begin);

  // 1. Raw blocks into shared memory (before the wait: weights are
  //    constants).  16-byte loads when the span allows, four per thread in
  //    flight; else 2-byte loads (blocks are 2-byte aligned).
  if (((reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(raw);
    const int n4 = (int)(bytes >> 4);
    for (int i0 = 0; i0 < n4; i0 += 4 * QKV_THREADS) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * QKV_THREADS + tid;
        if (i < n4) r[u] = __ldg(s4 + i);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * QKV_THREADS + tid;
        if (i < n4) d4[i] = r[u];
      }
    }
  } else {
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(raw);
    const int n2 = (int)(bytes >> 1);
    for (int i = tid; i < n2; i += QKV_THREADS) d2[i] = __ldg(s2 + i);
  }
  __syncthreads();
  // 2. Lane l decodes block l of the warp's row (before the wait).
  const int nb = cols >> 5;
  const uint8_t* rowp = raw + (size_t)min(warp, nr - 1) * row_bytes;
  float w[32];
  const bool one_group = nb <= 32;
  if (one_group) {
    if (lane < nb) {
      decode_block(rowp + (size_t)lane * bs, type, w);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) w[k] = 0.f;
    }
  }

  griddep_wait();
  // Epilogue inputs of this thread's first item (sequence, row or row pair),
  // loaded now so that their latency overlaps the dot products.
  const bool pairs = p.mode == 1 && m < 2;
  const int per_seq = pairs ? (nr >> 1) : nr;
  const int n_items = ns * per_seq;
  const float* bias = p.bias[m];
  int pre_pos = 0;
  float pre_b0 = 0.f, pre_b1 = 0.f;
  if (tid < n_items) {
    const int s = tid / per_seq, r = (pairs ? 2 : 1) * (tid - s * per_seq);
    if (p.mode == 1) pre_pos = p.pos[s_begin + s];
    if (bias) {
      pre_b0 = bias[r0 + r];
      if (pairs) pre_b1 = bias[r0 + r + 1];
    }
  }
  // 3. Dot products: warp = row, lane = block, two sequences at a time.
  if (warp < nr) {
    const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    if (one_group) {
      const bool have = lane < nb;
      int s = 0;
      for (; s + 1 < ns; s += 2) {
        float v0[32], v1[32];
        float y0 = 0.f, y1 = 0.f;
        if (have) {
          load_x32(p.x + (size_t)(s_begin + s) * cols + lane * 32, vec, v0);
          load_x32(p.x + (size_t)(s_begin + s + 1) * cols + lane * 32, vec, v1);
          y0 = dot32(w, v0);
          y1 = dot32(w, v1);
        }
        y0 = warp_sum(y0);
        y1 = warp_sum(y1);
        if (lane == 0) {
          ys[s * kQkvRows + warp] = y0;
          ys[(s + 1) * kQkvRows + warp] = y1;
        }
      }
      if (s < ns) {
        float v0[32];
        float y0 = 0.f;
        if (have) {
          load_x32(p.x + (size_t)(s_begin + s) * cols + lane * 32, vec, v0);
          y0 = dot32(w, v0);
        }
        y0 = warp_sum(y0);
        if (lane == 0) ys[s * kQkvRows + warp] = y0;
      }
    } else {
      for (int s = 0; s < ns; ++s) {
        float y0 = 0.f;
        for (int g = lane; g < nb; g += 32) {
          float v0[32];
          load_x32(p.x + (size_t)(s_begin + s) * cols + g * 32, vec, v0);
          decode_block(rowp + (size_t)g * bs, type, w);
          y0 += dot32(w, v0);
        }
        y0 = warp_sum(y0);
        if (lane == 0) ys[s * kQkvRows + warp] = y0;
      }
    }
  }
  const int hd = p.head_dim;
  float2 pre_cs = make_float2(1.f, 0.f);
  if (pairs && tid < n_items && pre_pos >= 0 && pre_pos < p.table_len) {
    const int r = 2 * (tid - (tid / per_seq) * per_seq);
    pre_cs = *reinterpret_cast<const float2*>(p.cs + (size_t)pre_pos * hd + (r0 + r) % hd);
  }
  __syncthreads();
  // 4. Epilogue (a thread's first item uses the values loaded above).
  if (p.mode != 1) {
    // Mode 0: y = W x (+ bias).  Mode 2: y += W x, the residual add of
    // tmac_gguf.cpp:1499 (elem_op 0) rounded once after the product sum.
    for (int i = tid; i < ns * nr; i += QKV_THREADS) {
      const int s = i / nr, r = i - s * nr;
      float y = ys[s * kQkvRows + r];
      if (bias) y = __fadd_rn(y, i == tid ? pre_b0 : bias[r0 + r]);
      float* dst = p.y[m] + (size_t)(s_begin + s) * rows + r0 + r;
      *dst = p.mode == 2 ? __fadd_rn(*dst, y) : y;
    }
  } else if (m < 2) {
    // q or k: bias, then the rotation of pairs (2i, 2i+1) of a head
    // (tmac_gguf.cpp:1000-1003): x0*c - x1*s, x0*s + x1*c.
    const int np = nr >> 1;
    for (int i = tid; i < ns * np; i += QKV_THREADS) {
      const int s = i / np, r = 2 * (i - s * np), seq = s_begin + s;
      const bool first = i == tid;
      float x0 = ys[s * kQkvRows + r], x1 = ys[s * kQkvRows + r + 1];
      if (bias) {
        x0 = __fadd_rn(x0, first ? pre_b0 : bias[r0 + r]);
        x1 = __fadd_rn(x1, first ? pre_b1 : bias[r0 + r + 1]);
      }
      const int pos = first ? pre_pos : p.pos[seq];
      if (pos < 0 || pos >= p.table_len) {
        record_error(p.err, kDevErrBadPos);
        continue;
      }
      const float2 cs = first ? pre_cs
                              : *reinterpret_cast<const float2*>(p.cs + (size_t)pos * hd +
                                                                 (r0 + r) % hd);
      const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
      const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
      const size_t o = (size_t)seq * rows + r0 + r;
      if (m == 0) {
        *reinterpret_cast<float2*>(p.q_out + o) = make_float2(y0, y1);
      } else {
        if (p.k_out) *reinterpret_cast<float2*>(p.k_out + o) = make_float2(y0, y1);
        const int local = pos - p.shard_start;
        if (local >= 0 && local < p.max_ctx) {
          const size_t co = ((size_t)seq * p.max_ctx + local) * rows + r0 + r;
          cache_store(p.k_cache, co, p.dtype, y0);
          cache_store(p.k_cache, co + 1, p.dtype, y1);
        }
      }
    }
  } else {
    // v: bias, then the cache row.
    for (int i = tid; i < ns * nr; i += QKV_THREADS) {
      const int s = i / nr, r = i - s * nr, seq = s_begin + s;
      const bool first = i == tid;
      float y = ys[s * kQkvRows + r];
      if (bias) y = __fadd_rn(y, first ? pre_b0 : bias[r0 + r]);
      if (p.v_out) p.v_out[(size_t)seq * rows + r0 + r] = y;
      const int pos = first ? pre_pos : p.pos[seq];
      const int local = pos - p.shard_start;
      if (local >= 0 && local < p.max_ctx)
        cache_store(p.v_cache, ((size_t)seq * p.max_ctx + local) * rows + r0 + r, p.dtype, y);
    }
  }
}

namespace {

constexpr int QG_THREADS = 128;  // 4 warps x 4 rows
constexpr int QG_KC = 32;        // columns per x chunk (one block)
constexpr int QG_TS = kQkvSeqs;  // sequences per CTA (2 per lane)

// The raw blocks are dead once decoded, so the x^T buffers reuse their
// bytes: [raw blocks | x^T [2][QG_KC][QG_TS]] then W^T [cols][16] fp32.
struct QgSmem {
  int xt_off;  // 0: shares the raw blocks' bytes
  int wt_off;
  int total;
};

__host__ __device__ inline QgSmem qkv_gemm_layout(int cols) {
  QgSmem L;
  const int raw = ((kQkvGemmRows * (cols / 32) * 34) + 15) & ~15;
  const int xt = 2 * QG_KC * QG_TS * 4;
  L.xt_off = 0;
  L.wt_off = raw > xt ? raw : xt;
  L.total = L.wt_off + cols * kQkvGemmRows * 4;
  return L;
}

// Epilogue of one output pair (rows lr, lr+1 of the CTA; one sequence) in
// mode 1 for q / k: bias, rotation, q_out / k cache row.
__device__ __forceinline__ void qg_store_pair(const QkvParams& p, int m, int rows, int r, int seq,
                                              float x0, float x1, const float* bias) {
  if (bias) {
    x0 = __fadd_rn(x0, bias[r]);
    x1 = __fadd_rn(x1, bias[r + 1]);
  }
  const int pos = p.pos[seq];
  if (pos < 0 || pos >= p.table_len) {
    record_error(p.err, kDevErrBadPos);
    return;
  }
  const float2 cs = *reinterpret_cast<const float2*>(p.cs + (size_t)pos * p.head_dim +
                                                     r % p.head_dim);
  const float y0 = __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y));
  const float y1 = __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
  const size_t o = (size_t)seq * rows + r;
  if (m == 0) {
    *reinterpret_cast<float2*>(p.q_out + o) = make_float2(y0, y1);
  } else {
    if (p.k_out) *reinterpret_cast<float2*>(p.k_out + o) = make_float2(y0, y1);
    const int local = pos - p.shard_start;
    if (local >= 0 && local < p.max_ctx) {
      const size_t co = ((size_t)seq * p.max_ctx + local) * rows + r;
      cache_store(p.k_cache, co, p.dtype, y0);
      cache_store(p.k_cache, co + 1, p.dtype, y1);
    }
  }
}

// Mode 0 / 2 output (2: added to y), or mode 1 v row (bias, cache row,
// v_out).
__device__ __forceinline__ void qg_store_one(const QkvParams& p, int m, int rows, int r, int seq,
                                             float y, const float* bias) {
  if (bias) y = __fadd_rn(y, bias[r]);
  if (p.mode != 1) {
    float* dst = p.y[m] + (size_t)seq * rows + r;
    *dst = p.mode == 2 ? __fadd_rn(*dst, y) : y;
    return;
  }
  if (p.v_out) p.v_out[(size_t)seq * rows + r] = y;
  const int local = p.pos[seq] - p.shard_start;
  if (local >= 0 && local < p.max_ctx)
    cache_store(p.v_cache, ((size_t)seq * p.max_ctx + local) * rows + r, p.dtype, y);
}

}  // namespace

__global__ void __launch_bounds__(QG_THREADS) qkv_gemm_kernel(const QkvParams p) {
  extern __shared__ __align__(16) unsigned char qsm[];
  griddep_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cols = p.cols, nb = cols >> 5;
  const QgSmem L = qkv_gemm_layout(cols);
  uint8_t* raw = qsm;
  float* wt = reinterpret_cast<float*>(qsm + L.wt_off);
  float* xt = reinterpret_cast<float*>(qsm + L.xt_off);

  int b = blockIdx.x, m = 0;
  while (m < 2 && b >= p.tiles[m]) {
    b -= p.tiles[m];
    ++m;
  }
  const int rows = p.rows[m], r0 = b * kQkvGemmRows, nr = min(kQkvGemmRows, rows - r0);
  const int type = p.wtype[m], bs = wtype_block_bytes(type);
  const size_t row_bytes = (size_t)nb * bs;
  const uint8_t* src = p.w[m] + (size_t)r0 * row_bytes;
  const size_t bytes = (size_t)nr * row_bytes;
  const int s_begin = blockIdx.y * QG_TS, ns = min(QG_TS, p.B - s_begin);

  // 1. Raw blocks into shared memory (before the wait).
  if (((reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(raw);
    const int n4 = (int)(bytes >> 4);
    for (int i0 = 0; i0 < n4; i0 += 8 * QG_THREADS) {
      uint4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * QG_THREADS + tid;
        if (i < n4) r[u] = __ldg(s4 + i);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * QG_THREADS + tid;
        if (i < n4) d4[i] = r[u];
      }
    }
  } else {
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(raw);
    const int n2 = (int)(bytes >> 1);
    for (int i = tid; i < n2; i += QG_THREADS) d2[i] = __ldg(s2 + i);
  }
  __syncthreads();
  // 2. Decode into W^T [k][16] (rows past nr are zero).
  for (int it = tid; it < kQkvGemmRows * nb; it += QG_THREADS) {
    const int r = it & (kQkvGemmRows - 1), blk = it / kQkvGemmRows;
    float w[32];
    if (r < nr) {
      decode_block(raw + (size_t)r * row_bytes + (size_t)blk * bs, type, w);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) wt[(blk * 32 + j) * kQkvGemmRows + r] = w[j];
  }
  __syncthreads();

  griddep_wait();
  // 3. K loop: x^T chunks of QG_KC columns, double-buffered through registers.
  //    Loader thread t: sequence t % 64, columns (t / 64) * 16 .. +15.
  const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
  const int ls = tid & (QG_TS - 1), lh = tid / QG_TS;
  float4 xr[4];
  auto load_chunk = [&](int c) {
    if (ls < ns) {
      const float* x = p.x + (size_t)(s_begin + ls) * cols + c * QG_KC + lh * 16;
      if (vec) {
#pragma unroll
        for (int q = 0; q < 4; ++q) xr[q] = __ldg(reinterpret_cast<const float4*>(x) + q);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xr[q] = make_float4(__ldg(x + 4 * q), __ldg(x + 4 * q + 1), __ldg(x + 4 * q + 2),
                              __ldg(x + 4 * q + 3));
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) xr[q] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  auto store_chunk = [&](int buf) {
    float* d = xt + buf * QG_KC * QG_TS + (lh * 16) * QG_TS + ls;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      d[(4 * q + 0) * QG_TS] = xr[q].x;
      d[(4 * q + 1) * QG_TS] = xr[q].y;
      d[(4 * q + 2) * QG_TS] = xr[q].z;
      d[(4 * q + 3) * QG_TS] = xr[q].w;
    }
  };
  float acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.f;
  load_chunk(0);
  store_chunk(0);
  __syncthreads();
  for (int c = 0; c < nb; ++c) {
    if (c + 1 < nb) load_chunk(c + 1);
    const float* xb = xt + (c & 1) * QG_KC * QG_TS + lane * 2;
    const float* wb = wt + (size_t)c * QG_KC * kQkvGemmRows + warp * 4;
#pragma unroll 8
    for (int k = 0; k < QG_KC; ++k) {
      const float4 w4 = *reinterpret_cast<const float4*>(wb + k * kQkvGemmRows);
      const float2 x2 = *reinterpret_cast<const float2*>(xb + k * QG_TS);
      acc[0][0] = fmaf(w4.x, x2.x, acc[0][0]);
      acc[0][1] = fmaf(w4.x, x2.y, acc[0][1]);
      acc[1][0] = fmaf(w4.y, x2.x, acc[1][0]);
      acc[1][1] = fmaf(w4.y, x2.y, acc[1][1]);
      acc[2][0] = fmaf(w4.z, x2.x, acc[2][0]);
      acc[2][1] = fmaf(w4.z, x2.y, acc[2][1]);
      acc[3][0] = fmaf(w4.w, x2.x, acc[3][0]);
      acc[3][1] = fmaf(w4.w, x2.y, acc[3][1]);
    }
    if (c + 1 < nb) store_chunk((c + 1) & 1);
    __syncthreads();
  }

  // 4. Epilogue from registers: rows r0 + 4*warp + {0..3}, sequences
  //    s_begin + 2*lane + {0, 1}.
  const float* bias = p.bias[m];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int sl = 2 * lane + i;
    if (sl >= ns) continue;
    const int seq = s_begin + sl;
#pragma unroll
    for (int t = 0; t < 4; t += 2) {
      const int lr = warp * 4 + t;
      if (lr >= nr) continue;
      if (p.mode == 1 && m < 2) {
        qg_store_pair(p, m, rows, r0 + lr, seq, acc[t][i], acc[t + 1][i], bias);
      } else {
        qg_store_one(p, m, rows, r0 + lr, seq, acc[t][i], bias);
        if (lr + 1 < nr) qg_store_one(p, m, rows, r0 + lr + 1, seq, acc[t + 1][i], bias);
      }
    }
  }
}

// ------------------------------------------------------------ tensor cores

namespace {

constexpr int TC_M = 128;                  // weight rows per CTA (TMEM lanes)
constexpr int TC_N = kQkvSeqs;             // sequences per CTA (TMEM columns)
constexpr int TC_KC = 32;                  // columns per chunk: one weight block
constexpr int TC_STAGES = 3;
constexpr int TC_B_BYTES = TC_N * TC_KC * 4;     // 8 KB
constexpr int TC_STAGE_BYTES = 2 * TC_B_BYTES;   // hi and lo of the inputs (B)
constexpr int TC_THREADS = 288;  // warps 0-7 producers and epilogue, 8 TMEM + MMA
// TMEM: the accumulator in columns [0, 64); the weights' (A) hi / lo parts of
// stage s in columns 64 + 64 s + [0, 32) / [32, 64), one tf32 per column.
constexpr uint32_t TC_A_COL0 = 64;
constexpr uint32_t TC_TMEM_COLS = 256;
static_assert(TC_A_COL0 + TC_STAGES * 64 <= TC_TMEM_COLS, "A stages fit the allocation");

constexpr int TC_MAX_SPLIT = 8;  // CTAs per cluster along the columns
// After the last MMA the stage buffers hold the CTA's partial sums
// [TC_N][TC_M] fp32, then the positions and cos/sin rows of the sequences
// the CTA finishes.
// Rank k of a cluster of S finishes sequence columns [64 k / S, 64 (k + 1) / S)
// of its group, at most tc_per(S) of them.
__host__ __device__ constexpr int tc_per(int split) { return (TC_N + split - 1) / split; }
// Partial sums received from the cluster's ranks: [split][tc_per][128] fp32
// (a region of its own: peers store into it while this CTA may still be in
// its main loop); the largest over widths 1-8 (7 x 10 columns).
constexpr int TC_RECV_BYTES = 70 * TC_M * 4;  // 35 KB
static_assert(7 * tc_per(7) <= 70 && 6 * tc_per(6) <= 70 && 5 * tc_per(5) <= 70 &&
                  3 * tc_per(3) <= 70 && 8 * tc_per(8) <= 70,
              "receive buffer holds every width");
// Positions and cos/sin rows (head_dim <= 128) overlay the stages, dead once
// every MMA has completed.
static_assert(256 + TC_N * 128 * 4 <= TC_STAGES * TC_STAGE_BYTES, "positions fit the stages");

struct TcSmem {
  int raw_off;    // the CTA's raw weight rows (its chunks only)
  int recv_off;   // partial sums received from the cluster
  int flags_off;  // abort flags received from the cluster [TC_MAX_SPLIT]
  int bar_off;    // full[TC_STAGES], empty[TC_STAGES], done
  int misc_off;  // TMEM base address, abort flag
  int total;     // bytes to request (with 1 KB for the alignment of the base)
};

// Chunks of 32 columns that a CTA of a `split`-wide cluster takes at most;
// rank k takes chunks [k n / split, (k + 1) n / split).
__host__ __device__ inline int tc_chunks_per_cta(int cols, int split) {
  return (cols / TC_KC + split - 1) / split;
}

// Shared-memory slot of one staged row segment of `seg` bytes: the segment
// keeps its global address's 2-byte phase within 4 bytes (it starts at
// offset (address & 2)), so that whole 4-byte words line up on both sides.
__host__ __device__ inline int tc_row_slot(int seg) { return (seg + 2 + 3) & ~3; }

__host__ __device__ inline TcSmem qkv_tc_layout(int cols, int split) {
  TcSmem L;
  L.raw_off = TC_STAGES * TC_STAGE_BYTES;
  const int raw_end = L.raw_off + TC_M * tc_row_slot(tc_chunks_per_cta(cols, split) * 34);
  L.recv_off = (raw_end + 15) & ~15;
  L.flags_off = L.recv_off + TC_RECV_BYTES;
  L.bar_off = L.flags_off + TC_MAX_SPLIT * 4;
  L.misc_off = L.bar_off + (2 * TC_STAGES + 1) * 8;
  L.total = 1024 + L.misc_off + 16;
  return L;
}

// Instruction descriptor of kind::tf32: fp32 accumulator, tf32 A and B,
// both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::tf32 (A: lane = row, one
// tf32 per column along K).
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 columns of this warp's 32 TMEM lanes from 16 registers per thread (no
// wait).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// Nearest tf32 (10 stored mantissa bits), as a float with the low 13 bits 0.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t y;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(y) : "f"(x));
  return __uint_as_float(y);
}

// Byte offset of element (row r, k) in a K-major tile of 32 four-byte
// elements per row, 128-byte swizzle (8-row atoms of 1024 bytes).
__device__ __forceinline__ uint32_t sw128_off(int r, int k) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 2) ^ r) & 7) << 4) + ((k & 3) << 2));
}

// Stages nr row segments of `seg` bytes (global rows row_bytes apart, every
// address 2-byte aligned) into slots of tc_row_slot(seg) bytes: warp w takes
// rows w, w + nwarps, ...; the 4-byte words inside a segment move by
// cp.async (many in flight, no registers), a 2-byte piece at either end by a
// plain load and store.  Reads stay inside the segments.  The caller waits
// with cp.async.wait_all and a barrier.
__device__ __forceinline__ void tc_stage_rows(uint8_t* raw, const uint8_t* src, size_t row_bytes,
                                              int seg, int nr, int warp, int lane, int nwarps) {
  const int slot = tc_row_slot(seg);
  for (int r = warp; r < nr; r += nwarps) {
    const uint8_t* a = src + (size_t)r * row_bytes;
    const int head = (int)(reinterpret_cast<uintptr_t>(a) & 2);  // 0 or 2
    uint8_t* d = raw + (size_t)r * slot + head;                     // d = a (mod 4)
    const int words = (seg - head) >> 2;
    const int tail = seg - head - 4 * words;  // 0 or 2
    const uint32_t d0 = smem_u32(d + head);
    for (int k = lane; k < words; k += 32)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d0 + 4u * k),
                   "l"(a + head + 4 * k)
                   : "memory");
    if (lane == 0 && head)
      *reinterpret_cast<uint16_t*>(d) = __ldg(reinterpret_cast<const uint16_t*>(a));
    if (lane == 1 && tail)
      *reinterpret_cast<uint16_t*>(d + head + 4 * words) =
          __ldg(reinterpret_cast<const uint16_t*>(a + head + 4 * words));
  }
}

// Where tc_stage_rows put row r's segment.
__device__ __forceinline__ const uint8_t* tc_staged_row(const uint8_t* raw, const uint8_t* src,
                                                        size_t row_bytes, int seg, int r) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src + (size_t)r * row_bytes);
  return raw + (size_t)r * tc_row_slot(seg) + (a & 2);
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity, err, kDevErrWaitFull)) return true;
  *abort_flag = 1;
  return false;
}

}  // namespace

// The batched projection on the tensor cores, 3xTF32: a decoded weight (an
// fp16 scale times a small integer, at most 19 significant bits) is exactly
// w_hi + w_lo with both parts tf32; x is split into x_hi = tf32(x) and
// x_lo = x - x_hi; D = w_hi x_hi + w_hi x_lo + w_lo x_hi accumulates in fp32
// in TMEM (the dropped w_lo x_lo and x_lo's own tf32 rounding are below
// 2^-21 of |w x|).  A cluster of S = gridDim.z CTAs (1 to 8) computes
// 128 weight rows x 64 sequences; rank k takes the columns of chunks
// [k n / S, (k + 1) n / S) of the n 32-column chunks:
//   warps 0-7  producers: per chunk thread t decodes half of weight row
//              t % 128's block from the raw rows staged in shared memory
//              (before the grid-dependency wait) and stores its hi / lo
//              parts into the stage's A columns of TMEM (lane = row: no
//              shared-memory traffic for the weights), and splits 8 inputs
//              of sequence t / 4, loaded two chunks ahead, into the stage's
//              B tiles in shared memory (K-major, 128-byte swizzle);
//   warp 8     allocates 256 TMEM columns; one thread issues per chunk 12
//              tcgen05.mma (4 K-steps x 3 products, M128 N64 K8, A from
//              TMEM) and commits the stage back to the producers;
//   reduction  rank k finishes sequences [64 k / S, 64 (k + 1) / S): warps
//              0-7 read the CTA's 128 x 64 partial sums from TMEM and store
//              each sequence's into its finishing rank's receive buffer
//              (distributed shared memory stores: no round trip), every
//              rank its abort flag likewise; after one cluster barrier rank
//              k sums its sequences' S partials in rank order from its own
//              shared memory and applies mode 0 / 1 / 2 exactly as
//              qkv_kernel does (a RoPE partner row is the neighbouring
//              lane).
// Every mbarrier wait is bounded; a failed wait raises the CTA's abort
// flag, all roles leave their loops, the issued MMAs are drained, every
// thread still takes the cluster barrier, the cluster stores nothing if any
// rank aborted, and TMEM is freed.
__global__ void __launch_bounds__(TC_THREADS, 1) qkv_tc_kernel(const QkvParams p) {
  extern __shared__ uint8_t tsm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) &
                                           ~uintptr_t(1023));
  griddep_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cols = p.cols, nchunks = cols / TC_KC;
  const int split = (int)gridDim.z, rank = (int)blockIdx.z;
  const int c_begin = rank * nchunks / split, nck = (rank + 1) * nchunks / split - c_begin;
  const TcSmem L = qkv_tc_layout(cols, split);
  uint8_t* raw = sm + L.raw_off;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L.bar_off);  // one arrival per producer warp
  uint64_t* empty = full + TC_STAGES;                              // MMA commit
  uint64_t* done = empty + TC_STAGES;                              // all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L.misc_off);
  int* abort_ptr = reinterpret_cast<int*>(sm + L.misc_off + 4);
  volatile int* abort_flag = abort_ptr;

  int b = blockIdx.x, m = 0;
  while (m < 2 && b >= p.tiles[m]) {
    b -= p.tiles[m];
    ++m;
  }
  const int rows = p.rows[m], r0 = b * TC_M, nr = min(TC_M, rows - r0);
  const int type = p.wtype[m], bs = wtype_block_bytes(type);
  const size_t row_bytes = (size_t)nchunks * bs;
  const int seg = nck * bs;  // bytes of each row in this CTA's chunks
  const uint8_t* src = p.w[m] + (size_t)r0 * row_bytes + (size_t)c_begin * bs;
  const int s_begin = blockIdx.y * TC_N, ns = min(TC_N, p.B - s_begin);

  if (tid == 0) {
    for (int i = 0; i < TC_STAGES; ++i) {
      mbar_init(&full[i], 8);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // Raw weight rows of the CTA's chunks into shared memory (constants:
  // before the wait).
  tc_stage_rows(raw, src, row_bytes, seg, nr, warp, lane, TC_THREADS / 32);
  asm volatile("cp.async.wait_all;" ::: "memory");
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();

  if (warp < 8) {
    // ------------------------------------------------------------ producers
    // Thread t: elements 16h..16h+15 (h = t / 128) of weight row t % 128's
    // block, and 8 inputs (columns 8u..8u+7, u = t % 4) of sequence t / 4.
    const int r = tid & (TC_M - 1), h = tid >> 7;
    const uint8_t* rowp = tc_staged_row(raw, src, row_bytes, seg, min(r, nr - 1));
    const int sq = tid >> 2, u = tid & 3;
    const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    const float* xrow =
        p.x + (size_t)(s_begin + min(sq, ns - 1)) * cols + (size_t)c_begin * TC_KC + u * 8;
    const uint32_t a_lane = tmem + ((uint32_t)((warp & 3) * 32) << 16) + TC_A_COL0 + 16 * h;
    float4 cur[2], nxt[2], nxt2[2];
    auto load = [&](int c, float4 (&d)[2]) {
      if (sq < ns) {
        const float* xp = xrow + c * TC_KC;
        if (vec) {
          d[0] = __ldg(reinterpret_cast<const float4*>(xp));
          d[1] = __ldg(reinterpret_cast<const float4*>(xp) + 1);
        } else {
#pragma unroll
          for (int q = 0; q < 2; ++q)
            d[q] = make_float4(__ldg(xp + 4 * q), __ldg(xp + 4 * q + 1), __ldg(xp + 4 * q + 2),
                               __ldg(xp + 4 * q + 3));
        }
      } else {
        d[0] = d[1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    load(0, cur);
    if (nck > 1) load(1, nxt);
    for (int c = 0; c < nck; ++c) {
      if (c + 2 < nck) load(c + 2, nxt2);
      const int st = c % TC_STAGES;
      // Lane 0 waits for the stage; the exit is warp-uniform (the TMEM
      // stores below are warp-collective).
      if (c >= TC_STAGES) {
        bool ok = true;
        if (lane == 0)
          ok = tc_wait(&empty[st], (uint32_t)(((c / TC_STAGES) & 1) ^ 1), p.err, abort_flag);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      }
      float w[16];
      if (r < nr) {
        decode_half(rowp + (size_t)c * bs, type, h, w);
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) w[k] = 0.f;
      }
      uint32_t whi[16], wlo[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const float hi = tf32_round(w[k]);
        whi[k] = __float_as_uint(hi);
        wlo[k] = __float_as_uint(w[k] - hi);
      }
      const uint32_t ta = a_lane + (uint32_t)(st * 64);
      tmem_st16(ta, whi);
      tmem_st16(ta + 32, wlo);
      uint8_t* bhi = sm + st * TC_STAGE_BYTES;
      uint8_t* blo = bhi + TC_B_BYTES;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float4 hi, lo;
        hi.x = tf32_round(cur[q].x);
        hi.y = tf32_round(cur[q].y);
        hi.z = tf32_round(cur[q].z);
        hi.w = tf32_round(cur[q].w);
        lo.x = cur[q].x - hi.x;
        lo.y = cur[q].y - hi.y;
        lo.z = cur[q].z - hi.z;
        lo.w = cur[q].w - hi.w;
        const uint32_t off = sw128_off(sq, 8 * u + 4 * q);
        *reinterpret_cast<float4*>(bhi + off) = hi;
        *reinterpret_cast<float4*>(blo + off) = lo;
      }
      // Each thread orders its own B stores (async proxy) and TMEM stores;
      // after the warp barrier one arrival publishes the warp's share.
      fence_proxy_async_smem();
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[st]);
      cur[0] = nxt[0];
      cur[1] = nxt[1];
      nxt[0] = nxt2[0];
      nxt[1] = nxt2[1];
    }
  } else if (lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t IDESC = idesc_tf32(TC_M, TC_N);
    const uint32_t base = smem_u32(sm);
    bool issued = false;
    for (int c = 0; c < nck; ++c) {
      const int st = c % TC_STAGES;
      if (!tc_wait(&full[st], (uint32_t)((c / TC_STAGES) & 1), p.err, abort_flag)) break;
      tc_fence_after();
      const uint32_t sb = base + st * TC_STAGE_BYTES;
      const uint64_t bhi = smem_desc_sw128(sb, 16, 1024);
      const uint64_t blo = smem_desc_sw128(sb + TC_B_BYTES, 16, 1024);
      const uint32_t ahi = tmem + TC_A_COL0 + (uint32_t)(st * 64), alo = ahi + 32;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // K-step: 8 TMEM columns of A, 32 bytes of B (+2)
        umma_tf32_ts(tmem, ahi + 8 * kk, bhi + 2 * kk, IDESC, (c > 0 || kk > 0) ? 1u : 0u);
        umma_tf32_ts(tmem, ahi + 8 * kk, blo + 2 * kk, IDESC, 1u);
        umma_tf32_ts(tmem, alo + 8 * kk, bhi + 2 * kk, IDESC, 1u);
      }
      umma_commit(&empty[st]);
      issued = true;
    }
    // done completes when every issued MMA has; wait for it (bounded) so
    // that TMEM is not freed under them.
    umma_commit(done);
    if (issued) mbar_wait(done, 0u, p.err, kDevErrWaitFull);
    if (!issued || *abort_flag) *abort_flag = 1;
  }

  // Sequences this rank finishes; positions and cos/sin rows staged in the
  // stage buffers (free once every MMA has completed).
  const int per = tc_per(split), jb = rank * TC_N / split;
  const int je = min((rank + 1) * TC_N / split, ns);
  float* recv = reinterpret_cast<float*>(sm + L.recv_off);  // [split][per][TC_M]
  int* flags = reinterpret_cast<int*>(sm + L.flags_off);
  int* pos_s = reinterpret_cast<int*>(sm);
  float* cs_s = reinterpret_cast<float*>(sm + 256);  // [per][head_dim]
  const bool pairs = p.mode == 1 && m < 2;
  const int lr = tid & (TC_M - 1), r = r0 + lr;  // epilogue row (warps 0-7)
  const bool row_ok = lr < nr;
  const float* bias = p.bias[m];
  float b_own = 0.f;
  if (warp < 8) {
    // ------------------------------------------------------------ partials
    const bool ok = tc_wait(done, 0u, p.err, abort_flag);
    if (bias && row_ok) b_own = __ldg(bias + r);  // in flight during the stores
    if (__all_sync(0xffffffffu, ok)) {
      // Warp w reads TMEM lanes 32 (w % 4).. and columns 32 (w / 4)..; the
      // sums of column j go to the rank k that finishes it, slot
      // [rank][j - 64 k / S].
      tc_fence_after();
      const int cb = (warp >> 2) * 32;
      const uint32_t taddr = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)cb;
      // Owner of the current column and its column range [b_lo, b_hi);
      // owners only grow with the column, by at most one per 8 columns.
      int owner = 0, b_lo = 0, b_hi = TC_N / split;
      while (cb >= b_hi) {
        ++owner;
        b_lo = b_hi;
        b_hi = (owner + 1) * TC_N / split;
      }
      auto slot_base = [&]() {
        return (owner == rank ? recv : cluster.map_shared_rank(recv, owner)) +
               (rank * per - b_lo) * TC_M + lr;
      };
      float* base = slot_base();  // column j of the owner: base[j * TC_M]
#pragma unroll 1
      for (int j0 = 0; j0 < 32; j0 += 8) {
        uint32_t v[8];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
            "tcgen05.wait::ld.sync.aligned;"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
              "=r"(v[7])
            : "r"(taddr + (uint32_t)j0));
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int j = cb + j0 + t;
          if (j >= b_hi) {  // warp-uniform
            ++owner;
            b_lo = b_hi;
            b_hi = (owner + 1) * TC_N / split;
            base = slot_base();
          }
          base[j * TC_M] = __uint_as_float(v[t]);
        }
      }
    }
    if (p.mode == 1) {
      if (tid < je - jb) pos_s[tid] = p.pos[s_begin + jb + tid];
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (pairs) {
        const int hd = p.head_dim;
        for (int i = tid; i < (je - jb) * hd; i += 256) {
          const int j = i / hd, d = i - j * hd;
          const int pos = pos_s[j];
          cs_s[i] = (pos >= 0 && pos < p.table_len) ? p.cs[(size_t)pos * hd + d] : 0.f;
        }
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();  // every role has finished: this CTA's abort flag is final
  if (tid < split)
    (tid == rank ? flags : cluster.map_shared_rank(flags, tid))[rank] = *abort_flag;
  // The cluster's partial sums and flags are in this CTA's shared memory
  // after this barrier; no CTA touches another's shared memory after it.
  cluster.sync();
  tc_fence_after();

  if (warp < 8) {
    // ------------------------------------------------------------ epilogue
    bool bad = false;
#pragma unroll
    for (int q = 0; q < TC_MAX_SPLIT; ++q)
      if (q < split) bad |= flags[q] != 0;
    if (!bad) {
      const float b_par = __shfl_xor_sync(0xffffffffu, b_own, 1);
      // Eight sequences per trip: every residual load (mode 2) of the trip
      // is issued before the first is used.
      constexpr int EU = 8;
#pragma unroll 1
      for (int j0 = jb + (tid >> 7); j0 < je; j0 += 2 * EU) {  // warp-uniform
        float yv[EU], hv[EU];
#pragma unroll
        for (int u = 0; u < EU; ++u) {
          const int j = j0 + 2 * u;
          yv[u] = 0.f;
          hv[u] = 0.f;
          if (j < je) {
            const float* rp = recv + (j - jb) * TC_M + lr;
            float y = rp[0];
#pragma unroll
            for (int q = 1; q < TC_MAX_SPLIT; ++q)
              if (q < split) y += rp[q * per * TC_M];  // rank order
            yv[u] = y;
            if (p.mode == 2 && row_ok) hv[u] = p.y[m][(size_t)(s_begin + j) * rows + r];
          }
        }
#pragma unroll
        for (int u = 0; u < EU; ++u) {
          const int j = j0 + 2 * u;
          if (j >= je) break;  // warp-uniform
          const int seq = s_begin + j;
          float y = yv[u];
          if (pairs) {
            const float other = __shfl_xor_sync(0xffffffffu, y, 1);
            if (!row_ok) continue;
            const bool even = (lr & 1) == 0;
            float x0 = even ? y : other, x1 = even ? other : y;
            if (bias) {
              x0 = __fadd_rn(x0, even ? b_own : b_par);
              x1 = __fadd_rn(x1, even ? b_par : b_own);
            }
            const int pos = pos_s[j - jb];
            if (pos < 0 || pos >= p.table_len) {
              record_error(p.err, kDevErrBadPos);
              continue;
            }
            const int re = r & ~1;
            const float2 cs = *reinterpret_cast<const float2*>(cs_s + (j - jb) * p.head_dim +
                                                               re % p.head_dim);
            const float out = even ? __fsub_rn(__fmul_rn(x0, cs.x), __fmul_rn(x1, cs.y))
                                   : __fadd_rn(__fmul_rn(x0, cs.y), __fmul_rn(x1, cs.x));
            const size_t o = (size_t)seq * rows + r;
            if (m == 0) {
              p.q_out[o] = out;
            } else {
              if (p.k_out) p.k_out[o] = out;
              const int local = pos - p.shard_start;
              if (local >= 0 && local < p.max_ctx)
                cache_store(p.k_cache, ((size_t)seq * p.max_ctx + local) * rows + r, p.dtype,
                            out);
            }
          } else if (row_ok) {
            if (bias) y = __fadd_rn(y, b_own);
            if (p.mode != 1) {
              p.y[m][(size_t)seq * rows + r] = p.mode == 2 ? __fadd_rn(hv[u], y) : y;
            } else {
              if (p.v_out) p.v_out[(size_t)seq * rows + r] = y;
              const int local = pos_s[j - jb] - p.shard_start;
              if (local >= 0 && local < p.max_ctx)
                cache_store(p.v_cache, ((size_t)seq * p.max_ctx + local) * rows + r, p.dtype,
                            y);
            }
          }
        }
      }
    }
  }
  if (warp == 8) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TC_TMEM_COLS)
                 : "memory");
  }
}

size_t qkv_smem(int cols) { return (size_t)qkv_smem_layout(cols).total; }

int qkv_gemm_max_cols() {
  int c = 32;
  while (qkv_gemm_layout(c + 32).total <= 227 * 1024) c += 32;
  return c;
}

bool qkv_use_gemm(int B, int cols) { return B >= kQkvGemmMinB && cols <= qkv_gemm_max_cols(); }

int qkv_tc_max_cols() {
  int c = 32;
  while (qkv_tc_layout(c + 32, 1).total <= 227 * 1024) c += 32;
  return c;
}

bool qkv_use_tc(int B, int cols) { return B >= kQkvGemmMinB && cols <= qkv_tc_max_cols(); }

int qkv_rows_per_cta(int B, int cols) {
  return qkv_use_tc(B, cols) ? TC_M : (qkv_use_gemm(B, cols) ? kQkvGemmRows : kQkvRows);
}

int qkv_max_cols() {
  // Largest multiple of 32 whose layout fits the 227 KB opt-in limit.
  int c = 32;
  while (qkv_smem_layout(c + 32).total <= 227 * 1024) c += 32;
  return c;
}

// Clusters of `split` tensor-core CTAs that the device keeps resident at
// once (cached per device, column count and split).
static int tc_resident_clusters(int dev, int cols, int split) {
  struct Entry {
    int dev, cols, split, n;
  };
  static Entry cache[64];
  static int used = 0;
  for (int i = 0; i < used; ++i)
    if (cache[i].dev == dev && cache[i].cols == cols && cache[i].split == split) return cache[i].n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(split, 1, split);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = (size_t)qkv_tc_layout(cols, split).total;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)split;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, qkv_tc_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (used < 64) cache[used++] = {dev, cols, split, n};
  return n;
}

static int g_tc_split_override = 0;

int set_qkv_tc_split(int split) {
  if (split < 0 || split > TC_MAX_SPLIT) return -1;
  g_tc_split_override = split;
  return 0;
}

int qkv_tc_split(int tiles, int cols, int dev) {
  const int nchunks = cols / TC_KC;
  if (g_tc_split_override > 0) {
    return g_tc_split_override < nchunks ? g_tc_split_override : nchunks;
  }
  // Cost in chunk times: waves x (chunks per CTA + ~3 chunks of fixed work:
  // TMEM allocation, staging, reduction and epilogue); ties keep the
  // narrower cluster.
  int best = 0;
  long best_cost = 0;
  for (int split = 1; split <= TC_MAX_SPLIT && split <= nchunks; ++split) {
    const int resident = tc_resident_clusters(dev, cols, split);
    if (resident <= 0) continue;
    const long waves = (tiles + resident - 1) / resident;
    const long cost = waves * (tc_chunks_per_cta(cols, split) + 3);
    if (best == 0 || cost < best_cost) {
      best = split;
      best_cost = cost;
    }
  }
  return best;
}

cudaError_t launch_qkv(const QkvParams& p, cudaStream_t st) {
  const int grid = p.tiles[0] + p.tiles[1] + p.tiles[2];
  if (grid <= 0 || p.B <= 0) return cudaSuccess;
  const int groups = (p.B + kQkvSeqs - 1) / kQkvSeqs;
  if (qkv_use_tc(p.B, p.cols)) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    // Opt in once per device to the largest request the kernel makes (the
    // whole tensor-core column range at split 1); the occupancy queries of
    // the split choice need it too.
    static bool opted_in[64] = {};
    if (!opted_in[dev]) {
      cudaError_t e =
          cudaFuncSetAttribute(qkv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               qkv_tc_layout(qkv_tc_max_cols(), 1).total);
      if (e != cudaSuccess) return e;
      opted_in[dev] = true;
    }
    const int split = qkv_tc_split(grid * groups, p.cols, dev);
    if (split <= 0) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, groups, split);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = (size_t)qkv_tc_layout(p.cols, split).total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = (unsigned)split;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, qkv_tc_kernel, p);
  }
  const bool gemm = qkv_use_gemm(p.B, p.cols);
  const size_t smem = gemm ? (size_t)qkv_gemm_layout(p.cols).total : qkv_smem(p.cols);
  void (*fn)(const QkvParams) = gemm ? qkv_gemm_kernel : qkv_kernel;
  static size_t configured[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > configured[gemm][dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured[gemm][dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, groups);
  cfg.blockDim = dim3(gemm ? QG_THREADS : QKV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

}  // namespace tg
