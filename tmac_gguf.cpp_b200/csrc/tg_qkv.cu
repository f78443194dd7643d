// tg_qkv.cu -- the Q/K/V projection of a decode step (sm_100a, CUDA cores).
//
//   qkv_kernel   y_m = W_m x for the layer's three projection matrices and B
//                input vectors, weights in the model file's 32-element
//                blocks (GGML Q5_0 / Q8_0, tmac_gguf.cpp:240-248, :311-328;
//                kernel_fused_qkv.metal:8-70).  Mode 0 writes y_m as
//                fused_qkv_op / matmul_q5_0 / matmul_q8_0 do
//                (metal_backend.hpp:320-338, :456-489).  Mode 1 fuses the
//                rest of the layer step up to attention
//                (tmac_gguf.cpp:1067-1091): the bias adds, RoPE of q and k
//                at each sequence's position (cos/sin from the host-libm
//                table, one rounding per product and sum), the k / v rows
//                written into the cache and the rotated q written out for
//                the attention kernel.
//
// Decomposition: CTA c takes kQkvRows = 8 consecutive rows of one matrix and
// every sequence.  It copies the rows' raw blocks into shared memory with
// 16-byte loads and decodes them to fp32 there (exact: an fp16 scale times a
// small integer), one warp per row then forms the dot products of all B
// inputs (lanes over columns, float4 loads, a shuffle reduction), and the
// epilogue runs over (sequence, row pair).  Weight rows are read once per
// launch; x rows are shared by the 8 warps through L1.
//
// PDL: the weight copy and decode come before griddepcontrol.wait, so they
// overlap the previous kernel on the stream (weights are constants of the
// model; the C ABI requires that the kernel launched just before a
// projection does not write its weights).  x, the outputs and the caches are
// touched only after the wait.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "tg_device.cuh"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace tg {

namespace {

constexpr int QKV_THREADS = kQkvRows * 32;

struct QkvSmem {
  int raw_bytes;   // staged blocks of kQkvRows rows (16-byte multiple)
  int w_off;       // fp32 weights [kQkvRows][cols]
  int y_off;       // dot products [kQkvChunk][kQkvRows]
  int total;
};

__host__ __device__ inline QkvSmem qkv_smem_layout(int cols) {
  QkvSmem L;
  const int max_row = (cols / 32) * 34;  // the larger block type
  L.raw_bytes = ((kQkvRows * max_row) + 15) & ~15;
  L.w_off = L.raw_bytes;
  L.y_off = L.w_off + kQkvRows * cols * 4;
  L.total = L.y_off + kQkvChunk * kQkvRows * 4;
  return L;
}

// f16_to_f32 of tmac_gguf.cpp:220-232: the exact widening, except that a
// zero of either sign becomes +0 (:225).
__device__ __forceinline__ float f16_scale(uint16_t h) {
  if ((h & 0x7fffu) == 0) return 0.0f;
  return __half2float(__ushort_as_half(h));
}

// Element j (0..31) of one block, decoded exactly as dequant_q5_0 /
// dequant_q8_0 (tmac_gguf.cpp:311-328, :240-248).  blk is 2-byte aligned.
__device__ __forceinline__ float dequant_elem(const uint8_t* blk, int type, int j) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(blk);
  const float d = f16_scale(h[0]);
  if (type == kWTypeQ5_0) {
    const uint32_t qh = (uint32_t)h[1] | ((uint32_t)h[2] << 16);
    const uint32_t byte = blk[6 + (j & 15)];
    const uint32_t lo = j < 16 ? (byte & 0xfu) : (byte >> 4);
    const int q = (int)((((qh >> j) & 1u) << 4) | lo) - 16;
    return d * (float)q;
  }
  return (float)(int8_t)blk[2 + j] * d;
}

// Cache element write: fp32, or bf16 rounded to nearest even.
__device__ __forceinline__ void cache_store(void* base, size_t off, int dtype, float v) {
  if (dtype == 0)
    static_cast<float*>(base)[off] = v;
  else
    static_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16_rn(v);
}

// Dot products of one fp32 weight row with two input rows (vector path:
// cols a multiple of 128, 16-byte aligned rows).
__device__ __forceinline__ void dot2_vec(const float* w, const float* x0, const float* x1,
                                         int cols, int lane, float& r0, float& r1) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll 4
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 w4 = *reinterpret_cast<const float4*>(w + c);
    const float4 u = __ldg(reinterpret_cast<const float4*>(x0 + c));
    const float4 v = __ldg(reinterpret_cast<const float4*>(x1 + c));
    a0 = fmaf(w4.x, u.x, a0);
    a1 = fmaf(w4.y, u.y, a1);
    a2 = fmaf(w4.z, u.z, a2);
    a3 = fmaf(w4.w, u.w, a3);
    b0 = fmaf(w4.x, v.x, b0);
    b1 = fmaf(w4.y, v.y, b1);
    b2 = fmaf(w4.z, v.z, b2);
    b3 = fmaf(w4.w, v.w, b3);
  }
  r0 = (a0 + a1) + (a2 + a3);
  r1 = (b0 + b1) + (b2 + b3);
}

__device__ __forceinline__ float dot1_vec(const float* w, const float* x0, int cols, int lane) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll 4
  for (int c = lane * 4; c < cols; c += 128) {
    const float4 w4 = *reinterpret_cast<const float4*>(w + c);
    const float4 u = __ldg(reinterpret_cast<const float4*>(x0 + c));
    a0 = fmaf(w4.x, u.x, a0);
    a1 = fmaf(w4.y, u.y, a1);
    a2 = fmaf(w4.z, u.z, a2);
    a3 = fmaf(w4.w, u.w, a3);
  }
  return (a0 + a1) + (a2 + a3);
}

__device__ __forceinline__ float dot1_scalar(const float* w, const float* x0, int cols, int lane) {
  float a0 = 0.f, a1 = 0.f;
  int c = lane;
  for (; c + 32 < cols; c += 64) {
    a0 = fmaf(w[c], __ldg(x0 + c), a0);
    a1 = fmaf(w[c + 32], __ldg(x0 + c + 32), a1);
  }
  if (c < cols) a0 = fmaf(w[c], __ldg(x0 + c), a0);
  return a0 + a1;
}

}  // namespace

__global__ void __launch_bounds__(QKV_THREADS) qkv_kernel(const QkvParams p) {
  extern __shared__ __align__(16) unsigned char qsm[];
  griddep_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int cols = p.cols;
  const QkvSmem L = qkv_smem_layout(cols);
  uint8_t* raw = qsm;
  float* wf = reinterpret_cast<float*>(qsm + L.w_off);
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

  // 1. Raw blocks into shared memory (before the wait: weights are
  //    constants).  16-byte loads when the span allows, else 2-byte loads
  //    (blocks are 2-byte aligned).
  if (((reinterpret_cast<uintptr_t>(src) | bytes) & 15) == 0) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    uint4* d4 = reinterpret_cast<uint4*>(raw);
    const int n4 = (int)(bytes >> 4);
    for (int i = tid; i < n4; i += QKV_THREADS) d4[i] = __ldg(s4 + i);
  } else {
    const uint16_t* s2 = reinterpret_cast<const uint16_t*>(src);
    uint16_t* d2 = reinterpret_cast<uint16_t*>(raw);
    const int n2 = (int)(bytes >> 1);
    for (int i = tid; i < n2; i += QKV_THREADS) d2[i] = __ldg(s2 + i);
  }
  __syncthreads();
  // 2. Decode to fp32 rows.
  const int n_el = nr * cols;
  for (int e = tid; e < n_el; e += QKV_THREADS) {
    const int r = e / cols, c = e - r * cols;
    wf[r * cols + c] = dequant_elem(raw + (size_t)r * row_bytes + (size_t)(c >> 5) * bs, type,
                                    c & 31);
  }
  __syncthreads();

  griddep_wait();
  const bool vec = (cols & 127) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
  const float* bias = p.bias[m];
  const int hd = p.head_dim;
  for (int s0 = 0; s0 < p.B; s0 += kQkvChunk) {
    const int ns = min(kQkvChunk, p.B - s0);
    // 3. Dot products: warp = row, two sequences at a time.
    if (warp < nr) {
      const float* wr = wf + warp * cols;
      int s = 0;
      if (vec) {
        for (; s + 1 < ns; s += 2) {
          float y0, y1;
          dot2_vec(wr, p.x + (size_t)(s0 + s) * cols, p.x + (size_t)(s0 + s + 1) * cols, cols,
                   lane, y0, y1);
          y0 = warp_sum(y0);
          y1 = warp_sum(y1);
          if (lane == 0) {
            ys[s * kQkvRows + warp] = y0;
            ys[(s + 1) * kQkvRows + warp] = y1;
          }
        }
        if (s < ns) {
          const float y0 = warp_sum(dot1_vec(wr, p.x + (size_t)(s0 + s) * cols, cols, lane));
          if (lane == 0) ys[s * kQkvRows + warp] = y0;
        }
      } else {
        for (; s < ns; ++s) {
          const float y0 = warp_sum(dot1_scalar(wr, p.x + (size_t)(s0 + s) * cols, cols, lane));
          if (lane == 0) ys[s * kQkvRows + warp] = y0;
        }
      }
    }
    __syncthreads();
    // 4. Epilogue.
    if (p.mode == 0) {
      for (int i = tid; i < ns * nr; i += QKV_THREADS) {
        const int s = i / nr, r = i - s * nr;
        float y = ys[s * kQkvRows + r];
        if (bias) y = __fadd_rn(y, bias[r0 + r]);
        p.y[m][(size_t)(s0 + s) * rows + r0 + r] = y;
      }
    } else if (m < 2) {
      // q or k: bias, then the rotation of pairs (2i, 2i+1) of a head
      // (tmac_gguf.cpp:1000-1003): x0*c - x1*s, x0*s + x1*c.
      const int np = nr >> 1;
      for (int i = tid; i < ns * np; i += QKV_THREADS) {
        const int s = i / np, r = 2 * (i - s * np), seq = s0 + s;
        float x0 = ys[s * kQkvRows + r], x1 = ys[s * kQkvRows + r + 1];
        if (bias) {
          x0 = __fadd_rn(x0, bias[r0 + r]);
          x1 = __fadd_rn(x1, bias[r0 + r + 1]);
        }
        const int pos = p.pos[seq];
        if (pos < 0 || pos >= p.table_len) {
          record_error(p.err, kDevErrBadPos);
          continue;
        }
        const int d = (r0 + r) % hd;
        const float2 cs = *reinterpret_cast<const float2*>(p.cs + (size_t)pos * hd + d);
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
        const int s = i / nr, r = i - s * nr, seq = s0 + s;
        float y = ys[s * kQkvRows + r];
        if (bias) y = __fadd_rn(y, bias[r0 + r]);
        if (p.v_out) p.v_out[(size_t)seq * rows + r0 + r] = y;
        const int pos = p.pos[seq];
        const int local = pos - p.shard_start;
        if (local >= 0 && local < p.max_ctx)
          cache_store(p.v_cache, ((size_t)seq * p.max_ctx + local) * rows + r0 + r, p.dtype, y);
      }
    }
    __syncthreads();
  }
}

size_t qkv_smem(int cols) { return (size_t)qkv_smem_layout(cols).total; }

int qkv_max_cols() {
  // Largest multiple of 32 whose layout fits the 227 KB opt-in limit.
  int c = 32;
  while (qkv_smem_layout(c + 32).total <= 227 * 1024) c += 32;
  return c;
}

cudaError_t launch_qkv(const QkvParams& p, cudaStream_t st) {
  const int grid = p.tiles[0] + p.tiles[1] + p.tiles[2];
  if (grid <= 0 || p.B <= 0) return cudaSuccess;
  const size_t smem = qkv_smem(p.cols);
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(QKV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qkv_kernel, p);
}

}  // namespace tg
