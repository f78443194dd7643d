// tg_prefill.cu -- causal prefill attention on the 5th-generation tensor
// cores (tcgen05 + TMEM), sm_100a.
//
// The reference has no batched prefill: process_prompt (tmac_gguf.cpp:1621-
// 1658) runs the decode step token by token, so the prompt's attention is
// the causal attention of every position t over rows 0..t (the GQA block of
// tmac_gguf.cpp:1093-1128 applied S times).  Here the S positions of a
// sequence are computed at once:
//
//   prefill_rope_kernel   RoPE of q and k at positions 0..S-1 in binary32
//                         exactly as apply_rope (tmac_gguf.cpp:990-1016),
//                         rounded to bf16 (RNE); k and v rows written to the
//                         bf16 KV cache, q to a bf16 staging buffer.
//   prefill_attn_kernel   flash attention over the cache, one CTA per SM,
//                         persistent over (sequence, query head, 128-row
//                         query tile) items, most expensive first.
//
// prefill_attn_kernel works on pairs of adjacent query tiles so that the
// tensor core computes one tile's products while the other tile's softmax
// runs (roles below, at the kernel).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tg_device.cuh"
#include "tg_tc.cuh"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace tg {

// ------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int x,
                                            int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 in, fp32 acc).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16: A is read from tensor
// memory (row m in lane m, two 16-bit elements per 32-bit column along K).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major ? (1u << 16) : 0u) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------ RoPE + rows

__global__ void __launch_bounds__(128) prefill_rope_kernel(const PrefillRopeParams p) {
  const int row = blockIdx.x;  // (sequence, position)
  const int s = row / p.S, t = row - s * p.S;
  const int hd = p.head_dim, half = hd >> 1;
  const float* cs = p.cs + (size_t)t * hd;
  const float* q = p.q + (size_t)row * p.n_head * hd;
  __nv_bfloat16* qo = reinterpret_cast<__nv_bfloat16*>(p.q_bf16) + (size_t)row * p.n_head * hd;
  for (int i = threadIdx.x; i < p.n_head * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half, idx = h * hd + 2 * j;
    const float x0 = q[idx], x1 = q[idx + 1], c = cs[2 * j], sn = cs[2 * j + 1];
    qo[idx] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    qo[idx + 1] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
  }
  const int kdim = p.n_kv * hd;
  const float* k = p.k + (size_t)row * kdim;
  const float* v = p.v + (size_t)row * kdim;
  __nv_bfloat16* kc =
      reinterpret_cast<__nv_bfloat16*>(p.k_cache) + ((size_t)s * p.max_ctx + t) * kdim;
  __nv_bfloat16* vc =
      reinterpret_cast<__nv_bfloat16*>(p.v_cache) + ((size_t)s * p.max_ctx + t) * kdim;
  for (int i = threadIdx.x; i < p.n_kv * half; i += blockDim.x) {
    const int h = i / half, j = i - h * half, idx = h * hd + 2 * j;
    const float x0 = k[idx], x1 = k[idx + 1], c = cs[2 * j], sn = cs[2 * j + 1];
    kc[idx] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn)));
    kc[idx + 1] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c)));
  }
  // v: bf16 into the cache, and fp16 of the same bf16 value (exact) as the
  // operand of the attention's P.V products.
  __half* vh = reinterpret_cast<__half*>(p.v_f16) + (size_t)row * kdim;
  for (int i = threadIdx.x; i < kdim; i += blockDim.x) {
    const __nv_bfloat16 b = __float2bfloat16_rn(v[i]);
    vc[i] = b;
    vh[i] = __float2half_rn(__bfloat162float(b));
  }
}

// The same work, one warp per (sequence, position) row and 8 rows per CTA,
// for head_dim 64 and inputs 16-byte aligned: each lane issues all its
// 16-byte loads of the row (q in batches of 8, k, v, and the one cos/sin
// float4 its columns share) before it uses the first, so the kernel keeps
// enough bytes in flight to stream at the copy rate.  Arithmetic per element
// as prefill_rope_kernel's.
__device__ __forceinline__ uint2 rope4_bf16(float4 x, float4 c) {
  const __nv_bfloat162 a =
      __floats2bfloat162_rn(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y)),
                            __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x)));
  const __nv_bfloat162 b =
      __floats2bfloat162_rn(__fsub_rn(__fmul_rn(x.z, c.z), __fmul_rn(x.w, c.w)),
                            __fadd_rn(__fmul_rn(x.z, c.w), __fmul_rn(x.w, c.z)));
  return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}

__global__ void __launch_bounds__(256) prefill_rope_rows_kernel(const PrefillRopeParams p) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);  // (sequence, position)
  if (row >= p.B * p.S) return;
  const int s = row / p.S, t = row - s * p.S;
  // float4 i of a row holds pairs 2m, 2m + 1 of its head, m = i % 16, whose
  // (cos, sin) are float4 m of the table row; a lane's i are all = lane (16).
  const float4 c4 = __ldg(reinterpret_cast<const float4*>(p.cs + (size_t)t * 64) + (lane & 15));
  const int nq = p.n_head * 16, nk = p.n_kv * 16;  // float4 per row
  const float4* __restrict__ q = reinterpret_cast<const float4*>(p.q) + (size_t)row * nq;
  uint2* __restrict__ qo = reinterpret_cast<uint2*>(p.q_bf16) + (size_t)row * nq;
  for (int i0 = 0; i0 < nq; i0 += 8 * 32) {
    float4 x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < nq) x[u] = __ldg(q + i);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < nq) qo[i] = rope4_bf16(x[u], c4);
    }
  }
  const float4* __restrict__ k = reinterpret_cast<const float4*>(p.k) + (size_t)row * nk;
  const float4* __restrict__ v = reinterpret_cast<const float4*>(p.v) + (size_t)row * nk;
  const size_t crow = ((size_t)s * p.max_ctx + t) * nk;
  uint2* __restrict__ kc = reinterpret_cast<uint2*>(p.k_cache) + crow;
  uint2* __restrict__ vc = reinterpret_cast<uint2*>(p.v_cache) + crow;
  uint2* __restrict__ vh = reinterpret_cast<uint2*>(p.v_f16) + (size_t)row * nk;
  for (int i0 = 0; i0 < nk; i0 += 4 * 32) {
    float4 xk[4], xv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < nk) {
        xk[u] = __ldg(k + i);
        xv[u] = __ldg(v + i);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * 32 + lane;
      if (i < nk) {
        kc[i] = rope4_bf16(xk[u], c4);
        // v: bf16 into the cache, and fp16 of the same bf16 value (exact) as
        // the operand of the attention's P.V products.
        const __nv_bfloat162 b0 = __floats2bfloat162_rn(xv[u].x, xv[u].y);
        const __nv_bfloat162 b1 = __floats2bfloat162_rn(xv[u].z, xv[u].w);
        vc[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&b0),
                           *reinterpret_cast<const uint32_t*>(&b1));
        const __half2 h0 = __floats2half2_rn(__low2float(b0), __high2float(b0));
        const __half2 h1 = __floats2half2_rn(__low2float(b1), __high2float(b1));
        vh[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&h0),
                           *reinterpret_cast<const uint32_t*>(&h1));
      }
    }
  }
}

// ------------------------------------------------------------ attention

constexpr int PF_M = 128;          // query rows per tile (TMEM lanes)
constexpr int PF_N = 128;          // cache rows per K/V tile
constexpr int PF_STAGES = 4;       // K/V ring depth
constexpr int PF_THREADS = 384;    // producer warpgroup (TMA, MMA, 2 idle warps), 2 softmax warpgroups
// Register split (setmaxnreg): the launch gives 384 x 168 = 64512; the
// producer warpgroup drops to 80 and the softmax warpgroups rise to 208:
// 128 x 80 + 256 x 208 = 63488.  Per sub-partition (three warps, one of each
// warpgroup) 80 + 208 + 208 registers per thread, 15872 of its 16384.  With
// these no role spills.
constexpr int PF_REG_PRODUCER = 80;
constexpr int PF_REG_SOFTMAX = 208;
constexpr int PF_TILE_BYTES = 128 * 128;   // 128 rows x 64 16-bit values (Q, K, V tiles)
constexpr int PF_OFF_Q = 0;                                       // [2 slots]
constexpr int PF_OFF_K = PF_OFF_Q + 2 * PF_TILE_BYTES;            // [stages]
constexpr int PF_OFF_V = PF_OFF_K + PF_STAGES * PF_TILE_BYTES;    // [stages], fp16
constexpr int PF_OFF_BAR = PF_OFF_V + PF_STAGES * PF_TILE_BYTES;
// barriers: q_full, q_empty, kv_full[S], kv_empty[S], and per slot s_full,
// s_free, p_full, pv_done
constexpr int PF_NBAR = 2 + 2 * PF_STAGES + 4 * 2;
constexpr int PF_OFF_MISC = PF_OFF_BAR + PF_NBAR * 8;  // tmem base, abort flag
constexpr size_t PF_SMEM = 1024 + PF_OFF_MISC + 16;
constexpr uint32_t PF_TMEM_COLS = 512;
// TMEM columns: S of slot x at 128x, O of slot x at 256 + 64x, P of slot x
// (128 fp16 per row, two per column) at 384 + 64x.
__device__ __forceinline__ uint32_t pf_col_s(int x) { return (uint32_t)(128 * x); }
__device__ __forceinline__ uint32_t pf_col_o(int x) { return (uint32_t)(256 + 64 * x); }
__device__ __forceinline__ uint32_t pf_col_p(int x) { return (uint32_t)(384 + 64 * x); }

// Instruction descriptor, kind::f16 with fp16 A and B (P.V), fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity, err, kDevErrWaitFull)) return true;
  *abort_flag = 1;
  return false;
}

// Warp-uniform wait: every lane polls (and so acquires the phase itself),
// then the warp agrees on one verdict, so no lane can fall out of step with a
// warp-collective tcgen05 instruction.
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                             volatile int* abort_flag) {
  const bool got = pf_wait(bar, parity, err, abort_flag);
  return __all_sync(0xffffffffu, got) != 0;
}

// A work item is a pair of adjacent query tiles (2m, 2m+1) of one (sequence,
// head): slot 0 and slot 1.  Both walk the same causal K/V tiles 0..2m+1 in
// lockstep (slot 0 skips the last), so they share every K/V load.
struct PfItem {
  int b, h, m;
  int qa, qb;        // query tiles of slot 0 / slot 1
  bool b_active;     // slot 1 exists (the last pair of an odd tile count has one tile)
  int nkv;           // K/V tiles the pair walks
};

__device__ __forceinline__ PfItem pf_item(const PrefillParams& p, int idx) {
  // Most expensive pairs (most causal K/V tiles) first.
  const int n_qp = (p.n_qt + 1) >> 1;
  const int bh = p.B * p.n_head;
  PfItem it;
  it.m = n_qp - 1 - idx / bh;
  const int r = idx - (idx / bh) * bh;
  it.b = r / p.n_head;
  it.h = r - it.b * p.n_head;
  it.qa = 2 * it.m;
  it.qb = 2 * it.m + 1;
  it.b_active = it.qb < p.n_qt;
  it.nkv = it.b_active ? it.qb + 1 : it.qa + 1;
  return it;
}

// Steps (K/V tiles) of slot x in an item.
__device__ __forceinline__ int pf_steps(const PfItem& it, int x) {
  return x == 0 ? it.qa + 1 : (it.b_active ? it.qb + 1 : 0);
}

// Roles (384 threads, three warpgroups):
//   warp 0      TMA producer: both Q tiles of an item (128 x 64 bf16 each)
//               and a ring of K (bf16, the cache) and V (fp16 copy) tiles of
//               128 positions, 128B swizzle, no multicast.
//   warp 1      owns TMEM (512 columns); one thread issues tcgen05.mma.  Per
//               slot, S = Q.K^T (M128 N128 K64, bf16) goes into the slot's S
//               columns as soon as the softmax has read the previous S, and
//               O += P.V (M128 N64 K128, fp16, P read from TMEM) follows each
//               P, so the tensor core works while either slot's softmax runs.
//   warps 2-3   idle (complete the producer warpgroup for the register split)
//   warps 4-7   softmax of slot 0, warps 8-11 softmax of slot 1: thread r of
//               a warpgroup owns query row r (TMEM lane r) and all 128 S
//               columns, so a row's maximum and sum never leave the thread.
//               It reads its S row into registers with tcgen05.ld and
//               releases the S columns at once, masks causally, keeps a
//               lazily moved exponent base (O is rescaled in TMEM only when
//               the row maximum grows by more than 2^8), writes its row of P
//               in fp16 (11 significant bits; v is fp16-exact) into the
//               slot's P columns of TMEM, and at the item's end normalises
//               its O row.
// Every mbarrier wait is bounded.  A failed wait records the error word and
// raises a CTA abort flag; every role then leaves its loop, so all threads
// reach the final barrier, issued TMA loads and MMAs are drained (bounded)
// and the TMEM columns are freed before exit.
__global__ void __launch_bounds__(PF_THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmq,
                        const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PF_OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;
  uint64_t* kv_empty = bars + 2 + PF_STAGES;
  uint64_t* s_full = bars + 2 + 2 * PF_STAGES;  // [slot]: Q.K^T done
  uint64_t* s_free = s_full + 2;                // [slot]: S read (4 warps)
  uint64_t* p_full = s_free + 2;                // [slot]: P written to TMEM (4 warps)
  uint64_t* pv_done = p_full + 2;               // [slot]: P.V done (P and O free)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PF_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + PF_OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.B * p.n_head * ((p.n_qt + 1) >> 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < PF_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(PF_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const uint32_t sQ = smem_u32(smem + PF_OFF_Q);
  const uint32_t sK = smem_u32(smem + PF_OFF_K);
  const uint32_t sV = smem_u32(smem + PF_OFF_V);

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PF_REG_PRODUCER));
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tmq);
      tma_prefetch_desc(&tmk);
      tma_prefetch_desc(&tmv);
      long long kvi = 0;
      int it_n = 0;
      for (int idx = blockIdx.x; idx < n_items; idx += gridDim.x, ++it_n) {
        const PfItem it = pf_item(p, idx);
        if (!pf_wait(q_empty, (uint32_t)((it_n & 1) ^ 1), p.err, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, 2 * PF_TILE_BYTES);
        // Slot 1's tile of a one-tile pair reads rows past this sequence
        // (another sequence's, or the map's zero fill); nothing uses them.
        tma_load_3d(smem + PF_OFF_Q, &tmq, q_full, 0, it.h, it.b * p.S + it.qa * PF_M);
        tma_load_3d(smem + PF_OFF_Q + PF_TILE_BYTES, &tmq, q_full, 0, it.h,
                    it.b * p.S + it.qb * PF_M);
        const int g = it.h / p.group;
        bool ok = true;
        for (int j = 0; j < it.nkv; ++j, ++kvi) {
          const int st = (int)(kvi % PF_STAGES);
          const uint32_t ph = (uint32_t)((kvi / PF_STAGES) & 1);
          if (!pf_wait(&kv_empty[st], ph ^ 1u, p.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * PF_TILE_BYTES);
          const int yk = (int)(p.row0 + (long long)it.b * p.max_ctx + (long long)j * PF_N);
          const int yv = it.b * p.S + j * PF_N;  // rows past the sequence are never weighted
          tma_load_2d(smem + PF_OFF_K + st * PF_TILE_BYTES, &tmk, &kv_full[st], 64 * g, yk);
          tma_load_2d(smem + PF_OFF_V + st * PF_TILE_BYTES, &tmv, &kv_full[st], 64 * g, yv);
        }
        if (!ok) break;
      }
      // Drain: the most recent loads of every buffer must have landed.
      if (it_n > 0) mbar_wait(q_full, (uint32_t)((it_n - 1) & 1), p.err, kDevErrWaitFull);
      for (long long k = kvi - PF_STAGES; k < kvi; ++k)
        if (k >= 0)
          mbar_wait(&kv_full[k % PF_STAGES], (uint32_t)((k / PF_STAGES) & 1), p.err,
                    kDevErrWaitFull);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = idesc_bf16(PF_M, PF_N, false);
      constexpr uint32_t IDESC_PV = idesc_f16(PF_M, 64, true);
      // Shared-memory descriptors of the region bases, built once: a
      // descriptor's address field is (byte address >> 4), so an operand at
      // base + off is the base descriptor + off / 16 (every offset here is a
      // multiple of 16 and the region stays below 256 KB, inside the field).
      const uint64_t dq0 = smem_desc_sw128(sQ, 16, 1024);
      const uint64_t dk0 = smem_desc_sw128(sK, 16, 1024);
      const uint64_t dv0 = smem_desc_sw128(sV, PF_TILE_BYTES, 1024);
      long long kvi = 0;
      long long nq[2] = {0, 0};  // Q.K^T issued per slot (S uses)
      long long np[2] = {0, 0};  // P.V issued per slot (P buffer uses)
      int it_n = 0;
      bool issued_any = false, ok = true;
      // S = Q.K^T of slot x from ring slot st; waits until the softmax has
      // read the slot's previous S.
      auto issue_qk = [&](int x, int st) -> bool {
        if (nq[x] > 0 &&
            !pf_wait(&s_free[x], (uint32_t)((nq[x] - 1) & 1), p.err, abort_flag))
          return false;
        tc_fence_after();
        const uint64_t a0 = dq0 + (uint64_t)(x * (PF_TILE_BYTES >> 4));
        const uint64_t b0 = dk0 + (uint64_t)(st * (PF_TILE_BYTES >> 4));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 32 bytes along K per step: +2
          umma_f16(tmem + pf_col_s(x), a0 + 2 * kk, b0 + 2 * kk, IDESC_QK, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[x]);
        ++nq[x];
        issued_any = true;
        return true;
      };
      // O += P.V of slot x: P from the slot's TMEM columns (16 keys = 8
      // columns per step), V from ring slot st (MN-major, 16 rows = +128).
      auto issue_pv = [&](int x, int st, bool first) -> bool {
        if (!pf_wait(&p_full[x], (uint32_t)(np[x] & 1), p.err, abort_flag)) return false;
        tc_fence_after();
        const uint64_t vb = dv0 + (uint64_t)(st * (PF_TILE_BYTES >> 4));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_ts(tmem + pf_col_o(x), tmem + pf_col_p(x) + 8 * kk, vb + 128 * kk, IDESC_PV,
                      (!first || kk > 0) ? 1u : 0u);
        umma_commit(&pv_done[x]);
        ++np[x];
        return true;
      };
      for (int idx = blockIdx.x; idx < n_items && ok; idx += gridDim.x, ++it_n) {
        const PfItem it = pf_item(p, idx);
        const int n0 = pf_steps(it, 0), n1 = pf_steps(it, 1);
        if (!pf_wait(q_full, (uint32_t)(it_n & 1), p.err, abort_flag)) break;
        if (!pf_wait(&kv_full[(int)(kvi % PF_STAGES)], (uint32_t)((kvi / PF_STAGES) & 1), p.err,
                     abort_flag))
          break;
        tc_fence_after();
        ok = issue_qk(0, (int)(kvi % PF_STAGES));
        if (ok && n1 > 0) ok = issue_qk(1, (int)(kvi % PF_STAGES));
        for (int j = 0; j < it.nkv && ok; ++j) {
          const long long slot = kvi + j;
          const int st = (int)(slot % PF_STAGES), st1 = (int)((slot + 1) % PF_STAGES);
          // The next Q.K^T of each slot as soon as its S has been read ...
          if (j + 1 < it.nkv) {
            if (!pf_wait(&kv_full[st1], (uint32_t)(((slot + 1) / PF_STAGES) & 1), p.err,
                         abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            if (j + 1 < n0) ok = issue_qk(0, st1);
            if (ok && j + 1 < n1) ok = issue_qk(1, st1);
            if (!ok) break;
          }
          // ... and this step's P.V of each slot once its P is written.
          if (j < n0) ok = issue_pv(0, st, j == 0);
          if (ok && j < n1) ok = issue_pv(1, st, j == 0);
          if (!ok) break;
          umma_commit(&kv_empty[st]);  // both slots' products of tile j issued
          if (j + 1 == it.nkv) umma_commit(q_empty);
        }
        kvi += it.nkv;
      }
      // Drain: wait (bounded) until every issued MMA has completed.
      if (issued_any) {
        umma_commit(q_empty);
        mbar_wait(q_empty, (uint32_t)(it_n & 1), p.err, kDevErrWaitFull);
      }
    }
    __syncwarp();
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(PF_REG_SOFTMAX));
    // ------------------------------------------------------------ softmax
    const int x = (warp - 4) >> 2;          // slot of this warpgroup
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;    // query row within the tile
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const float scale = p.scale_log2;
    // The exponent base of a row (m_use, raw score units) is only moved when
    // the row's max has grown by more than kLazy in log2 units; until then
    // probabilities may reach 2^kLazy, and O and l need no rescaling.
    constexpr float kLazy = 8.f;
    long long xs = 0;  // this slot's steps so far (barrier phases)
    for (int idx = blockIdx.x; idx < n_items; idx += gridDim.x) {
      const PfItem it = pf_item(p, idx);
      const int nx = pf_steps(it, x);
      if (nx == 0) continue;
      const int qt = x == 0 ? it.qa : it.qb;
      const int q_pos = qt * PF_M + row;
      float m_use = -INFINITY;
      float l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < nx; ++j, ++xs) {
        if (!pf_wait_warp(&s_full[x], (uint32_t)(xs & 1), p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[128];
        TG_TMEM_LD64(tmem + lane_addr + pf_col_s(x), sv);
        TG_TMEM_LD64(tmem + lane_addr + pf_col_s(x) + 64, (sv + 64));
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);  // the next Q.K^T may overwrite S
        // Key position j*128 + c is visible to query q_pos when it is not
        // after it and lies inside the sequence; only the diagonal tile and a
        // partial last tile need the mask.
        const int lim = min(q_pos - j * PF_N, p.S - 1 - j * PF_N);
        // Row maximum over 8 independent running maxima (a single running
        // maximum would be a chain of 128 dependent operations).
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx8[u] = -INFINITY;
        if (__reduce_min_sync(0xffffffffu, lim) >= 127) {
#pragma unroll
          for (int c = 0; c < 128; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(sv[c]));
        } else {
#pragma unroll
          for (int c = 0; c < 128; ++c) {
            const float s = (c <= lim) ? __uint_as_float(sv[c]) : -INFINITY;
            sv[c] = __float_as_uint(s);
            mx8[c & 7] = fmaxf(mx8[c & 7], s);
          }
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        float alpha = 1.f;
        if (j == 0) {
          m_use = mx;
        } else if ((mx - m_use) * scale > kLazy) {
          alpha = ex2((m_use - mx) * scale);
          m_use = mx;
        }
        // The previous P.V of this slot must be done before its P columns
        // are rewritten or its O row rescaled.
        if (j > 0 || xs > 0) {
          if (!pf_wait_warp(&pv_done[x], (uint32_t)((xs - 1) & 1), p.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t ov[32];
            const uint32_t oaddr = tmem + lane_addr + pf_col_o(x) + c0;
            TG_TMEM_LD32(oaddr, ov);
#pragma unroll
            for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
            TG_TMEM_ST32(oaddr, ov);
          }
        }
        const float neg = -m_use * scale;
        // p = 2^(s*scale - m) in fp16 (RNE), two per TMEM column, written in
        // two stores of 32 columns.
        float ls4[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t w[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = half * 64 + 2 * e;
            const float p0 = ex2(fmaf(__uint_as_float(sv[c]), scale, neg));
            const float p1 = ex2(fmaf(__uint_as_float(sv[c + 1]), scale, neg));
            ls4[e & 3] += p0 + p1;
            const __half2 h2 = __floats2half2_rn(p0, p1);
            w[e] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          TG_TMEM_ST32(tmem + lane_addr + pf_col_p(x) + 32 * half, w);
        }
        const float lsum = (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
        l_run = l_run * alpha + lsum;
        tc_fence_before();  // the P stores (waited) before the MMA that reads them
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      if (!ok) break;
      // Epilogue: the last P.V, then O / l for this row.
      if (!pf_wait_warp(&pv_done[x], (uint32_t)((xs - 1) & 1), p.err, abort_flag)) break;
      tc_fence_after();
      uint32_t ov[64];
      TG_TMEM_LD64(tmem + lane_addr + pf_col_o(x), ov);
      tc_fence_before();
      if (q_pos < p.S) {
        const float inv = 1.f / l_run;
        float* dst = p.out + (((size_t)it.b * p.S + q_pos) * p.n_head + it.h) * 64;
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          float4 w;
          w.x = __uint_as_float(ov[c]) * inv;
          w.y = __uint_as_float(ov[c + 1]) * inv;
          w.z = __uint_as_float(ov[c + 2]) * inv;
          w.w = __uint_as_float(ov[c + 3]) * inv;
          *reinterpret_cast<float4*>(dst + c) = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(PF_TMEM_COLS)
                 : "memory");
  }
}

size_t prefill_attn_smem() { return PF_SMEM; }

cudaError_t launch_prefill_rope(const PrefillRopeParams& p, cudaStream_t st) {
  if (p.B <= 0 || p.S <= 0) return cudaSuccess;
  const bool rows16 =
      p.head_dim == 64 &&
      ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k) |
        reinterpret_cast<uintptr_t>(p.v) | reinterpret_cast<uintptr_t>(p.cs) |
        reinterpret_cast<uintptr_t>(p.q_bf16) | reinterpret_cast<uintptr_t>(p.k_cache) |
        reinterpret_cast<uintptr_t>(p.v_cache) | reinterpret_cast<uintptr_t>(p.v_f16)) &
       15) == 0;
  if (rows16)
    prefill_rope_rows_kernel<<<(p.B * p.S + 7) / 8, 256, 0, st>>>(p);
  else
    prefill_rope_kernel<<<p.B * p.S, 128, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_prefill_attn(const CUtensorMap& tq, const CUtensorMap& tk,
                                const CUtensorMap& tv, const PrefillParams& p, int grid,
                                cudaStream_t st) {
  static size_t configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (configured[dev] < PF_SMEM) {
    cudaError_t e = cudaFuncSetAttribute(prefill_attn_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM);
    if (e != cudaSuccess) return e;
    configured[dev] = PF_SMEM;
  }
  prefill_attn_kernel<<<grid, PF_THREADS, PF_SMEM, st>>>(tq, tk, tv, p);
  return cudaGetLastError();
}

}  // namespace tg
