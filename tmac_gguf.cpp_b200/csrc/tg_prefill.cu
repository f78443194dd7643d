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
// prefill_attn_kernel roles (320 threads):
//   warp 0      TMA producer: the item's Q tile (128 x 64 bf16) and a ring of
//               K/V tiles (128 positions x 64 bf16 each), 128B swizzle.
//   warp 1      owns TMEM (512 columns) and one thread issues tcgen05.mma:
//               S = Q.K^T (M128 N128 K64) into one of two TMEM S buffers,
//               O += P.V (M128 N64 K128) into the TMEM O accumulator.
//   warps 2-9   softmax / correction / epilogue: query row i (TMEM lane i)
//               belongs to two threads, one per half of the S columns.  Each
//               reads its half row with tcgen05.ld, masks causally, trades
//               its half-row maximum with the partner through shared memory,
//               computes the online softmax, rescales its half of the O row
//               in TMEM and writes its half of P to shared memory as bf16 hi
//               and lo parts; the MMA issues P_hi.V and P_lo.V, so the
//               probabilities keep ~15 mantissa bits.
//
// Every mbarrier wait is bounded.  A failed wait records the error word and
// raises a CTA abort flag; every role then leaves its loop, so all threads
// reach the final barrier, issued TMA loads and MMAs are drained (bounded)
// and the TMEM columns are freed before exit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "tg_device.cuh"
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

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
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

// Arrive on `bar` once every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 64 consecutive TMEM columns of this thread's lane; the wait is part of the
// same asm statement so the destination registers are defined only after
// the load has completed.
#define TG_TMEM_LD64(taddr, v)                                                                 \
  asm volatile(                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "  \
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "  \
      "%28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, "  \
      "%45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, "  \
      "%62, %63}, [%64];\n\ttcgen05.wait::ld.sync.aligned;"                                  \
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),    \
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),            \
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),         \
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),         \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),         \
        "=r"(v[31]), "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]),         \
        "=r"(v[37]), "=r"(v[38]), "=r"(v[39]), "=r"(v[40]), "=r"(v[41]), "=r"(v[42]),         \
        "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]), "=r"(v[48]),         \
        "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]),         \
        "=r"(v[55]), "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]),         \
        "=r"(v[61]), "=r"(v[62]), "=r"(v[63])                                                 \
      : "r"(taddr))

// Store 64 columns of this thread's lane and wait for completion.
#define TG_TMEM_ST64(taddr, v)                                                                 \
  asm volatile(                                                                                \
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "     \
      "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, "  \
      "%27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, "  \
      "%44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, "  \
      "%61, %62, %63, %64};\n\ttcgen05.wait::st.sync.aligned;" ::"r"(taddr),                  \
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), \
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),       \
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),     \
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),     \
      "r"(v[29]), "r"(v[30]), "r"(v[31]), "r"(v[32]), "r"(v[33]), "r"(v[34]), "r"(v[35]),     \
      "r"(v[36]), "r"(v[37]), "r"(v[38]), "r"(v[39]), "r"(v[40]), "r"(v[41]), "r"(v[42]),     \
      "r"(v[43]), "r"(v[44]), "r"(v[45]), "r"(v[46]), "r"(v[47]), "r"(v[48]), "r"(v[49]),     \
      "r"(v[50]), "r"(v[51]), "r"(v[52]), "r"(v[53]), "r"(v[54]), "r"(v[55]), "r"(v[56]),     \
      "r"(v[57]), "r"(v[58]), "r"(v[59]), "r"(v[60]), "r"(v[61]), "r"(v[62]), "r"(v[63])      \
      : "memory")

#define TG_TMEM_LD32(taddr, v)                                                                 \
  asm volatile(                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "  \
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "  \
      "%28, %29, %30, %31}, [%32];\n\ttcgen05.wait::ld.sync.aligned;"                          \
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),    \
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),            \
        "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]),         \
        "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),         \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]),         \
        "=r"(v[31])                                                                            \
      : "r"(taddr))

#define TG_TMEM_ST32(taddr, v)                                                                 \
  asm volatile(                                                                                \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, "     \
      "%10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, "  \
      "%27, %28, %29, %30, %31, %32};\n\ttcgen05.wait::st.sync.aligned;" ::"r"(taddr),         \
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), \
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),       \
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),     \
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),     \
      "r"(v[29]), "r"(v[30]), "r"(v[31])                                                      \
      : "memory")

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: canonical K-major or MN-major layout with
// 128-byte swizzle (8-row atoms of 1024 bytes), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
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
  for (int i = threadIdx.x; i < kdim; i += blockDim.x) vc[i] = __float2bfloat16_rn(v[i]);
}

// ------------------------------------------------------------ attention

constexpr int PF_M = 128;          // query rows per tile (TMEM lanes)
constexpr int PF_N = 128;          // cache rows per K/V tile
constexpr int PF_STAGES = 2;       // K/V ring depth
constexpr int PF_THREADS = 320;   // TMA warp, MMA warp, 8 softmax warps
constexpr int PF_TILE_BYTES = PF_M * 128;  // 128 rows x 64 bf16
constexpr int PF_OFF_Q = 0;
constexpr int PF_OFF_K = PF_OFF_Q + PF_TILE_BYTES;
constexpr int PF_OFF_V = PF_OFF_K + PF_STAGES * PF_TILE_BYTES;
// P: two buffers (steps alternate), each a hi and a lo part of 2 K-blocks.
constexpr int PF_P_BYTES = 2 * PF_TILE_BYTES;  // one part: 128 rows x 128 bf16
constexpr int PF_OFF_P = PF_OFF_V + PF_STAGES * PF_TILE_BYTES;
constexpr int PF_OFF_BAR = PF_OFF_P + 2 * 2 * PF_P_BYTES;
// barriers: q_full, q_empty, kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full,
// o_done[2] (per P buffer), xbar[4] (row-statistics exchange within a lane quarter)
constexpr int PF_NBAR = 2 + 2 * PF_STAGES + 2 + 2 + 1 + 2 + 4;
constexpr int PF_OFF_XCH = PF_OFF_BAR + PF_NBAR * 8;       // float [2 parity][2 half][128]
constexpr int PF_OFF_MISC = PF_OFF_XCH + 2 * 2 * 128 * 4;  // tmem base, abort flag
constexpr size_t PF_SMEM = 1024 + PF_OFF_MISC + 16;
constexpr uint32_t PF_TMEM_COLS = 512;
constexpr uint32_t PF_COL_S0 = 0, PF_COL_S1 = 128, PF_COL_O = 256;

__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait(bar, parity, err, kDevErrWaitFull)) return true;
  *abort_flag = 1;
  return false;
}

// Warp-uniform wait: every lane polls (and so acquires the phase itself),
// then the warp agrees on one verdict, so no lane can fall out of step with a
// warp-collective tcgen05 instruction or leave its partner waiting.
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                             volatile int* abort_flag, int lane) {
  (void)lane;
  const bool got = pf_wait(bar, parity, err, abort_flag);
  return __all_sync(0xffffffffu, got) != 0;
}

struct PfItem {
  int b, h, qt;
};

__device__ __forceinline__ PfItem pf_item(const PrefillParams& p, int idx) {
  // Most expensive query tiles (most causal K/V tiles) first.
  const int bh = p.B * p.n_head;
  PfItem it;
  it.qt = p.n_qt - 1 - idx / bh;
  const int r = idx - (idx / bh) * bh;
  it.b = r / p.n_head;
  it.h = r - it.b * p.n_head;
  return it;
}

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
  uint64_t* s_full = bars + 2 + 2 * PF_STAGES;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 1;  // [2]: P.V of the steps using P buffer 0 / 1
  uint64_t* xbar = o_done + 2;
  float* xch = reinterpret_cast<float*>(smem + PF_OFF_XCH);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + PF_OFF_MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + PF_OFF_MISC + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.B * p.n_head * p.n_qt;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < PF_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 8);
    }
    mbar_init(p_full, 8);
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 64);
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
  const uint32_t sP = smem_u32(smem + PF_OFF_P);  // buffer b part h at b*2*PF_P_BYTES + h*PF_P_BYTES

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
        mbar_arrive_expect_tx(q_full, PF_TILE_BYTES);
        tma_load_3d(smem + PF_OFF_Q, &tmq, q_full, 0, it.h, it.b * p.S + it.qt * PF_M);
        const int g = it.h / p.group;
        const int nkv = it.qt + 1;
        bool ok = true;
        for (int j = 0; j < nkv; ++j, ++kvi) {
          const int st = (int)(kvi % PF_STAGES);
          const uint32_t ph = (uint32_t)((kvi / PF_STAGES) & 1);
          if (!pf_wait(&kv_empty[st], ph ^ 1u, p.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * PF_TILE_BYTES);
          const int y = (int)(p.row0 + (long long)it.b * p.max_ctx + (long long)j * PF_N);
          tma_load_2d(smem + PF_OFF_K + st * PF_TILE_BYTES, &tmk, &kv_full[st], 64 * g, y);
          tma_load_2d(smem + PF_OFF_V + st * PF_TILE_BYTES, &tmv, &kv_full[st], 64 * g, y);
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
      constexpr uint32_t IDESC_PV = idesc_bf16(PF_M, 64, true);
      long long kvi = 0, sc = 0;  // K/V ring slot counter, S step counter
      int it_n = 0;
      bool issued_any = false;
      auto issue_qk = [&](long long step, long long slot) -> bool {
        const int st = (int)(slot % PF_STAGES);
        if (!pf_wait(&kv_full[st], (uint32_t)((slot / PF_STAGES) & 1), p.err, abort_flag))
          return false;
        const int sb = (int)(step & 1);
        if (!pf_wait(&s_free[sb], (uint32_t)(((step >> 1) & 1) ^ 1), p.err, abort_flag))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + (sb ? PF_COL_S1 : PF_COL_S0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t a = smem_desc_sw128(sQ + kk * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(sK + st * PF_TILE_BYTES + kk * 32, 16, 1024);
          umma_f16(d, a, b, IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        issued_any = true;
        return true;
      };
      for (int idx = blockIdx.x; idx < n_items; idx += gridDim.x, ++it_n) {
        const PfItem it = pf_item(p, idx);
        const int nkv = it.qt + 1;
        if (!pf_wait(q_full, (uint32_t)(it_n & 1), p.err, abort_flag)) break;
        tc_fence_after();
        if (!issue_qk(sc, kvi)) break;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
          const long long step = sc + j, slot = kvi + j;
          if (j + 1 < nkv) {
            if (!issue_qk(step + 1, slot + 1)) {
              ok = false;
              break;
            }
          } else {
            umma_commit(q_empty);  // the item's last Q.K^T has been issued
          }
          if (!pf_wait(p_full, (uint32_t)(step & 1), p.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int st = (int)(slot % PF_STAGES);
          const uint32_t pbuf = sP + (uint32_t)(step & 1) * 2 * PF_P_BYTES;
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            const uint32_t pbase = pbuf + part * PF_P_BYTES;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t a =
                  smem_desc_sw128(pbase + (kk >> 2) * PF_TILE_BYTES + (kk & 3) * 32, 16, 1024);
              const uint64_t b =
                  smem_desc_sw128(sV + st * PF_TILE_BYTES + kk * 2048, PF_TILE_BYTES, 1024);
              umma_f16(tmem + PF_COL_O, a, b, IDESC_PV, (j > 0 || part > 0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&o_done[step & 1]);
          umma_commit(&kv_empty[st]);
        }
        if (!ok) break;
        sc += nkv;
        kvi += nkv;
      }
      // Drain: wait (bounded) until every issued MMA has completed.
      if (issued_any) {
        umma_commit(q_empty);
        mbar_wait(q_empty, (uint32_t)(it_n & 1), p.err, kDevErrWaitFull);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    // Warps 2..9: warp pairs (w, w+4) share TMEM lane quarter w%4 (query
    // rows 32*(w%4)..+31); the first of a pair owns S columns 0-63, O
    // columns 0-31 and P block 0, the second the other halves.
    const int sw = warp - 2;
    const int quarter = warp & 3;
    const int half = sw >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const float scale = p.scale_log2;
    // The exponent base of a row (m_use, raw score units) is only moved when
    // the row's max has grown by more than kLazy in log2 units; until then
    // probabilities may reach 2^kLazy, and O and l need no rescaling.
    constexpr float kLazy = 8.f;
    long long sc = 0;
    uint32_t xph = 0;  // phase counter of this quarter's exchange barrier
    // P.V of global step t used P buffer t&1; it is that buffer's use t>>1.
    auto wait_pv = [&](long long t) -> bool {
      return pf_wait_warp(&o_done[t & 1], (uint32_t)((t >> 1) & 1), p.err, abort_flag, lane);
    };
    for (int idx = blockIdx.x; idx < n_items; idx += gridDim.x) {
      const PfItem it = pf_item(p, idx);
      const int nkv = it.qt + 1;
      const int q_pos = it.qt * PF_M + row;
      float m_use = -INFINITY;
      float l_run = 0.f;  // this half-row's share of the softmax sum
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const long long step = sc + j;
        const int sb = (int)(step & 1);
        if (!pf_wait_warp(&s_full[sb], (uint32_t)((step >> 1) & 1), p.err, abort_flag, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[64];
        TG_TMEM_LD64(tmem + lane_addr + (sb ? PF_COL_S1 : PF_COL_S0) + half * 64, sv);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[sb]);
        // Key position j*128 + half*64 + c is visible to query q_pos when it
        // is not after it and lies inside the sequence; only the diagonal
        // tile and a partial last tile need the mask.
        const int k0 = j * PF_N + half * 64;
        const int lim = min(q_pos - k0, p.S - 1 - k0);
        float mx = -INFINITY;
        if (__reduce_min_sync(0xffffffffu, lim) >= 63) {
#pragma unroll
          for (int c = 0; c < 64; ++c) mx = fmaxf(mx, __uint_as_float(sv[c]));
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) {
            const float s = (c <= lim) ? __uint_as_float(sv[c]) : -INFINITY;
            sv[c] = __float_as_uint(s);
            mx = fmaxf(mx, s);
          }
        }
        // Exchange the half-row maxima with the partner warp (bounded wait).
        float* xc = xch + (xph & 1) * 256;
        xc[half * 128 + row] = mx;
        mbar_arrive(&xbar[quarter]);
        if (!pf_wait_warp(&xbar[quarter], xph & 1, p.err, abort_flag, lane)) {
          ok = false;
          break;
        }
        ++xph;
        const float m_tile = fmaxf(mx, xc[(half ^ 1) * 128 + row]);
        float alpha = 1.f;
        if (j == 0) {
          m_use = m_tile;
        } else if ((m_tile - m_use) * scale > kLazy) {
          alpha = ex2((m_use - m_tile) * scale);
          m_use = m_tile;
        }
        // O rescale: needs every earlier P.V finished (the last one issued).
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          if (!wait_pv(step - 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t ov[32];
          const uint32_t oaddr = tmem + lane_addr + PF_COL_O + half * 32;
          TG_TMEM_LD32(oaddr, ov);
#pragma unroll
          for (int c = 0; c < 32; ++c) ov[c] = __float_as_uint(__uint_as_float(ov[c]) * alpha);
          TG_TMEM_ST32(oaddr, ov);
        }
        // P buffer step&1 is free once the P.V two steps back has finished.
        if (step >= 2 && !wait_pv(step - 2)) {
          ok = false;
          break;
        }
        const float neg = -m_use * scale;
        // p = 2^(s*scale - m); P = hi + lo with hi = p truncated to bf16 and
        // lo = bf16(p - hi): ~2^-14 relative, packed with byte permutes.
        float lsum = 0.f;
        const uint32_t pbase =
            sP + (uint32_t)(step & 1) * 2 * PF_P_BYTES + half * PF_TILE_BYTES + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = ch * 8 + 2 * e;
            const float p0 = ex2(fmaf(__uint_as_float(sv[c]), scale, neg));
            const float p1 = ex2(fmaf(__uint_as_float(sv[c + 1]), scale, neg));
            lsum += p0 + p1;
            const uint32_t b0 = __float_as_uint(p0), b1 = __float_as_uint(p1);
            const float r0 = p0 - __uint_as_float(b0 & 0xFFFF0000u);
            const float r1 = p1 - __uint_as_float(b1 & 0xFFFF0000u);
            hi[e] = __byte_perm(b0, b1, 0x7632);
            lo[e] = __byte_perm(__float_as_uint(r0), __float_as_uint(r1), 0x7632);
          }
          const uint32_t off = pbase + ((ch ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(off), "r"(hi[0]),
                       "r"(hi[1]), "r"(hi[2]), "r"(hi[3])
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(off + PF_P_BYTES),
                       "r"(lo[0]), "r"(lo[1]), "r"(lo[2]), "r"(lo[3])
                       : "memory");
        }
        l_run = l_run * alpha + lsum;
        fence_proxy_async_smem();  // P (generic writes) before the tensor core reads it
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      sc += nkv;
      // Epilogue: the two halves' sums, then O / l for this warp's 32 columns.
      if (!wait_pv(sc - 1)) break;
      tc_fence_after();
      float* xc = xch + (xph & 1) * 256;
      xc[half * 128 + row] = l_run;
      mbar_arrive(&xbar[quarter]);
      if (!pf_wait_warp(&xbar[quarter], xph & 1, p.err, abort_flag, lane)) break;
      ++xph;
      const float l_tot = l_run + xc[(half ^ 1) * 128 + row];
      uint32_t ov[32];
      TG_TMEM_LD32(tmem + lane_addr + PF_COL_O + half * 32, ov);
      tc_fence_before();
      if (q_pos < p.S) {
        const float inv = 1.f / l_tot;
        float* dst = p.out + (((size_t)it.b * p.S + q_pos) * p.n_head + it.h) * 64 + half * 32;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
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
