// tg_kernels.cu -- CUDA kernels of the decode-attention hot path (sm_100a).
//
//   rope_cache_write_kernel   RoPE on q and k + K/V cache-write, one CTA per
//                             sequence (tmac_gguf.cpp:990-1016, :1090-1091;
//                             kernel_rope.metal, kernel_elem.metal op 2).
//   decode_mma_kernel<NKV>    split-KV GQA decode attention over a bf16
//                             cache: TMA-staged K/V tiles, warp-level bf16
//                             tensor-core products with hi/lo operand
//                             splitting, online softmax with warp shuffles
//                             (tmac_gguf.cpp:1093-1128, kernel_attn.metal).
//   decode_generic_kernel<T>  the same contract on CUDA cores for fp32 (and
//                             any shape the tensor-core kernel does not take).
//   decode_small_kernel<T>    caches of at most kSmallMaxRows positions
//                             (head_dim 64): one CTA per (sequence, KV head),
//                             no split, no merge.
//   merge_kernel              combines the partial records of sequences that
//                             were split across CTAs.
//   gather_merge_kernel       combines per-GPU records after the all-gather.
//   elem_kernel, fill_normal_kernel  elem_op ops 0/2 and synthetic inputs.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cooperative_groups.h>

#include <mutex>

#include <utility>

#include "tg_device.cuh"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace tg {

// ===================================================================== RoPE

__global__ void __launch_bounds__(128) rope_cache_write_kernel(const RopeParams p) {
  griddep_launch_dependents();
  griddep_wait();
  const int s = blockIdx.x;
  const int pos = p.pos ? p.pos[s] : p.pos_scalar;
  if (pos < 0 || pos >= p.table_len) {
    if (threadIdx.x == 0) record_error(p.err, kDevErrBadPos);
    return;
  }
  const int hd = p.head_dim, half = hd >> 1;
  const float* cs = p.cs + (size_t)pos * hd;  // [half][cos, sin]

  // Every thread first loads up to RU pairs (and their cos/sin), then
  // rotates and stores them: one memory latency per batch, not per pair.
  constexpr int RU = 4;
  if (p.q) {
    float* q = p.q + (size_t)s * p.n_head * hd;
    const int n_pairs = p.n_head * half;
    for (int b0 = 0; b0 < n_pairs; b0 += blockDim.x * RU) {
      float2 x[RU], c2[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int i = b0 + u * blockDim.x + threadIdx.x;
        if (i < n_pairs) {
          const int h = i / half, j = i - h * half;
          x[u] = *reinterpret_cast<const float2*>(q + h * hd + 2 * j);
          c2[u] = *reinterpret_cast<const float2*>(cs + 2 * j);
        }
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int i = b0 + u * blockDim.x + threadIdx.x;
        if (i < n_pairs) {
          const int h = i / half, j = i - h * half;
          // x0*c - x1*s and x0*s + x1*c, each product and sum rounded once.
          float2 y;
          y.x = __fsub_rn(__fmul_rn(x[u].x, c2[u].x), __fmul_rn(x[u].y, c2[u].y));
          y.y = __fadd_rn(__fmul_rn(x[u].x, c2[u].y), __fmul_rn(x[u].y, c2[u].x));
          *reinterpret_cast<float2*>(q + h * hd + 2 * j) = y;
        }
      }
    }
  }

  const int kdim = p.n_kv * hd;
  const int local = pos - p.shard_start;
  const bool write = p.k_cache && local >= 0 && local < p.max_ctx;
  const size_t row = ((size_t)s * p.max_ctx + (write ? local : 0)) * kdim;

  if (p.k) {
    float* k = p.k + (size_t)s * kdim;
    const int n_pairs = p.n_kv * half;
    for (int b0 = 0; b0 < n_pairs; b0 += blockDim.x * RU) {
      float2 x[RU], c2[RU];
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int i = b0 + u * blockDim.x + threadIdx.x;
        if (i < n_pairs) {
          const int h = i / half, j = i - h * half;
          x[u] = *reinterpret_cast<const float2*>(k + h * hd + 2 * j);
          c2[u] = *reinterpret_cast<const float2*>(cs + 2 * j);
        }
      }
#pragma unroll
      for (int u = 0; u < RU; ++u) {
        const int i = b0 + u * blockDim.x + threadIdx.x;
        if (i < n_pairs) {
          const int h = i / half, j = i - h * half;
          const int idx = h * hd + 2 * j;
          const float r0 = __fsub_rn(__fmul_rn(x[u].x, c2[u].x), __fmul_rn(x[u].y, c2[u].y));
          const float r1 = __fadd_rn(__fmul_rn(x[u].x, c2[u].y), __fmul_rn(x[u].y, c2[u].x));
          *reinterpret_cast<float2*>(k + idx) = make_float2(r0, r1);
          if (write) {
            if (p.dtype == 0) {
              *reinterpret_cast<float2*>(static_cast<float*>(p.k_cache) + row + idx) =
                  make_float2(r0, r1);
            } else {
              *reinterpret_cast<__nv_bfloat162*>(static_cast<__nv_bfloat16*>(p.k_cache) + row +
                                                 idx) = __floats2bfloat162_rn(r0, r1);
            }
          }
        }
      }
    }
  }
  if (write && p.v) {
    const float* v = p.v + (size_t)s * kdim;
    for (int i = threadIdx.x; i < kdim; i += blockDim.x) {
      if (p.dtype == 0)
        static_cast<float*>(p.v_cache)[row + i] = v[i];
      else
        static_cast<__nv_bfloat16*>(p.v_cache)[row + i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// ============================================================ tile schedule

// Builds prefix[0..B] (tiles per sequence, exclusive scan) in shared memory
// with all threads of the block; warp_tot is 32 ints of scratch.  Invalid
// positions are recorded and contribute no tiles.
__device__ void build_tile_prefix(const DecodeParams& p, int tile, int* prefix,
                                  int* warp_tot) {
  const int NT = blockDim.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int chunk = (p.B + NT - 1) / NT;
  const int b0 = min(t * chunk, p.B), b1 = min(b0 + chunk, p.B);
  const int pos_limit = p.shard_start + p.max_ctx;
  int sum = 0;
  for (int s = b0; s < b1; ++s) {
    const int pl = past_of(p, s);
    int tiles = 0;
    if (pl < 0 || (p.mode == 0 && pl >= pos_limit)) {
      record_error(p.err, kDevErrBadPos);
    } else {
      const int n = local_rows(pl, p.shard_start, p.max_ctx);
      tiles = (n + tile - 1) / tile;
    }
    prefix[s + 1] = tiles;
    sum += tiles;
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int nw = (NT + 31) >> 5;
    const int v = lane < nw ? warp_tot[lane] : 0;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane < nw) warp_tot[lane] = inc - v;
  }
  __syncthreads();
  int run = warp_tot[w] + incl - sum;
  if (t == 0) prefix[0] = 0;
  for (int s = b0; s < b1; ++s) {
    run += prefix[s + 1];
    prefix[s + 1] = run;
  }
  __syncthreads();
}

// Where a finished segment's state goes.
struct SegDest {
  float* ptr;     // record base or output row base
  bool normalise; // write O / L (mode 0, complete sequence)
};

__device__ __forceinline__ SegDest segment_dest(const DecodeParams& p, int s,
                                                long long seg_lo,
                                                long long seg_hi,
                                                long long t_lo,
                                                const int* prefix, int cta) {
  const int rf = record_floats(p.n_head, p.head_dim);
  const bool complete = seg_lo == prefix[s] && seg_hi == prefix[s + 1];
  SegDest d;
  if (complete) {
    if (p.mode == 0) {
      d.ptr = p.out + (size_t)s * p.n_head * p.head_dim;
      d.normalise = true;
    } else {
      d.ptr = p.records + (size_t)s * rf;
      d.normalise = false;
    }
  } else {
    const int slot = 2 * cta + (seg_lo == t_lo ? 0 : 1);
    d.ptr = p.part + (size_t)slot * rf;
    d.normalise = false;
  }
  return d;
}

// ========================================================= tensor-core path

template <int NKV>
struct MmaCfg {
  static constexpr int TILE = 64;                 // cache rows per stage
  // 128 KB ring: enough K/V in flight per SM to cover loaded HBM latency
  // (a pure TMA stream of this tiling reaches the copy peak with it).
  static constexpr int STAGES = (128 * 1024) / (2 * NKV * TILE * 128);
  static constexpr int CWARPS = 2 * NKV;          // consumer warps
  static constexpr int THREADS = 32 * (CWARPS + 1);
  static constexpr int BOX = TILE * 128;          // one KV head's rows: 64 bf16
  static constexpr int STAGE_BYTES = 2 * NKV * BOX;
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int MRG_FLOATS = 8 * 64 + 16;  // o[8][64], m[8], l[8]
  static constexpr int OFF_MRG = OFF_BAR + 2 * STAGES * 8;
  static constexpr int OFF_WTOT = OFF_MRG + CWARPS * MRG_FLOATS * 4;
  static constexpr int OFF_PREFIX = OFF_WTOT + 32 * 4;
  static constexpr size_t smem_bytes(int B) {
    return 1024 + OFF_PREFIX + (size_t)(B + 1) * 4;
  }
};

__device__ __forceinline__ void consumer_bar_sync(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// One CTA: a producer warp streams K/V tiles of its flat tile range into a
// STAGES-deep shared-memory ring with TMA; consumer warp w handles KV head
// g = w/2 and rows [32*(w%2), 32*(w%2)+32) of every tile.  Each consumer
// warp keeps an online-softmax state for the (up to 8) query heads of its KV
// head: rows 0-7 of the m16 tile carry the bf16 "hi" part of q (or of the
// probabilities), rows 8-15 the bf16 "lo" remainder, so one m16n8k16 product
// yields hi + lo in the same thread and the products keep ~17 mantissa bits.
template <int NKV>
__global__ void __launch_bounds__(MmaCfg<NKV>::THREADS, 1)
    decode_mma_kernel(const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmv,
                      const DecodeParams p) {
  using Cfg = MmaCfg<NKV>;
  constexpr int TILE = Cfg::TILE, STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  float* mrg = reinterpret_cast<float*>(smem + Cfg::OFF_MRG);
  int* warp_tot = reinterpret_cast<int*>(smem + Cfg::OFF_WTOT);
  int* prefix = reinterpret_cast<int*>(smem + Cfg::OFF_PREFIX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  griddep_launch_dependents();
  griddep_wait();
  build_tile_prefix(p, TILE, prefix, warp_tot);
  const long long T = prefix[p.B];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= p.B; i += blockDim.x) p.sched[i] = prefix[i];
  // Effective grid: never more CTAs than tiles, so no CTA range is empty.
  const int G = (int)min((long long)gridDim.x, T), cta = blockIdx.x;
  if (cta >= G) return;
  const long long t_lo = cta_tile_lo(cta, G, T), t_hi = cta_tile_lo(cta + 1, G, T);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Cfg::CWARPS);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == Cfg::CWARPS) {
    // ------------------------------------------------------------ producer
    if (lane != 0) return;
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    int s = 0;
    long long i = 0;
    bool ok = true;
    for (long long t = t_lo; t < t_hi; ++t, ++i) {
      while (prefix[s + 1] <= t) ++s;
      const int j = (int)(t - prefix[s]);
      const int st = (int)(i % STAGES);
      const uint32_t ph = (uint32_t)((i / STAGES) & 1);
      if (!mbar_wait(&empty[st], ph ^ 1u, p.err, kDevErrWaitEmpty)) {
        ok = false;
        break;
      }
      uint8_t* stage = smem + st * Cfg::STAGE_BYTES;
      mbar_arrive_expect_tx(&full[st], Cfg::STAGE_BYTES);
      const int y = (int)(p.row0 + (long long)s * p.max_ctx + (long long)j * TILE);
#pragma unroll
      for (int g = 0; g < NKV; ++g) {
        tma_load_2d(stage + g * Cfg::BOX, &tmk, &full[st], 64 * g, y);
        tma_load_2d(stage + (NKV + g) * Cfg::BOX, &tmv, &full[st], 64 * g, y);
      }
    }
    // Drain: every issued load must land before the CTA may exit.
    const long long issued = i;
    for (long long k = issued - STAGES; k < issued; ++k) {
      if (k < 0) continue;
      const int st = (int)(k % STAGES);
      mbar_wait(&full[st], (uint32_t)((k / STAGES) & 1), p.err, kDevErrWaitFull);
    }
    (void)ok;
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g = warp >> 1, hf = warp & 1;
  const int r = lane >> 2, qd = lane & 3;  // mma row (query head) / quad lane
  const bool row_ok = r < p.group;
  const float sl2 = p.scale_log2;
  float* my_mrg = mrg + warp * Cfg::MRG_FLOATS;

  uint32_t qa[4][4];                 // q A-fragments, 4 k-steps of 16 dims
  float o[8][4];                     // O accumulators, 8 chunks of 8 dims
  float m_run = kNegBig, l_run = 0.f;
  bool failed = false;

  int s = 0;
  long long i = 0;
  long long seg_lo = t_lo;
  for (long long t = t_lo; t < t_hi; ++t, ++i) {
    const bool new_seg = (t == seg_lo) || (t == prefix[s + 1]);
    while (prefix[s + 1] <= t) ++s;
    if (new_seg) {
      seg_lo = t;
      // Load this warp's query heads and split them into bf16 hi + lo.
      const float* qh = p.q + ((size_t)s * p.n_head + (size_t)g * p.group + (row_ok ? r : 0)) * 64;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float2 v = make_float2(0.f, 0.f);
          if (row_ok) v = *reinterpret_cast<const float2*>(qh + 16 * kk + 8 * half + 2 * qd);
          float h0, l0, h1, l1;
          split_bf16(v.x, h0, l0);
          split_bf16(v.y, h1, l1);
          qa[kk][2 * half] = pack_bf16x2(h0, h1);
          qa[kk][2 * half + 1] = pack_bf16x2(l0, l1);
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) o[c][0] = o[c][1] = o[c][2] = o[c][3] = 0.f;
      m_run = kNegBig;
      l_run = 0.f;
    }
    const int j = (int)(t - prefix[s]);
    const int n_loc = local_rows(past_of(p, s), p.shard_start, p.max_ctx);
    const int tile_valid = min(TILE, n_loc - j * TILE);
    const int my_valid = max(0, min(32, tile_valid - 32 * hf));

    const int st = (int)(i % STAGES);
    const uint32_t ph = (uint32_t)((i / STAGES) & 1);
    if (!failed && !mbar_wait(&full[st], ph, p.err, kDevErrWaitFull)) failed = true;

    if (!failed && my_valid > 0) {
      uint8_t* kbox = smem + st * Cfg::STAGE_BYTES + g * Cfg::BOX;
      uint8_t* vbox = smem + st * Cfg::STAGE_BYTES + (NKV + g) * Cfg::BOX;
      const int rb = 32 * hf;  // first row of this warp in the tile
      if (my_valid < 32) {
        // Rows past the attended window may hold anything; zero their V so
        // that 0-weighted rows add exactly zero.
        for (int e = lane; e < (32 - my_valid) * 8; e += 32) {
          const int row = rb + my_valid + (e >> 3);
          reinterpret_cast<uint4*>(vbox + row * 128)[e & 7] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
      }
      const uint32_t kb = smem_u32(kbox), vb = smem_u32(vbox);

      // S = q . K^T for 32 rows: 4 n-tiles of 8 rows.
      float sc[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int row = rb + 8 * nt + (lane & 7);
#pragma unroll
        for (int kq = 0; kq < 2; ++kq) {
          const int chunk = 4 * kq + (lane >> 3);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(kb + row * 128 + ((chunk ^ (row & 7)) << 4), b0, b1, b2, b3);
          mma_bf16_16816(acc, qa[2 * kq], b0, b1);
          mma_bf16_16816(acc, qa[2 * kq + 1], b2, b3);
        }
        const int c0 = 8 * nt + 2 * qd;
        sc[nt][0] = (c0 < my_valid) ? (acc[0] + acc[2]) * sl2 : -INFINITY;
        sc[nt][1] = (c0 + 1 < my_valid) ? (acc[1] + acc[3]) * sl2 : -INFINITY;
      }
      // Online softmax over the 32 rows (per query head = per quad).
      float mx = fmaxf(fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1])),
                       fmaxf(fmaxf(sc[2][0], sc[2][1]), fmaxf(sc[3][0], sc[3][1])));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = ex2(m_run - m_new);
      m_run = m_new;
      float pr[4][2];
      float lsum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        pr[nt][0] = ex2(sc[nt][0] - m_new);
        pr[nt][1] = ex2(sc[nt][1] - m_new);
        lsum += pr[nt][0] + pr[nt][1];
      }
      l_run = l_run * alpha + lsum;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        o[c][0] *= alpha; o[c][1] *= alpha; o[c][2] *= alpha; o[c][3] *= alpha;
      }
      // O += P . V, two k-steps of 16 rows.
#pragma unroll
      for (int kp = 0; kp < 2; ++kp) {
        uint32_t pa[4];
        float h0, l0, h1, l1;
        split_bf16(pr[2 * kp][0], h0, l0);
        split_bf16(pr[2 * kp][1], h1, l1);
        pa[0] = pack_bf16x2(h0, h1);
        pa[1] = pack_bf16x2(l0, l1);
        split_bf16(pr[2 * kp + 1][0], h0, l0);
        split_bf16(pr[2 * kp + 1][1], h1, l1);
        pa[2] = pack_bf16x2(h0, h1);
        pa[3] = pack_bf16x2(l0, l1);
        const int row = rb + 16 * kp + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int cp = 0; cp < 4; ++cp) {
          const int chunk = 2 * cp + (lane >> 4);
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(vb + row * 128 + ((chunk ^ (row & 7)) << 4), b0, b1, b2, b3);
          mma_bf16_16816(o[2 * cp], pa, b0, b1);
          mma_bf16_16816(o[2 * cp + 1], pa, b2, b3);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);

    // Segment end: merge the two warps of each KV head and write out.
    const bool seg_end = (t + 1 == t_hi) || (t + 1 == prefix[s + 1]);
    if (seg_end) {
      float l_tot = l_run;
      l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 1);
      l_tot += __shfl_xor_sync(0xffffffffu, l_tot, 2);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int d = 8 * c + 2 * qd;
        my_mrg[r * 64 + d] = o[c][0] + o[c][2];
        my_mrg[r * 64 + d + 1] = o[c][1] + o[c][3];
      }
      if (qd == 0) {
        my_mrg[512 + r] = m_run;
        my_mrg[520 + r] = l_tot;
      }
      consumer_bar_sync(32 * Cfg::CWARPS);
      if (hf == 0 && row_ok) {
        const float* other = my_mrg + Cfg::MRG_FLOATS;
        const float m0 = my_mrg[512 + r], m1 = other[512 + r];
        const float M = fmaxf(m0, m1);
        const float w0 = ex2(m0 - M), w1 = ex2(m1 - M);
        const float L = my_mrg[520 + r] * w0 + other[520 + r] * w1;
        const SegDest dst = segment_dest(p, s, seg_lo, t + 1, t_lo, prefix, cta);
        const int h = g * p.group + r;
        const float inv = dst.normalise ? 1.f / L : 1.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int d = 8 * c + 2 * qd;
          float2 v;
          v.x = (my_mrg[r * 64 + d] * w0 + other[r * 64 + d] * w1) * inv;
          v.y = (my_mrg[r * 64 + d + 1] * w0 + other[r * 64 + d + 1] * w1) * inv;
          *reinterpret_cast<float2*>(dst.ptr + h * 64 + d) = v;
        }
        if (!dst.normalise && qd == 0) {
          dst.ptr[p.n_head * 64 + h] = M;
          dst.ptr[p.n_head * 64 + p.n_head + h] = L;
        }
      }
      consumer_bar_sync(32 * Cfg::CWARPS);
    }
  }
}

// ============================================================ CUDA-core path

constexpr int GEN_TILE = 32;
constexpr int GEN_THREADS = 128;
constexpr int GEN_MAX_OUT = 32;  // outputs per thread: n_head*head_dim <= 4096

struct GenLayout {
  int q_off, k_off, v_off, p_off, ml_off, wt_off, pre_off, total;
  int row_pad;
};

__host__ __device__ inline GenLayout gen_layout(int B, int n_head, int n_kv,
                                                int hd) {
  GenLayout L;
  const int kdim = n_kv * hd;
  L.row_pad = kdim + 1;
  int off = 0;
  L.q_off = off;  off += n_head * hd;
  L.k_off = off;  off += GEN_TILE * L.row_pad;
  L.v_off = off;  off += GEN_TILE * L.row_pad;
  L.p_off = off;  off += n_head * GEN_TILE;
  L.ml_off = off; off += 3 * n_head;  // m, l, alpha
  L.wt_off = off; off += 32;
  L.pre_off = off; off += B + 1;
  L.total = off * 4;
  return L;
}

size_t decode_generic_smem(int B, int n_head, int n_kv, int hd) {
  return (size_t)gen_layout(B, n_head, n_kv, hd).total;
}

template <typename Elem>
__global__ void __launch_bounds__(GEN_THREADS, 4) decode_generic_kernel(const DecodeParams p) {
  extern __shared__ float gsm[];
  const GenLayout Ly = gen_layout(p.B, p.n_head, p.n_kv, p.head_dim);
  float* q_s = gsm + Ly.q_off;
  float* k_s = gsm + Ly.k_off;
  float* v_s = gsm + Ly.v_off;
  float* p_s = gsm + Ly.p_off;
  float* m_s = gsm + Ly.ml_off;
  float* l_s = m_s + p.n_head;
  float* a_s = l_s + p.n_head;
  int* warp_tot = reinterpret_cast<int*>(gsm + Ly.wt_off);
  int* prefix = reinterpret_cast<int*>(gsm + Ly.pre_off);

  griddep_launch_dependents();
  griddep_wait();
  build_tile_prefix(p, GEN_TILE, prefix, warp_tot);
  const long long T = prefix[p.B];
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i <= p.B; i += blockDim.x) p.sched[i] = prefix[i];
  // Effective grid: never more CTAs than tiles, so no CTA range is empty.
  const int G = (int)min((long long)gridDim.x, T), cta = blockIdx.x;
  if (cta >= G) return;
  const long long t_lo = cta_tile_lo(cta, G, T), t_hi = cta_tile_lo(cta + 1, G, T);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hd = p.head_dim, kdim = p.n_kv * hd, qdim = p.n_head * hd;
  const int rp = Ly.row_pad;
  const Elem* kbase = static_cast<const Elem*>(p.k);
  const Elem* vbase = static_cast<const Elem*>(p.v);

  float acc[GEN_MAX_OUT];
  int s = 0;
  long long seg_lo = t_lo;
  for (long long t = t_lo; t < t_hi; ++t) {
    const bool new_seg = (t == seg_lo) || (t == prefix[s + 1]);
    while (prefix[s + 1] <= t) ++s;
    if (new_seg) {
      seg_lo = t;
      const float* qsrc = p.q + (size_t)s * qdim;
      if ((qdim & 3) == 0 && (reinterpret_cast<uintptr_t>(qsrc) & 15) == 0) {
        // All of this thread's 16-byte loads first, then the stores.
        constexpr int QU = 8;  // 8 x 128 x 4 floats covers n_head*head_dim <= 4096
        float4 r[QU];
#pragma unroll
        for (int u = 0; u < QU; ++u) {
          const int e = tid + u * GEN_THREADS;
          if (e < (qdim >> 2)) r[u] = reinterpret_cast<const float4*>(qsrc)[e];
        }
#pragma unroll
        for (int u = 0; u < QU; ++u) {
          const int e = tid + u * GEN_THREADS;
          if (e < (qdim >> 2)) reinterpret_cast<float4*>(q_s)[e] = r[u];
        }
      } else {
        for (int i = tid; i < qdim; i += GEN_THREADS) q_s[i] = qsrc[i];
      }
      for (int h = tid; h < p.n_head; h += GEN_THREADS) {
        m_s[h] = -INFINITY;
        l_s[h] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < GEN_MAX_OUT; ++i) acc[i] = 0.f;
    }
    const int j = (int)(t - prefix[s]);
    const int n_loc = local_rows(past_of(p, s), p.shard_start, p.max_ctx);
    const int nv = min(GEN_TILE, n_loc - j * GEN_TILE);
    const size_t row0 = (size_t)s * p.max_ctx + (size_t)j * GEN_TILE;
    // Stage the valid rows of K and V as fp32 with a padded row stride.  With
    // 16-byte aligned rows, every 16-byte load of a batch is issued before
    // any of them is used, so a tile costs one memory latency, not one per
    // loop trip.
    if (p.aligned16) {
      constexpr int VEC = 16 / sizeof(Elem);
      constexpr int UNROLL = 4;
      const int nvec = nv * kdim / VEC;
      const uint4* ksrc = reinterpret_cast<const uint4*>(kbase + row0 * kdim);
      const uint4* vsrc = reinterpret_cast<const uint4*>(vbase + row0 * kdim);
      for (int b0 = 0; b0 < nvec; b0 += GEN_THREADS * UNROLL) {
        uint4 kr[UNROLL], vr[UNROLL];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const int e = b0 + u * GEN_THREADS + tid;
          if (e < nvec) {
            kr[u] = ksrc[e];
            vr[u] = vsrc[e];
          }
        }
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const int e = b0 + u * GEN_THREADS + tid;
          if (e < nvec) {
            const int idx = e * VEC, rr = idx / kdim, cc = idx - rr * kdim;
            const Elem* ke = reinterpret_cast<const Elem*>(&kr[u]);
            const Elem* ve = reinterpret_cast<const Elem*>(&vr[u]);
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
              k_s[rr * rp + cc + i] = to_f32(ke[i]);
              v_s[rr * rp + cc + i] = to_f32(ve[i]);
            }
          }
        }
      }
    } else {
      for (int e = tid; e < nv * kdim; e += GEN_THREADS) {
        const int rr = e / kdim, cc = e - rr * kdim;
        k_s[rr * rp + cc] = to_f32(kbase[(row0 + rr) * kdim + cc]);
        v_s[rr * rp + cc] = to_f32(vbase[(row0 + rr) * kdim + cc]);
      }
    }
    __syncthreads();
    // Scores and the online-softmax update: warp w owns heads w, w+4, ...
    for (int h = warp; h < p.n_head; h += GEN_THREADS / 32) {
      const int kv = h / p.group;
      float sc = -INFINITY;
      if (lane < nv) {
        const float* qh = q_s + h * hd;
        const float* kr = k_s + lane * rp + kv * hd;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int d = 0;
        for (; d + 3 < hd; d += 4) {
          a0 = fmaf(qh[d], kr[d], a0);
          a1 = fmaf(qh[d + 1], kr[d + 1], a1);
          a2 = fmaf(qh[d + 2], kr[d + 2], a2);
          a3 = fmaf(qh[d + 3], kr[d + 3], a3);
        }
        for (; d < hd; ++d) a0 = fmaf(qh[d], kr[d], a0);
        sc = ((a0 + a1) + (a2 + a3)) * p.scale_log2;
      }
      const float mx = warp_max(sc);
      const float m_old = m_s[h];
      const float m_new = fmaxf(m_old, mx);
      const float e = ex2(sc - m_new);
      const float alpha = ex2(m_old - m_new);
      const float sum = warp_sum(e);
      p_s[h * GEN_TILE + lane] = e;
      __syncwarp();
      if (lane == 0) {
        a_s[h] = alpha;
        l_s[h] = l_s[h] * alpha + sum;
        m_s[h] = m_new;
      }
    }
    __syncthreads();
    // O = O*alpha + P.V for this thread's outputs.
#pragma unroll
    for (int i = 0; i < GEN_MAX_OUT; ++i) {
      const int idx = tid + i * GEN_THREADS;
      if (idx < qdim) {
        const int h = idx / hd, d = idx - h * hd;
        const int col = (h / p.group) * hd + d;
        float a = acc[i] * a_s[h];
        const float* ph = p_s + h * GEN_TILE;
        for (int r2 = 0; r2 < nv; ++r2) a = fmaf(ph[r2], v_s[r2 * rp + col], a);
        acc[i] = a;
      }
    }
    const bool seg_end = (t + 1 == t_hi) || (t + 1 == prefix[s + 1]);
    if (seg_end) {
      const SegDest dst = segment_dest(p, s, seg_lo, t + 1, t_lo, prefix, cta);
#pragma unroll
      for (int i = 0; i < GEN_MAX_OUT; ++i) {
        const int idx = tid + i * GEN_THREADS;
        if (idx < qdim) {
          const int h = idx / hd;
          dst.ptr[idx] = dst.normalise ? acc[i] / l_s[h] : acc[i];
        }
      }
      if (!dst.normalise)
        for (int h = tid; h < p.n_head; h += GEN_THREADS) {
          dst.ptr[qdim + h] = m_s[h];
          dst.ptr[qdim + p.n_head + h] = l_s[h];
        }
    }
    __syncthreads();
  }
}

// ========================================================== short caches

// A cluster of p.split CTAs (1, 2, 4 or 8) per (sequence, KV head) for
// caches of at most kSmallMaxRows positions and head_dim 64 (configs 1-2
// and the compatible attention_op): CTA c of the cluster attends rows
// [c n / C, (c+1) n / C) for the KV head's whole query group, and the
// cluster merges its softmax states through distributed shared memory, so
// there is no merge launch.  With p.rope the CTAs also rotate the query
// heads and the KV head's part of the new k row at the sequence's position
// (tmac_gguf.cpp:990-1016, one rounding per product and sum) and attend
// with their own copy of the new row; rank 0 writes the rotated q / k back
// and the new k / v row into the cache (:1090-1091): one launch per layer.
// Phase 1: one thread per row of the CTA's share loads the row's 64 keys
// (all loads issued together) and forms the scores of the group's heads (q
// broadcast from shared memory).  Phase 2: warp g takes head g's maximum and
// sum.  Phase 3: the 8 warps split the share's rows for P.V, lane l holding
// dimensions 2l and 2l+1 of every head.  With p.stage_v the CTA's V rows
// were copied to shared memory (cp.async) right after its K rows were
// requested, so the two memory round trips overlap; otherwise 16 rows of V
// are requested at a time in phase 3.
// Phase 4: every rank stores its state of head g into the shared memory of
// rank g % C (distributed shared memory stores: no round trip), and after one
// cluster barrier rank c merges heads c, c + C, ... from its own memory.
constexpr int SMALL_THREADS = 256;
constexpr int SMALL_WARPS = SMALL_THREADS / 32;

template <typename Elem>
__device__ __forceinline__ void load_row64(const Elem* src, bool vec, float (&kr)[64]);
template <>
__device__ __forceinline__ void load_row64<float>(const float* src, bool vec, float (&kr)[64]) {
  if (vec) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(src) + i);
      kr[4 * i] = f.x;
      kr[4 * i + 1] = f.y;
      kr[4 * i + 2] = f.z;
      kr[4 * i + 3] = f.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) kr[i] = __ldg(src + i);
  }
}
template <>
__device__ __forceinline__ void load_row64<__nv_bfloat16>(const __nv_bfloat16* src, bool vec,
                                                          float (&kr)[64]) {
  if (vec) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kr[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        kr[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 64; ++i) kr[i] = __bfloat162float(src[i]);
  }
}

template <typename Elem>
__device__ __forceinline__ float2 load_pair(const Elem* src);
template <>
__device__ __forceinline__ float2 load_pair<float>(const float* src) {
  return make_float2(__ldg(src), __ldg(src + 1));
}
template <>
__device__ __forceinline__ float2 load_pair<__nv_bfloat16>(const __nv_bfloat16* src) {
  const uint32_t w = __ldg(reinterpret_cast<const unsigned int*>(src));
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Two consecutive elements of a V row staged in shared memory, widened.
template <typename Elem>
__device__ __forceinline__ float2 smem_pair(const Elem* src);
template <>
__device__ __forceinline__ float2 smem_pair<float>(const float* src) {
  return *reinterpret_cast<const float2*>(src);
}
template <>
__device__ __forceinline__ float2 smem_pair<__nv_bfloat16>(const __nv_bfloat16* src) {
  const uint32_t w = *reinterpret_cast<const uint32_t*>(src);
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Score rows are padded to a multiple of 4 floats so that the partial
// outputs after them stay 16-byte aligned (they are stored as float2).
__host__ __device__ inline int small_row_stride(int rows) { return (rows + 3) & ~3; }
// Rows a CTA of a cluster of `split` takes at most.
__host__ __device__ inline int small_chunk_rows(int max_ctx, int split) {
  return (max_ctx + split - 1) / split;
}

// Floats of the short-cache kernel's shared memory before its V rows (a
// multiple of 4, so that the 16-byte copies of the rows land aligned).
__host__ __device__ inline size_t small_vstage_offset(int group, int max_ctx, int split) {
  const size_t f = (size_t)group * 64 +
                   (size_t)group * small_row_stride(small_chunk_rows(max_ctx, split)) +
                   SMALL_WARPS * group * 64 + 2 * group + 2 * 64 + (size_t)split * group * 66;
  return (f + 3) & ~size_t(3);
}

size_t decode_small_smem(int group, int max_ctx, int split) {
  return small_vstage_offset(group, max_ctx, split) * 4;
}

template <typename Elem>
__device__ __forceinline__ void store_elem(Elem* dst, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float* dst, float v) {
  *dst = v;
}
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* dst, float v) {
  *dst = __float2bfloat16_rn(v);
}
// The value a cache element of type Elem holds after store_elem.
template <typename Elem>
__device__ __forceinline__ float as_stored(float v);
template <>
__device__ __forceinline__ float as_stored<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float as_stored<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

template <typename Elem>
__global__ void __launch_bounds__(SMALL_THREADS) decode_small_kernel(const DecodeParams p) {
  extern __shared__ float ssm[];
  griddep_launch_dependents();
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  constexpr int HD = 64;
  const int C = p.split;                       // CTAs per (sequence, KV head)
  const int crank = (int)cluster.block_rank();
  const int item = blockIdx.x / C;
  const int G = p.group;
  const int cap = small_row_stride(small_chunk_rows(p.max_ctx, C));  // score row stride
  const int seq = item / p.n_kv, kvh = item - seq * p.n_kv;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* q_s = ssm;                           // [G][64]
  float* s_s = q_s + G * HD;                  // [G][cap] scores, then 2^(s - m)
  float* o_s = s_s + (size_t)G * cap;         // [8][G][64] per-warp partial outputs
  float* m_s = o_s + SMALL_WARPS * G * HD;    // [G] this CTA's maxima
  float* l_s = m_s + G;                       // [G] this CTA's sums
  float* kn_s = l_s + G;                      // new k row (this KV head), rope mode
  float* vn_s = kn_s + HD;                    // new v row
  float* r_m = vn_s + HD;                     // [C][G] maxima received from rank c
  float* r_l = r_m + C * G;                   // [C][G] sums received
  float* r_o = r_l + C * G;                   // [C][G][64] output sums received
  Elem* v_s = reinterpret_cast<Elem*>(ssm + small_vstage_offset(G, p.max_ctx, C));  // [rows][64]

  griddep_wait();
  // Every CTA of a cluster has the same sequence: the checks below end the
  // whole cluster or none of it.
  const int pl = past_of(p, seq);
  const bool fuse = p.rope != 0;
  if (pl < 0 || pl >= p.max_ctx || (fuse && pl >= p.table_len)) {
    if (tid == 0) record_error(p.err, kDevErrBadPos);
    return;
  }
  const int n = pl + 1;
  const int lo = (int)((long long)crank * n / C), hi = (int)((long long)(crank + 1) * n / C);
  const int nloc = hi - lo;
  const int kdim = p.n_kv * HD;
  const size_t seq_rows = (size_t)seq * p.max_ctx;
  const Elem* kb = static_cast<const Elem*>(p.k) + seq_rows * kdim + kvh * HD;
  const Elem* vb = static_cast<const Elem*>(p.v) + seq_rows * kdim + kvh * HD;
  const bool vec = p.aligned16 != 0;
  // The thread's first key row is requested before q is staged, so the two
  // loads overlap (the new row, in rope mode, comes from shared memory).
  float kr[64];
  if (tid < nloc && !(fuse && lo + tid == pl)) load_row64<Elem>(kb + (size_t)(lo + tid) * kdim, vec, kr);
  if (p.stage_v) {
    // The V rows of this CTA's share, 16 bytes per copy (the new row in
    // rope mode comes from shared memory instead).
    constexpr int CH = HD * (int)sizeof(Elem) / 16;
    constexpr int EPC = 16 / (int)sizeof(Elem);
    for (int i = tid; i < nloc * CH; i += SMALL_THREADS) {
      const int t = i / CH, c = i - t * CH;
      if (fuse && lo + t == pl) continue;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                       smem_u32(v_s + (size_t)t * HD + c * EPC)),
                   "l"(vb + (size_t)(lo + t) * kdim + c * EPC)
                   : "memory");
    }
  }
  const size_t qoff = (size_t)seq * p.n_head * HD + (size_t)kvh * G * HD;
  const size_t koff = (size_t)seq * kdim + kvh * HD;
  if (!fuse) {
    const float* qsrc = p.q + qoff;
    for (int i = tid; i < G * HD; i += SMALL_THREADS) q_s[i] = qsrc[i];
  } else {
    // RoPE of the group's query heads and of this KV head's part of the new
    // k row: pairs (2j, 2j+1), x0*c - x1*s and x0*s + x1*c.  Every CTA of
    // the cluster rotates for itself; rank 0 writes the results back after
    // the cluster barrier, when no CTA reads the raw values any more.
    const float* cs = p.cs + (size_t)pl * HD;
    for (int i = tid; i < (G + 1) * (HD / 2); i += SMALL_THREADS) {
      const int g = i / (HD / 2), j = i - g * (HD / 2);
      const float* src = g < G ? p.q_io + qoff + g * HD + 2 * j : p.k_io + koff + 2 * j;
      const float2 x = *reinterpret_cast<const float2*>(src);
      const float2 c = *reinterpret_cast<const float2*>(cs + 2 * j);
      const float y0 = __fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y));
      const float y1 = __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x));
      float* dst = g < G ? q_s + g * HD + 2 * j : kn_s + 2 * j;
      dst[0] = y0;
      dst[1] = y1;
    }
    for (int i = tid; i < HD; i += SMALL_THREADS) vn_s[i] = p.v_new[koff + i];
  }
  __syncthreads();
  // The new row as the cache stores it (rounded to the cache type).
  const auto new_k = [&](int d) { return as_stored<Elem>(kn_s[d]); };
  if (fuse && tid < nloc && lo + tid == pl) {
#pragma unroll
    for (int d = 0; d < HD; ++d) kr[d] = new_k(d);
  }

  // 1. Scores of this CTA's rows, one thread per row.
  for (int t = tid; t < nloc; t += SMALL_THREADS) {
    const int r = lo + t;
    if (t != tid) {
      if (fuse && r == pl) {
#pragma unroll
        for (int d = 0; d < HD; ++d) kr[d] = new_k(d);
      } else {
        load_row64<Elem>(kb + (size_t)r * kdim, vec, kr);
      }
    }
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      if (g < G) {
        const float* qg = q_s + g * HD;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int d = 0; d < HD; d += 4) {
          const float4 q4 = *reinterpret_cast<const float4*>(qg + d);
          a0 = fmaf(q4.x, kr[d], a0);
          a1 = fmaf(q4.y, kr[d + 1], a1);
          a2 = fmaf(q4.z, kr[d + 2], a2);
          a3 = fmaf(q4.w, kr[d + 3], a3);
        }
        s_s[(size_t)g * cap + t] = ((a0 + a1) + (a2 + a3)) * p.scale_log2;
      }
    }
  }
  __syncthreads();
  // 2. This CTA's softmax state of head g on warp g: maximum and sum.
  if (warp < G) {
    float* sg = s_s + (size_t)warp * cap;
    float mx = -INFINITY;
    for (int t = lane; t < nloc; t += 32) mx = fmaxf(mx, sg[t]);
    mx = warp_max(mx);
    float sum = 0.f;
    for (int t = lane; t < nloc; t += 32) {
      const float e = ex2(sg[t] - mx);
      sg[t] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    if (lane == 0) {
      m_s[warp] = mx;
      l_s[warp] = sum;
    }
  }
  if (p.stage_v) asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  // 3. P.V over this warp's share of the CTA's rows, every head of the group.
  float acc[8][2];
#pragma unroll
  for (int g = 0; g < 8; ++g) acc[g][0] = acc[g][1] = 0.f;
  const int t0 = (warp * nloc) / SMALL_WARPS, t1 = ((warp + 1) * nloc) / SMALL_WARPS;
  const Elem* vcol = vb + 2 * lane;
  const float2 vnew = make_float2(as_stored<Elem>(vn_s[2 * lane]), as_stored<Elem>(vn_s[2 * lane + 1]));
  int t = t0;
  // 16 rows of V requested at a time: one memory latency per 16 rows.
  for (; t + 15 < t1; t += 16) {
    float2 v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u)
      v[u] = (fuse && lo + t + u == pl) ? vnew
             : p.stage_v ? smem_pair<Elem>(v_s + (size_t)(t + u) * HD + 2 * lane)
                         : load_pair<Elem>(vcol + (size_t)(lo + t + u) * kdim);
#pragma unroll
    for (int u = 0; u < 16; ++u)
#pragma unroll
      for (int g = 0; g < 8; ++g)
        if (g < G) {
          const float pr = s_s[(size_t)g * cap + t + u];
          acc[g][0] = fmaf(pr, v[u].x, acc[g][0]);
          acc[g][1] = fmaf(pr, v[u].y, acc[g][1]);
        }
  }
  for (; t < t1; ++t) {
    const float2 v = (fuse && lo + t == pl) ? vnew
                     : p.stage_v ? smem_pair<Elem>(v_s + (size_t)t * HD + 2 * lane)
                                 : load_pair<Elem>(vcol + (size_t)(lo + t) * kdim);
#pragma unroll
    for (int g = 0; g < 8; ++g)
      if (g < G) {
        const float pr = s_s[(size_t)g * cap + t];
        acc[g][0] = fmaf(pr, v.x, acc[g][0]);
        acc[g][1] = fmaf(pr, v.y, acc[g][1]);
      }
  }
#pragma unroll
  for (int g = 0; g < 8; ++g)
    if (g < G)
      *reinterpret_cast<float2*>(o_s + (warp * G + g) * HD + 2 * lane) =
          make_float2(acc[g][0], acc[g][1]);
  __syncthreads();
  // 4. Merge the cluster's states: rank c finishes heads c, c + C, ....
  //    This CTA's (m, l, o) of head g go to rank g % C's receive buffers
  //    (slot crank); the cluster barrier makes them visible there.
  for (int i = tid; i < G * HD; i += SMALL_THREADS) {
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < SMALL_WARPS; ++w) o += o_s[w * G * HD + i];
    const int g = i / HD, owner = g % C;
    (owner == crank ? r_o : cluster.map_shared_rank(r_o, owner))[(crank * G + g) * HD + i - g * HD] = o;
  }
  if (tid < G) {
    const int owner = tid % C;
    (owner == crank ? r_m : cluster.map_shared_rank(r_m, owner))[crank * G + tid] = m_s[tid];
    (owner == crank ? r_l : cluster.map_shared_rank(r_l, owner))[crank * G + tid] = l_s[tid];
  }
  // No CTA touches another's shared memory after this barrier.
  cluster.sync();
  float* out = p.out + qoff;
  for (int g = crank; g < G; g += C) {
    for (int d = tid; d < HD; d += SMALL_THREADS) {
      float M = -INFINITY;
      for (int c = 0; c < C; ++c) M = fmaxf(M, r_m[c * G + g]);
      float L = 0.f, O = 0.f;
      for (int c = 0; c < C; ++c) {
        const float w = ex2(r_m[c * G + g] - M);
        L = fmaf(w, r_l[c * G + g], L);
        O = fmaf(w, r_o[(c * G + g) * HD + d], O);
      }
      out[g * HD + d] = O / L;
    }
  }
  // 5. Rank 0 writes the rotated q / k back and the new row into the cache.
  if (fuse && crank == 0) {
    float* qw = p.q_wb ? p.q_wb : p.q_io;
    float* kw = p.k_wb ? p.k_wb : p.k_io;
    for (int i = tid; i < G * HD; i += SMALL_THREADS) qw[qoff + i] = q_s[i];
    const size_t crow = (seq_rows + pl) * kdim + kvh * HD;
    for (int i = tid; i < HD; i += SMALL_THREADS) {
      kw[koff + i] = kn_s[i];
      store_elem<Elem>(static_cast<Elem*>(p.k_cache) + crow + i, kn_s[i]);
      store_elem<Elem>(static_cast<Elem*>(p.v_cache) + crow + i, vn_s[i]);
    }
  }
}

// ================================================================== merges

// One CTA per (sequence, head); thread d owns output dimension d.  The
// partial records of a split sequence are folded with a single-pass online
// combine; slot values are loaded in batches of 8 so the loads overlap.
constexpr int MERGE_BATCH = 8;

__global__ void __launch_bounds__(128) merge_kernel(const MergeParams p) {
  griddep_launch_dependents();
  griddep_wait();
  const int s = blockIdx.x / p.n_head, h = blockIdx.x - s * p.n_head;
  const int t0 = p.sched[s], t1 = p.sched[s + 1];
  const long long T = p.sched[p.B];
  const int hd = p.head_dim, qdim = p.n_head * hd;
  const int rf = record_floats(p.n_head, hd);
  if (t1 == t0) {
    if (p.mode == 1) {
      float* rec = p.records + (size_t)s * rf;
      for (int d = threadIdx.x; d < hd; d += blockDim.x) rec[h * hd + d] = 0.f;
      if (threadIdx.x == 0) {
        rec[qdim + h] = kNegBig;
        rec[qdim + p.n_head + h] = 0.f;
      }
    }
    return;
  }
  const int G = (int)min((long long)p.G, T);  // the decode kernel's effective grid
  const int c1 = cta_of_tile(t0, G, T), c2 = cta_of_tile(t1 - 1, G, T);
  if (c1 == c2) return;
  const int first_slot = 2 * c1 + (cta_tile_lo(c1, G, T) == t0 ? 0 : 1);
  const int n_parts = 1 + (c2 - c1);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float M = kNegBig, O = 0.f, L = 0.f;
    for (int k0 = 0; k0 < n_parts; k0 += MERGE_BATCH) {
      float mv[MERGE_BATCH], lv[MERGE_BATCH], ov[MERGE_BATCH];
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) {
        const int k = k0 + u;
        mv[u] = kNegBig;
        lv[u] = 0.f;
        ov[u] = 0.f;
        if (k < n_parts) {
          const float* rec = p.part + (size_t)(k == 0 ? first_slot : 2 * (c1 + k)) * rf;
          mv[u] = rec[qdim + h];
          lv[u] = rec[qdim + p.n_head + h];
          ov[u] = rec[h * hd + d];
        }
      }
      float Mb = M;
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) Mb = fmaxf(Mb, mv[u]);
      const float a = ex2(M - Mb);
      O *= a;
      L *= a;
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) {
        const float w = ex2(mv[u] - Mb);
        O = fmaf(ov[u], w, O);
        L = fmaf(lv[u], w, L);
      }
      M = Mb;
    }
    if (p.mode == 0) {
      p.out[(size_t)s * qdim + h * hd + d] = O / L;
    } else {
      float* rec = p.records + (size_t)s * rf;
      rec[h * hd + d] = O;
      if (d == 0) {
        rec[qdim + h] = M;
        rec[qdim + p.n_head + h] = L;
      }
    }
  }
}

__global__ void __launch_bounds__(128) gather_merge_kernel(const GatherMergeParams p) {
  griddep_launch_dependents();
  griddep_wait();
  const int s = blockIdx.x / p.n_head, h = blockIdx.x - s * p.n_head;
  const int hd = p.head_dim, qdim = p.n_head * hd;
  const int rf = record_floats(p.n_head, hd);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float M = kNegBig, O = 0.f, L = 0.f;
    for (int r0 = 0; r0 < p.world; r0 += MERGE_BATCH) {
      float mv[MERGE_BATCH], lv[MERGE_BATCH], ov[MERGE_BATCH];
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) {
        const int r = r0 + u;
        mv[u] = kNegBig;
        lv[u] = 0.f;
        ov[u] = 0.f;
        if (r < p.world) {
          const float* rec = p.records + ((size_t)r * p.B + s) * rf;
          mv[u] = rec[qdim + h];
          lv[u] = rec[qdim + p.n_head + h];
          ov[u] = rec[h * hd + d];
        }
      }
      float Mb = M;
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) Mb = fmaxf(Mb, mv[u]);
      const float a = ex2(M - Mb);
      O *= a;
      L *= a;
#pragma unroll
      for (int u = 0; u < MERGE_BATCH; ++u) {
        const float w = ex2(mv[u] - Mb);
        O = fmaf(ov[u], w, O);
        L = fmaf(lv[u], w, L);
      }
      M = Mb;
    }
    p.out[(size_t)s * qdim + h * hd + d] = O / L;
  }
}

// ============================================================ elementwise

// elem_op (kernel_elem.metal:6-21): op 0 data += aux, op 2 data = aux.
__global__ void elem_kernel(int op, float* data, const float* aux, int dim) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= dim) return;
  if (op == 0)
    data[i] = __fadd_rn(data[i], aux[i]);
  else
    data[i] = aux[i];
}

// Synthetic N(0,1) values: the splitmix64 + Box-Muller stream of the oracle
// (draw k is splitmix64 of seed + (k+1)*gamma), evaluated with the device's
// double-precision libm and rounded to the cache type.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(void* out, size_t n, int dtype, uint64_t seed) {
  const uint64_t gamma = 0x9E3779B97F4A7C15ULL;
  const size_t pairs = (n + 1) / 2;
  for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < pairs;
       k += (size_t)gridDim.x * blockDim.x) {
    const uint64_t a = mix64(seed + (2 * k + 1) * gamma);
    const uint64_t b = mix64(seed + (2 * k + 2) * gamma);
    const double u1 = ((double)(a >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
    const double rr = sqrt(-2.0 * log(u1));
    const double ang = 6.283185307179586476925286766559 * u2;
    const float z0 = (float)(rr * cos(ang)), z1 = (float)(rr * sin(ang));
    const size_t i0 = 2 * k;
    if (dtype == 0) {
      float* o = static_cast<float*>(out);
      o[i0] = z0;
      if (i0 + 1 < n) o[i0 + 1] = z1;
    } else {
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
      o[i0] = __float2bfloat16_rn(z0);
      if (i0 + 1 < n) o[i0 + 1] = __float2bfloat16_rn(z1);
    }
  }
}

// f32 -> cache type (RNE for bf16), used to upload rows.
__global__ void convert_rows_kernel(void* dst, const float* src, size_t n, int dtype) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    if (dtype == 0)
      static_cast<float*>(dst)[i] = src[i];
    else
      static_cast<__nv_bfloat16*>(dst)[i] = __float2bfloat16_rn(src[i]);
  }
}

// ================================================================ launchers

// Launch with programmatic stream serialization: the kernel may be
// launched while its predecessor on the stream is still running; every
// kernel here waits (griddepcontrol.wait) before touching memory, so the
// overlap only hides launch latency.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, std::forward<Args>(args)...);
}

cudaError_t launch_rope(const RopeParams& p, cudaStream_t st) {
  if (p.B <= 0) return cudaSuccess;
  return launch_pdl(rope_cache_write_kernel, dim3(p.B), dim3(128), 0, st, p);
}

// Dynamic shared-memory limits set on the CUDA-core decode kernel, per device.
static size_t g_generic_cfg_f32[64] = {}, g_generic_cfg_bf16[64] = {};

// Raises a kernel's dynamic shared-memory limit once per device and size
// (never lowers it); callers on several threads share the caches.
static std::mutex g_attr_mu;
template <typename F>
static cudaError_t ensure_smem(F* fn, size_t smem, size_t* cache) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  if (smem <= cache[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) cache[dev] = smem;
  return e;
}

// Dynamic shared-memory limits set on decode_mma_kernel<NKV>, per device.
template <int NKV>
static size_t* mma_configured() {
  static size_t configured[64] = {};
  return configured;
}

template <int NKV>
static cudaError_t launch_mma_nkv(const CUtensorMap& tk, const CUtensorMap& tv,
                                  const DecodeParams& p, int grid,
                                  cudaStream_t st) {
  const size_t smem = MmaCfg<NKV>::smem_bytes(p.B);
  cudaError_t e = ensure_smem(decode_mma_kernel<NKV>, smem, mma_configured<NKV>());
  if (e != cudaSuccess) return e;
  return launch_pdl(decode_mma_kernel<NKV>, dim3(grid), dim3(MmaCfg<NKV>::THREADS), smem, st,
                    tk, tv, p);
}

size_t decode_mma_smem(int nkv, int B) {
  switch (nkv) {
    case 1: return MmaCfg<1>::smem_bytes(B);
    case 2: return MmaCfg<2>::smem_bytes(B);
    case 4: return MmaCfg<4>::smem_bytes(B);
    default: return 0;
  }
}

// One warp per CTA (so that CTAs fit beside a decode CTA, whose registers
// leave room for single warps only), 4 x 16 bytes in flight per thread.
// The copies run before the grid-dependency wait: the source is this call's
// page-locked staging, written by the host before the launch, and the
// destinations are slots no earlier kernel uses.  The next kernel is let
// launch only after the copies are stored and fenced, because kernels read
// some inputs (positions, projection weights) before their own
// grid-dependency wait.  The wait comes last so that the next kernel's wait
// on this one also covers the previous kernel.
__global__ void __launch_bounds__(32) stage_copy_kernel(const StageParams p) {
  const int stride = gridDim.x * 32;
  for (int r = 0; r < p.n_runs; ++r) {
    const StageRun c = p.run[r];
    for (int i0 = blockIdx.x * 32 + threadIdx.x; i0 < c.n16; i0 += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * stride;
        if (i < c.n16) v[u] = c.src[i];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * stride;
        if (i < c.n16) c.dst[i] = v[u];
      }
    }
  }
  __threadfence();
  griddep_launch_dependents();
  griddep_wait();
}

// The outputs a batch's kernels left in device slots go to their
// page-locked host buffers in one launch at the end of the batch, so that
// no kernel inside the batch writes host memory (a kernel that does ends
// only once its writes have crossed the host link, and the next kernel's
// grid-dependency wait waits for that).  The entry list is host-written
// before the launch, so it is read before the wait; the copies come after
// it.  16-byte words when both ends and the size allow, else 4-byte words,
// else bytes.
__global__ void __launch_bounds__(256) store_out_kernel(const StoreEntry* list, int n) {
  griddep_launch_dependents();
  StoreEntry e{};
  if ((int)blockIdx.x < n) e = list[blockIdx.x];
  griddep_wait();
  for (int i0 = blockIdx.x; i0 < n; i0 += gridDim.x) {
    if (i0 != (int)blockIdx.x) e = list[i0];
    const uintptr_t a = reinterpret_cast<uintptr_t>(e.dst) | reinterpret_cast<uintptr_t>(e.src);
    if (((a | e.bytes) & 15) == 0) {
      const uint4* s = static_cast<const uint4*>(e.src);
      uint4* d = static_cast<uint4*>(e.dst);
      for (size_t i = threadIdx.x; i < e.bytes / 16; i += blockDim.x) d[i] = __ldcg(s + i);
    } else if (((a | e.bytes) & 3) == 0) {
      const unsigned* s = static_cast<const unsigned*>(e.src);
      unsigned* d = static_cast<unsigned*>(e.dst);
      for (size_t i = threadIdx.x; i < e.bytes / 4; i += blockDim.x) d[i] = __ldcg(s + i);
    } else {
      const unsigned char* s = static_cast<const unsigned char*>(e.src);
      unsigned char* d = static_cast<unsigned char*>(e.dst);
      for (size_t i = threadIdx.x; i < e.bytes; i += blockDim.x) d[i] = s[i];
    }
  }
}

cudaError_t launch_store_out(const StoreEntry* list, int n, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  return launch_pdl(store_out_kernel, dim3((unsigned)(n < 1024 ? n : 1024)), dim3(256), 0, st,
                    list, n);
}

cudaError_t launch_stage_copy(const StageParams& p, int total16, cudaStream_t st) {
  int grid = (total16 + 4 * 32 - 1) / (4 * 32);
  if (grid < 1) grid = 1;
  if (grid > 64) grid = 64;
  return launch_pdl(stage_copy_kernel, dim3(grid), dim3(32), 0, st, p);
}

cudaError_t prepare_decode_kernels(int max_seqs) {
  const size_t cap = 227 * 1024;
  auto lim = [&](size_t x) { return x < cap ? x : cap; };
  cudaError_t e = ensure_smem(decode_mma_kernel<1>, lim(MmaCfg<1>::smem_bytes(max_seqs)),
                              mma_configured<1>());
  if (e == cudaSuccess)
    e = ensure_smem(decode_mma_kernel<2>, lim(MmaCfg<2>::smem_bytes(max_seqs)),
                    mma_configured<2>());
  if (e == cudaSuccess)
    e = ensure_smem(decode_mma_kernel<4>, lim(MmaCfg<4>::smem_bytes(max_seqs)),
                    mma_configured<4>());
  if (e == cudaSuccess) e = ensure_smem(decode_generic_kernel<float>, cap, g_generic_cfg_f32);
  if (e == cudaSuccess)
    e = ensure_smem(decode_generic_kernel<__nv_bfloat16>, cap, g_generic_cfg_bf16);
  return e;
}

cudaError_t launch_decode_mma(const CUtensorMap& tk, const CUtensorMap& tv,
                              const DecodeParams& p, int grid, cudaStream_t st) {
  switch (p.n_kv) {
    case 1: return launch_mma_nkv<1>(tk, tv, p, grid, st);
    case 2: return launch_mma_nkv<2>(tk, tv, p, grid, st);
    case 4: return launch_mma_nkv<4>(tk, tv, p, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

// V rows staged in shared memory when the caches are 16-byte aligned and a
// CTA's share takes at most this many bytes (two CTAs per SM stay resident).
constexpr size_t kSmallVStageMax = 32 * 1024;

cudaError_t launch_decode_small(const DecodeParams& p_in, int dtype, cudaStream_t st) {
  if (p_in.B <= 0) return cudaSuccess;
  DecodeParams p = p_in;
  const size_t vbytes = (size_t)small_chunk_rows(p.max_ctx, p.split) * 64 * (dtype == 0 ? 4 : 2);
  p.stage_v = (p.aligned16 && vbytes <= kSmallVStageMax) ? 1 : 0;
  const size_t smem = decode_small_smem(p.group, p.max_ctx, p.split) + (p.stage_v ? vbytes : 0);
  static size_t configured_f32[64] = {}, configured_bf16[64] = {};
  void (*fn)(const DecodeParams) =
      dtype == 0 ? decode_small_kernel<float> : decode_small_kernel<__nv_bfloat16>;
  cudaError_t e = dtype == 0 ? ensure_smem(decode_small_kernel<float>, smem, configured_f32)
                             : ensure_smem(decode_small_kernel<__nv_bfloat16>, smem, configured_bf16);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.B * p.n_kv * p.split));
  cfg.blockDim = dim3(SMALL_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)p.split;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

cudaError_t launch_decode_generic(const DecodeParams& p, int dtype, int grid,
                                  cudaStream_t st) {
  size_t* configured_f32 = g_generic_cfg_f32;
  size_t* configured_bf16 = g_generic_cfg_bf16;
  const size_t smem = decode_generic_smem(p.B, p.n_head, p.n_kv, p.head_dim);
  cudaError_t e;
  if (dtype == 0) {
    e = ensure_smem(decode_generic_kernel<float>, smem, configured_f32);
    if (e != cudaSuccess) return e;
    return launch_pdl(decode_generic_kernel<float>, dim3(grid), dim3(GEN_THREADS), smem, st, p);
  } else {
    e = ensure_smem(decode_generic_kernel<__nv_bfloat16>, smem, configured_bf16);
    if (e != cudaSuccess) return e;
    return launch_pdl(decode_generic_kernel<__nv_bfloat16>, dim3(grid), dim3(GEN_THREADS), smem,
                      st, p);
  }
}

int decode_generic_blocks_per_sm(int dtype, size_t smem) {
  // Resident CTAs per SM for a dynamic shared-memory size, cached per device
  // and dtype; the limit is raised through the launcher's cache so that a
  // query never lowers what a launch relies on.
  static std::mutex mu;
  static size_t last_smem[64][2] = {};
  static int last_n[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 1;
  }
  const int di = dtype == 0 ? 0 : 1;
  std::lock_guard<std::mutex> lock(mu);
  if (last_n[dev][di] && last_smem[dev][di] == smem) return last_n[dev][di];
  int n = 0;
  if (dtype == 0) {
    if (ensure_smem(decode_generic_kernel<float>, smem, g_generic_cfg_f32) == cudaSuccess)
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_generic_kernel<float>,
                                                    GEN_THREADS, smem);
  } else {
    if (ensure_smem(decode_generic_kernel<__nv_bfloat16>, smem, g_generic_cfg_bf16) ==
        cudaSuccess)
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_generic_kernel<__nv_bfloat16>,
                                                    GEN_THREADS, smem);
  }
  cudaGetLastError();
  n = n < 1 ? 1 : n;
  last_smem[dev][di] = smem;
  last_n[dev][di] = n;
  return n;
}

cudaError_t launch_merge(const MergeParams& p, cudaStream_t st) {
  if (p.B <= 0) return cudaSuccess;
  const int threads = p.head_dim <= 64 ? 64 : 128;
  return launch_pdl(merge_kernel, dim3(p.B * p.n_head), dim3(threads), 0, st, p);
}

cudaError_t launch_gather_merge(const GatherMergeParams& p, cudaStream_t st) {
  if (p.B <= 0) return cudaSuccess;
  const int threads = p.head_dim <= 64 ? 64 : 128;
  return launch_pdl(gather_merge_kernel, dim3(p.B * p.n_head), dim3(threads), 0, st, p);
}

cudaError_t launch_elem(int op, float* data, const float* aux, int dim,
                        cudaStream_t st) {
  if (dim <= 0) return cudaSuccess;
  elem_kernel<<<(dim + 255) / 256, 256, 0, st>>>(op, data, aux, dim);
  return cudaGetLastError();
}

cudaError_t launch_fill_normal(void* out, size_t n, int dtype, uint64_t seed,
                               int num_sms, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  fill_normal_kernel<<<num_sms * 8, 256, 0, st>>>(out, n, dtype, seed);
  return cudaGetLastError();
}

cudaError_t launch_convert_rows(void* dst, const float* src, size_t n, int dtype,
                                int num_sms, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  convert_rows_kernel<<<num_sms * 4, 256, 0, st>>>(dst, src, n, dtype);
  return cudaGetLastError();
}

int mma_threads(int nkv) { return 32 * (2 * nkv + 1); }

}  // namespace tg
