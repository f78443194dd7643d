// tg_decode_fused.cu -- the decode step of one layer over a bf16 cache in two
// PDL-chained launches: RoPE of q and k (tmac_gguf.cpp:990-1016), the
// cache-write of the new row (tmac_gguf.cpp:1090-1091) and GQA attention
// (tmac_gguf.cpp:1093-1128) in the decode kernel; the split-KV merge, the
// write-back of the rotated q / k and -- across the GPUs of one box -- the
// exchange of per-GPU softmax records over peer memory in the merge kernel.
//
// Decode kernel (same tile schedule and tensor-core inner loop as
// decode_mma_kernel in tg_kernels.cu):
//  * consumers rotate q on the fly from the raw q and the host-libm cos/sin
//    table when a sequence starts (bit-identical to the RoPE kernel);
//  * the warp whose rows hold a sequence's new position overwrites that row
//    of the TMA-staged K and V tile with the rotated k and the new v (bf16,
//    RNE) and stores it to the cache, so no separate cache-write launch and
//    no ordering between a writer kernel and the TMA loads is needed;
//  * a sequence that lies within one CTA is finished there (output, or its
//    record for the exchange); the pieces of a split sequence go to the
//    CTA's two partial-record slots;
//  * before its grid-dependency wait: the schedule, the TMA descriptors, an
//    optional L2 prefetch and (tuning, off by default) the first ring stages.
// Merge kernel: one item per (sequence, head), spread over many SMs so the
// tail of the step is short; in mode 2 (split-KV across GPUs) it stores its
// record slice into every GPU's receive words over NVLink, each 4-byte value
// packed with the launch's epoch tag into one 8-byte store, so receivers poll
// the data itself (bounded) and need no fence or flag; then it merges.
// Receive words alternate between launches (epoch parity) because a GPU can
// be at most one launch ahead of the others.
//
// Every wait is bounded (mbarriers, peer words); on expiry the error word is
// set and the kernel still reaches its end.  With stamps on, every CTA of
// both kernels records %globaltimer values (FusedParams::stamps).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "tg_device.cuh"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace tg {

template <int NKV, int RING_KB>
struct FusedCfg {
  static constexpr int TILE = 64;
  // RING_KB of K/V per CTA: 128 covers loaded HBM latency (a pure TMA stream
  // of this tiling reaches the copy peak with it); 192 lets a small shard
  // load more of its tiles before the grid-dependency wait.
  static constexpr int STAGES = (RING_KB * 1024) / (2 * NKV * TILE * 128);
  // Consumer warps per KV head: each takes RW rows of every tile.  Four (16
  // rows) give every SM sub-partition two or more warps to interleave; with
  // four KV heads, two (32 rows) keep the CTA within the register file.
  static constexpr int WPH = NKV >= 4 ? 2 : 4;
  static constexpr int RW = TILE / WPH;
  static constexpr int NT = RW / 8;   // n-tiles of 8 rows in S = q K^T
  static constexpr int KP = RW / 16;  // k-steps of 16 rows in O += P V
  static constexpr int CWARPS = WPH * NKV;
  static constexpr int CTHREADS = 32 * CWARPS;
  static constexpr int THREADS = CTHREADS + 32;
  static constexpr int BOX = TILE * 128;
  static constexpr int STAGE_BYTES = 2 * NKV * BOX;
  static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
  static constexpr int MRG_FLOATS = 8 * 64 + 16;
  static constexpr int OFF_MRG = OFF_BAR + 2 * STAGES * 8;
  static constexpr int OFF_WTOT = OFF_MRG + CWARPS * MRG_FLOATS * 4;
  static constexpr int OFF_PREFIX = OFF_WTOT + 32 * 4;
  static constexpr size_t smem_bytes(int B) { return 1024 + (size_t)OFF_PREFIX + (size_t)(B + 1) * 4; }
};

// Iteration cap of every poll loop; the time bound is FusedParams::wait_ns.
constexpr long long kPollCap = 1LL << 28;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void cons_sync(int n) {
  asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory");
}

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// x0*c - x1*s, x0*s + x1*c with one rounding per product and sum
// (tmac_gguf.cpp:999-1000 without contraction).
__device__ __forceinline__ float2 rot(float2 x, float2 c) {
  return make_float2(__fsub_rn(__fmul_rn(x.x, c.x), __fmul_rn(x.y, c.y)),
                     __fadd_rn(__fmul_rn(x.x, c.y), __fmul_rn(x.y, c.x)));
}

// Tiles of one sequence on this shard; 0 for a position outside the cache /
// RoPE table (the decode kernel reports it).
__device__ __forceinline__ int seq_tiles(const FusedParams& p, int pl) {
  if (pl < 0 || pl >= p.table_len || (p.mode == 0 && pl >= p.shard_start + p.max_ctx)) return -1;
  return (local_rows(pl, p.shard_start, p.max_ctx) + 63) / 64;
}

// Tile prefix over sequences, as build_tile_prefix in tg_kernels.cu.  Reads
// only the positions, so it may run before the grid-dependency wait: the
// only kernel of this library that writes positions is the staging copy of
// host inputs, which stores and fences them before it lets the next kernel
// launch.  The reads go to L2 (no stale L1 line of a reused staging slot).
__device__ void fused_prefix(const FusedParams& p, int* prefix, int* warp_tot) {
  const int NT = blockDim.x, t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int chunk = (p.B + NT - 1) / NT;
  const int b0 = min(t * chunk, p.B), b1 = min(b0 + chunk, p.B);
  int sum = 0;
  for (int s = b0; s < b1; ++s) {
    int tiles = seq_tiles(p, __ldcg(p.pos + s));
    if (tiles < 0) {
      record_error(p.err, kDevErrBadPos);
      tiles = 0;
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

template <int NKV, int RING_KB>
__global__ void __launch_bounds__(FusedCfg<NKV, RING_KB>::THREADS, 1)
    decode_fused_kernel(const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, const FusedParams p) {
  using Cfg = FusedCfg<NKV, RING_KB>;
  constexpr int TILE = Cfg::TILE, STAGES = Cfg::STAGES, NCT = Cfg::CTHREADS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* empty = full + STAGES;
  float* mrg = reinterpret_cast<float*>(smem + Cfg::OFF_MRG);
  int* warp_tot = reinterpret_cast<int*>(smem + Cfg::OFF_WTOT);
  int* prefix = reinterpret_cast<int*>(smem + Cfg::OFF_PREFIX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qdim = p.n_head * 64;
  const int rf = record_floats(p.n_head, 64);
  unsigned long long* stamp = p.stamps ? p.stamps + (size_t)blockIdx.x * kStampsPerCta : nullptr;

  griddep_launch_dependents();
  if (stamp && threadIdx.x == 0) stamp[0] = global_ns();
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], Cfg::CWARPS);
    }
    fence_mbar_init();
  }
  // Before the wait for the previous kernel: the schedule (positions only;
  // its barriers also publish the mbarrier initialisation), the TMA
  // descriptors, the first ring stages when the host allows it (p.preload),
  // and an L2 prefetch of the following tiles (p.prefetch: when the host
  // expects the wait to be long).  A prefetch never returns stale data (the
  // loads after the wait read through L2).
  fused_prefix(p, prefix, warp_tot);
  const long long T = prefix[p.B];
  const int G = (int)min((long long)gridDim.x, T), cta = blockIdx.x;
  const bool active = cta < G;
  long long t_lo = 0, t_hi = 0;
  if (active) {
    t_lo = cta_tile_lo(cta, G, T);
    t_hi = cta_tile_lo(cta + 1, G, T);
  }
  // Producer state, carried from the pre-wait loads into the main loop.
  int pt = (int)t_lo, ps = 0, pst = 0, pissued = 0;
  uint32_t pph = 0;
  bool pok = true;
  const bool producer = active && warp == Cfg::CWARPS && lane == 0;
  // Issues the loads of tiles [pt, t_stop); with `guard`, stops before the
  // first tile holding a sequence's new-token row (a row the previous
  // kernel may write).  TMA row of tile t: row0 + s*max_ctx +
  // (t - prefix[s])*TILE (< 2^31, checked when the cache is created).
  auto produce = [&](int t_stop, bool guard) {
    while (pt < t_stop && pok) {
      while (prefix[ps + 1] <= pt) ++ps;
      const int j = pt - prefix[ps];
      if (guard) {
        const int local_new = __ldcg(p.pos + ps) - p.shard_start;
        if (local_new >= j * TILE && local_new < (j + 1) * TILE) break;
      }
      if (!mbar_wait(&empty[pst], pph ^ 1u, p.err, kDevErrWaitEmpty)) {
        pok = false;
        break;
      }
      uint8_t* stage = smem + pst * Cfg::STAGE_BYTES;
      mbar_arrive_expect_tx(&full[pst], Cfg::STAGE_BYTES);
      const int y = (int)(p.row0 + (long long)ps * p.max_ctx) + j * TILE;
#pragma unroll
      for (int g = 0; g < NKV; ++g) {
        tma_load_2d(stage + g * Cfg::BOX, &tmk, &full[pst], 64 * g, y);
        tma_load_2d(stage + (NKV + g) * Cfg::BOX, &tmv, &full[pst], 64 * g, y);
      }
      ++pissued;
      ++pt;
      if (++pst == STAGES) {
        pst = 0;
        pph ^= 1u;
      }
    }
  };
  if (producer) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmv);
    if (p.preload) produce((int)min(t_hi, t_lo + STAGES), !p.new_row);
    if (p.prefetch) {
      int s = ps;
      const int t_pf = (int)min(t_hi, (long long)pt + STAGES);
      for (int t = pt; t < t_pf; ++t) {
        while (prefix[s + 1] <= t) ++s;
        const int y = (int)(p.row0 + (long long)s * p.max_ctx) + (t - prefix[s]) * TILE;
#pragma unroll
        for (int g = 0; g < NKV; ++g) {
          tma_prefetch_l2_2d(&tmk, 64 * g, y);
          tma_prefetch_l2_2d(&tmv, 64 * g, y);
        }
      }
    }
  }
  griddep_wait();
  if (stamp && threadIdx.x == 0) stamp[1] = global_ns();
  // The previous launch's merge kernel has finished: it read the schedule
  // buffer and, in mode 2, the decode-done count of the other parity, which
  // block 0 clears here for the next launch.
  // The previous launch's merge kernel has finished: it read the schedule
  // buffer and, in mode 2, the exchange epoch, which advances here once per
  // launch (the merge kernel of this launch reads it after its own wait).
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i <= p.B; i += blockDim.x) p.sched[i] = prefix[i];
    if (p.mode == 2 && threadIdx.x == 0) *p.epoch += 1u;
  }
  __syncthreads();

  if (producer) {
    // ------------------------------------------------------------ producer
    produce((int)t_hi, false);
    // Drain: every issued load lands before the CTA exits.
    for (int k2 = max(0, pissued - STAGES); k2 < pissued; ++k2)
      mbar_wait(&full[k2 % STAGES], (uint32_t)((k2 / STAGES) & 1), p.err, kDevErrWaitFull);
  } else if (active && warp < Cfg::CWARPS) {
    // ------------------------------------------------------------ consumers
    constexpr int WPH = Cfg::WPH, RW = Cfg::RW, NT = Cfg::NT, KP = Cfg::KP;
    const int g = warp / WPH, hf = warp % WPH;
    const int r = lane >> 2, qd = lane & 3;
    const bool row_ok = r < p.group;
    const float sl2 = p.scale_log2;
    float* my_mrg = mrg + warp * Cfg::MRG_FLOATS;

    uint32_t qa[4][4];
    float o[8][4];
    float m_run = kNegBig, l_run = 0.f;
    bool failed = false;
    const int tlo = (int)t_lo, thi = (int)t_hi;
    int st = 0, s = 0;
    uint32_t ph = 0;
    for (int t = tlo; t < thi; ++s) {
      // One segment: the tiles of sequence s inside [tlo, thi).  Everything
      // per sequence lives in registers for the tile loop.
      while (prefix[s + 1] <= t) ++s;
      const int seg_lo = t, seq_lo = prefix[s], seq_hi = prefix[s + 1];
      const int s_end = min(thi, seq_hi);
      const int pos_s = p.pos[s];
      const int n_loc = local_rows(pos_s, p.shard_start, p.max_ctx);
      const int local_new = pos_s - p.shard_start;  // this shard's row of the new token
      const bool has_new = p.new_row && local_new >= 0 && local_new < p.max_ctx;
      {
        const float* qh = p.q_in + ((size_t)s * p.n_head + (size_t)g * p.group + (row_ok ? r : 0)) * 64;
        const float2* cs = reinterpret_cast<const float2*>(p.cs + (size_t)pos_s * 64);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int d = 16 * kk + 8 * half + 2 * qd;
            float2 v = make_float2(0.f, 0.f);
            if (row_ok) {
              v = *reinterpret_cast<const float2*>(qh + d);
              if (p.rope) v = rot(v, cs[d >> 1]);
            }
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
      for (; t < s_end; ++t) {
      const int j = t - seq_lo;
      const int tile_valid = min(TILE, n_loc - j * TILE);
      const int my_valid = max(0, min(RW, tile_valid - RW * hf));
      if (!failed && !mbar_wait(&full[st], ph, p.err, kDevErrWaitFull)) failed = true;

      if (!failed && my_valid > 0) {
        uint8_t* kbox = smem + st * Cfg::STAGE_BYTES + g * Cfg::BOX;
        uint8_t* vbox = smem + st * Cfg::STAGE_BYTES + (NKV + g) * Cfg::BOX;
        const int rb = RW * hf;
        bool touched = false;
        if (my_valid < RW) {
          // Rows past the attended window may hold anything; zero their V so
          // that 0-weighted rows add exactly zero.
          for (int e = lane; e < (RW - my_valid) * 8; e += 32) {
            const int row = rb + my_valid + (e >> 3);
            reinterpret_cast<uint4*>(vbox + row * 128)[e & 7] = make_uint4(0, 0, 0, 0);
          }
          touched = true;
        }
        // The new token's row: rotated k and v in bf16 into the staged tile
        // and into the cache.
        const int r_new = local_new - j * TILE - rb;
        if (has_new && r_new >= 0 && r_new < RW) {
          if (lane < 8) {
            const int row = rb + r_new;
            const int e0 = g * 64 + lane * 8;
            const float* kr = p.k_io + (size_t)s * p.n_kv * 64 + e0;
            const float* vr = p.v_new + (size_t)s * p.n_kv * 64 + e0;
            const float2* cs = reinterpret_cast<const float2*>(p.cs + (size_t)pos_s * 64);
            uint4 kq, vq;
            uint32_t* kw = reinterpret_cast<uint32_t*>(&kq);
            uint32_t* vw = reinterpret_cast<uint32_t*>(&vq);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              float2 x = *reinterpret_cast<const float2*>(kr + 2 * u);
              x = p.rope ? rot(x, cs[lane * 4 + u]) : x;
              const __nv_bfloat162 kb = __floats2bfloat162_rn(x.x, x.y);
              const __nv_bfloat162 vb = __floats2bfloat162_rn(vr[2 * u], vr[2 * u + 1]);
              kw[u] = *reinterpret_cast<const uint32_t*>(&kb);
              vw[u] = *reinterpret_cast<const uint32_t*>(&vb);
            }
            const int sw = (lane ^ (row & 7)) << 4;
            *reinterpret_cast<uint4*>(kbox + row * 128 + sw) = kq;
            *reinterpret_cast<uint4*>(vbox + row * 128 + sw) = vq;
            const size_t crow = ((size_t)s * p.max_ctx + (pos_s - p.shard_start)) * p.n_kv * 64 + e0;
            *reinterpret_cast<uint4*>(p.kc_layer + crow) = kq;
            *reinterpret_cast<uint4*>(p.vc_layer + crow) = vq;
          }
          touched = true;
        }
        if (touched) {
          fence_proxy_async_smem();
          __syncwarp();
        }
        const uint32_t kb = smem_u32(kbox), vb = smem_u32(vbox);
        // S = q . K^T for this warp's RW rows: NT n-tiles of 8 rows.
        float sc[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // Two accumulators (dims 0-31 / 32-63) halve the dependent chain.
          float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
          const int row = rb + 8 * nt + (lane & 7);
#pragma unroll
          for (int kq = 0; kq < 2; ++kq) {
            const int chunk = 4 * kq + (lane >> 3);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(kb + row * 128 + ((chunk ^ (row & 7)) << 4), b0, b1, b2, b3);
            mma_bf16_16816(acc[kq], qa[2 * kq], b0, b1);
            mma_bf16_16816(acc[kq], qa[2 * kq + 1], b2, b3);
          }
          const int c0 = 8 * nt + 2 * qd;
          sc[nt][0] = (c0 < my_valid) ? ((acc[0][0] + acc[0][2]) + (acc[1][0] + acc[1][2])) * sl2 : -INFINITY;
          sc[nt][1] = (c0 + 1 < my_valid) ? ((acc[0][1] + acc[0][3]) + (acc[1][1] + acc[1][3])) * sl2 : -INFINITY;
        }
        // Online softmax over the RW rows (per query head = per quad).
        float mx = sc[0][0];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mx = fmaxf(mx, fmaxf(sc[nt][0], sc[nt][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = ex2(m_run - m_new);
        m_run = m_new;
        float pr[NT][2];
        float lsum = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          pr[nt][0] = ex2(sc[nt][0] - m_new);
          pr[nt][1] = ex2(sc[nt][1] - m_new);
          lsum += pr[nt][0] + pr[nt][1];
        }
        l_run = l_run * alpha + lsum;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          o[c][0] *= alpha; o[c][1] *= alpha; o[c][2] *= alpha; o[c][3] *= alpha;
        }
        // O += P . V, KP k-steps of 16 rows.
#pragma unroll
        for (int kp = 0; kp < KP; ++kp) {
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
      if (++st == STAGES) {
        st = 0;
        ph ^= 1u;
      }
      }
      // Segment end: merge the WPH warps of each KV head and write out.
      {
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
        cons_sync(NCT);
        const bool complete = seg_lo == seq_lo && s_end == seq_hi;
        float* dst = complete ? (p.mode == 0 ? p.out + (size_t)s * qdim : p.records + (size_t)s * rf)
                              : p.part + (size_t)(2 * cta + (seg_lo == tlo ? 0 : 1)) * rf;
        const bool normalise = complete && p.mode == 0;
        if (hf == 0 && row_ok) {
          float M = kNegBig;
#pragma unroll
          for (int w = 0; w < WPH; ++w) M = fmaxf(M, my_mrg[w * Cfg::MRG_FLOATS + 512 + r]);
          float wt[WPH];
          float L = 0.f;
#pragma unroll
          for (int w = 0; w < WPH; ++w) {
            wt[w] = ex2(my_mrg[w * Cfg::MRG_FLOATS + 512 + r] - M);
            L = fmaf(my_mrg[w * Cfg::MRG_FLOATS + 520 + r], wt[w], L);
          }
          const float inv = normalise ? 1.f / L : 1.f;
          const int h = g * p.group + r;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int d = 8 * c + 2 * qd;
            float2 v = make_float2(0.f, 0.f);
#pragma unroll
            for (int w = 0; w < WPH; ++w) {
              v.x = fmaf(my_mrg[w * Cfg::MRG_FLOATS + r * 64 + d], wt[w], v.x);
              v.y = fmaf(my_mrg[w * Cfg::MRG_FLOATS + r * 64 + d + 1], wt[w], v.y);
            }
            v.x *= inv;
            v.y *= inv;
            *reinterpret_cast<float2*>(dst + h * 64 + d) = v;
          }
          if (!normalise && qd == 0) {
            dst[qdim + h] = M;
            dst[qdim + p.n_head + h] = L;
          }
        }
        if (complete && p.rope) {
          // Only this CTA read the raw q of s (segment start) and k of its new
          // row (tile loop), and the barrier above ordered those reads: the
          // rotated pairs go back to the caller, one thread per pair.
          const float2* cs2 = reinterpret_cast<const float2*>(p.cs + (size_t)pos_s * 64);
          const float2* qi = reinterpret_cast<const float2*>(p.q_in + (size_t)s * qdim);
          float2* qo = reinterpret_cast<float2*>(p.q_out + (size_t)s * qdim);
          for (int e = threadIdx.x; e < qdim / 2; e += NCT) qo[e] = rot(qi[e], cs2[e & 31]);
          if (p.k_io) {
            const float2* ki = reinterpret_cast<const float2*>(p.k_io + (size_t)s * p.n_kv * 64);
            float2* ko = reinterpret_cast<float2*>(p.k_out + (size_t)s * p.n_kv * 64);
            for (int e = threadIdx.x; e < p.n_kv * 32; e += NCT) ko[e] = rot(ki[e], cs2[e & 31]);
          }
        }
        cons_sync(NCT);
      }
    }
  }
  if (stamp && threadIdx.x == 0) stamp[2] = global_ns();
  if (stamp && threadIdx.x == 0) stamp[3] = global_ns();
}


// ------------------------------------------------------------ merge / exchange

constexpr int kMaxMergeGroups = 4;
constexpr int kPartBatch = 16;  // parts per group per load round

// One item per (sequence s, head h) and 64 * GROUPS threads: thread d of
// group grp handles dimension d of parts grp, grp + GROUPS, ...  Every part's
// m, l and o are loaded in the same round (kPartBatch per group) and merged
// online, then the groups are combined through shared memory.
//   1. this GPU's record slice of (s, h): the merge of the partial records of
//      a split sequence, the complete record the decode kernel wrote, or a
//      neutral record when this shard holds no row of s;
//   2. mode 0: output of split sequences; mode 1: the record;
//      mode 2: the slice is stored into every GPU's receive words, each
//      value tagged with the launch's epoch, the words of all GPUs are
//      awaited (bounded) and the slices merged into the output;
//   3. with RoPE, the rotated q (and k for h < n_kv) of the sequences that
//      the decode kernel did not finish inside one CTA go back to the caller.
// In mode 2 the grid is persistent: CTA c takes items c, c + grid, ... in
// increasing order on every GPU, and the grid is small enough to be
// resident, so a CTA waiting for another GPU's item i only ever waits for a
// CTA that processes i next.
template <int GROUPS>
__global__ void __launch_bounds__(64 * GROUPS) merge_exchange_kernel(const FusedParams p) {
  __shared__ float o_grp[GROUPS][64];
  __shared__ float ml_grp[GROUPS][2];
  __shared__ int pre[64 * GROUPS + 1];
  __shared__ int wsum[2 * GROUPS];
  const int tid = threadIdx.x, d = tid & 63, grp = tid >> 6;
  griddep_launch_dependents();
  unsigned long long* stamp = (p.stamps && (int)blockIdx.x < 2 * p.grid)
                                  ? p.stamps + (size_t)(p.grid + blockIdx.x) * kStampsPerCta
                                  : nullptr;
  if (stamp && tid == 0) stamp[0] = global_ns();
  // With at most one sequence per thread, the tile prefix is rebuilt from the
  // positions before the wait (as the decode kernel does); otherwise the
  // decode kernel's copy is read after it.
  const bool local_sched = p.B <= 64 * GROUPS;
  // The RoPE row of this CTA's first item (the table is written only when
  // it is created).
  const int s_first = blockIdx.x / p.n_head;
  const int pos_first = s_first < p.B ? __ldcg(p.pos + s_first) : -1;
  float2 cs_first = make_float2(0.f, 0.f);
  if (p.rope && pos_first >= 0 && pos_first < p.table_len)
    cs_first = reinterpret_cast<const float2*>(p.cs + (size_t)pos_first * 64)[d >> 1];
  if (local_sched) {
    const int lane = tid & 31, w = tid >> 5;
    const int tiles = tid < p.B ? max(seq_tiles(p, __ldcg(p.pos + tid)), 0) : 0;
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) wsum[w] = incl;
    __syncthreads();
    int off = 0;
    for (int i = 0; i < w; ++i) off += wsum[i];
    if (tid < p.B) pre[tid + 1] = off + incl;
    if (tid == 0) pre[0] = 0;
    __syncthreads();
  }
  griddep_wait();
  if (stamp && tid == 0) stamp[1] = global_ns();
  const int* sched = local_sched ? pre : p.sched;
  const int H = p.n_head, qdim = H * 64, rf = record_floats(H, 64);
  const uint32_t epoch = (p.mode == 2) ? *reinterpret_cast<volatile unsigned*>(p.epoch) : 0u;
  const int T = sched[p.B];
  const int G = min(p.grid, T);
  const int items = p.B * H;
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int s = it / H, h = it - s * H;
    const int t0 = sched[s], t1 = sched[s + 1];
    const int c1 = t1 > t0 ? cta_of_tile(t0, G, T) : 0;
    const int c2 = t1 > t0 ? cta_of_tile(t1 - 1, G, T) : 0;
    const bool split = t1 > t0 && c1 != c2;
    if (p.mode == 0 && !split) continue;  // finished by the decode kernel
    const bool first = it == (int)blockIdx.x;
    const int pos_s = first ? pos_first : p.pos[s];
    const bool rope = p.rope && (split || t1 == t0) && grp == 0 && pos_s >= 0 &&
                      pos_s < p.table_len;
    const bool has_k = rope && p.k_io && h < p.n_kv;
    // Raw q / k pair of this thread, loaded with everything else.
    float2 xq = make_float2(0.f, 0.f), xk = make_float2(0.f, 0.f), cs = make_float2(0.f, 0.f);
    if (rope) {
      const float* qi = p.q_in + (size_t)s * qdim + h * 64;
      xq = make_float2(qi[d & ~1], qi[d | 1]);
      cs = first ? cs_first : reinterpret_cast<const float2*>(p.cs + (size_t)pos_s * 64)[d >> 1];
      if (has_k) {
        const float* kk = p.k_io + (size_t)s * p.n_kv * 64 + h * 64;
        xk = make_float2(kk[d & ~1], kk[d | 1]);
      }
    }
    float o = 0.f, m = kNegBig, l = 0.f;  // this GPU's record slice (group 0)
    if (split) {
      const int first_slot = 2 * c1 + (cta_tile_lo(c1, G, T) == t0 ? 0 : 1);
      const int n_parts = 1 + (c2 - c1);
      float mg = kNegBig, lg = 0.f, og = 0.f;
      for (int k0 = grp; k0 < n_parts; k0 += GROUPS * kPartBatch) {
        float mv[kPartBatch], lv[kPartBatch], ov[kPartBatch];
#pragma unroll
        for (int u = 0; u < kPartBatch; ++u) {
          const int kk = k0 + u * GROUPS;
          mv[u] = kNegBig;
          lv[u] = 0.f;
          ov[u] = 0.f;
          if (kk < n_parts) {
            const float* r = p.part + (size_t)(kk == 0 ? first_slot : 2 * (c1 + kk)) * rf;
            mv[u] = r[qdim + h];
            lv[u] = r[qdim + H + h];
            ov[u] = r[h * 64 + d];
          }
        }
        float Mb = mg;
#pragma unroll
        for (int u = 0; u < kPartBatch; ++u) Mb = fmaxf(Mb, mv[u]);
        const float a = ex2(mg - Mb);
        og *= a;
        lg *= a;
#pragma unroll
        for (int u = 0; u < kPartBatch; ++u) {
          const float w = ex2(mv[u] - Mb);
          og = fmaf(ov[u], w, og);
          lg = fmaf(lv[u], w, lg);
        }
        mg = Mb;
      }
      if (GROUPS > 1) {
        o_grp[grp][d] = og;
        if (d == 0) {
          ml_grp[grp][0] = mg;
          ml_grp[grp][1] = lg;
        }
        __syncthreads();
        if (grp == 0) {
          float M = kNegBig;
#pragma unroll
          for (int g2 = 0; g2 < GROUPS; ++g2) M = fmaxf(M, ml_grp[g2][0]);
          o = 0.f;
          l = 0.f;
#pragma unroll
          for (int g2 = 0; g2 < GROUPS; ++g2) {
            const float w = ex2(ml_grp[g2][0] - M);
            o = fmaf(o_grp[g2][d], w, o);
            l = fmaf(ml_grp[g2][1], w, l);
          }
          m = M;
        }
      } else {
        o = og;
        m = mg;
        l = lg;
      }
    } else if (t1 > t0 && p.mode != 0 && grp == 0) {
      const float* rec = p.records + (size_t)s * rf;
      o = rec[h * 64 + d];
      m = rec[qdim + h];
      l = rec[qdim + H + h];
    }
    if (p.mode == 0) {
      if (grp == 0) p.out[(size_t)s * qdim + h * 64 + d] = o / l;
    } else if (p.mode == 1) {
      if ((split || t1 == t0) && grp == 0) {
        float* rec = p.records + (size_t)s * rf;
        rec[h * 64 + d] = o;
        if (d == 0) {
          rec[qdim + h] = m;
          rec[qdim + H + h] = l;
        }
      }
    } else {
      // Peer exchange: each value travels with its epoch tag in one 8-byte
      // store (single-copy atomic), so a receiver that sees the tag sees the
      // value -- no fence and no separate flag.  Receive words alternate
      // between launches by epoch parity (a GPU is at most one launch ahead).
      const int par = (int)(epoch & 1);
      const unsigned long long tag = (unsigned long long)epoch << 32;  // epoch >= 1
      const size_t item_words = (size_t)kXchgWords;
      const size_t mine = (((size_t)(par * p.world + p.rank) * p.b_cap + s) * H + h) * item_words;
      if (grp == 0) {
        const unsigned long long wo = tag | __float_as_uint(o);
        const unsigned long long wm = tag | __float_as_uint(m);
        const unsigned long long wl = tag | __float_as_uint(l);
        for (int r = 0; r < p.world; ++r) {
          unsigned long long* dst = (r == p.rank ? p.xchg_local : p.xchg_peer[r]) + mine;
          st_relaxed_sys_u64(dst + d, wo);
          if (d == 0) {
            st_relaxed_sys_u64(dst + 64, wm);
            st_relaxed_sys_u64(dst + 65, wl);
          }
        }
        if (stamp && tid == 0 && it == (int)blockIdx.x) stamp[2] = global_ns();
        // Gather: this thread's dimension and every GPU's m and l.
        const unsigned long long* base =
            p.xchg_local + (((size_t)(par * p.world) * p.b_cap + s) * H + h) * item_words;
        const size_t stride = (size_t)p.b_cap * H * item_words;
        float mv[kMaxPeers], lv[kMaxPeers], ov[kMaxPeers];
        unsigned pending = (1u << p.world) - 1u;
        const unsigned long long t_end = global_ns() + (unsigned long long)p.wait_ns;
        for (long long n = 0; pending && n < kPollCap; ++n) {
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) {
            if (!(pending >> r & 1u)) continue;
            const unsigned long long* rr = base + r * stride;
            const unsigned long long x = ld_relaxed_sys_u64(rr + d);
            const unsigned long long y = ld_relaxed_sys_u64(rr + 64);
            const unsigned long long z = ld_relaxed_sys_u64(rr + 65);
            if ((x >> 32) == (tag >> 32) && (y >> 32) == (tag >> 32) && (z >> 32) == (tag >> 32)) {
              ov[r] = __uint_as_float((unsigned)x);
              mv[r] = __uint_as_float((unsigned)y);
              lv[r] = __uint_as_float((unsigned)z);
              pending &= ~(1u << r);
            }
          }
          if (pending && global_ns() > t_end) break;
        }
        if (pending) {
          record_error(p.err, kDevErrPeerTimeout);
        } else {
          float M = kNegBig;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r)
            if (r < p.world) M = fmaxf(M, mv[r]);
          float O = 0.f, L = 0.f;
#pragma unroll
          for (int r = 0; r < kMaxPeers; ++r) {
            if (r < p.world) {
              const float w = ex2(mv[r] - M);
              O = fmaf(ov[r], w, O);
              L = fmaf(lv[r], w, L);
            }
          }
          p.out[(size_t)s * qdim + h * 64 + d] = O / L;
        }
      }
    }
    if (rope) {
      // All readers of the raw q / k of s have finished (previous kernel);
      // each thread writes only the element of the pair it owns.
      const float2 rq = rot(xq, cs);
      p.q_out[(size_t)s * qdim + h * 64 + d] = (d & 1) ? rq.y : rq.x;
      if (has_k) {
        const float2 rk = rot(xk, cs);
        p.k_out[(size_t)s * p.n_kv * 64 + h * 64 + d] = (d & 1) ? rk.y : rk.x;
      }
    }
    if (GROUPS > 1) __syncthreads();
  }
  if (stamp && tid == 0) stamp[3] = global_ns();
}

// ---------------------------------------------------------------- launch

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl_f(void (*fn)(KArgs...), dim3 grid, dim3 block, size_t smem,
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

template <int NKV, int RING_KB>
static cudaError_t launch_fused_cfg(const CUtensorMap& tk, const CUtensorMap& tv,
                                    const FusedParams& p, int grid, cudaStream_t st) {
  using Cfg = FusedCfg<NKV, RING_KB>;
  static size_t configured[64] = {};
  const size_t smem = Cfg::smem_bytes(p.B);
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(decode_fused_kernel<NKV, RING_KB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(decode_fused_kernel<NKV, RING_KB>,
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    configured[dev] = smem;
  }
  return launch_pdl_f(decode_fused_kernel<NKV, RING_KB>, dim3(grid), dim3(Cfg::THREADS), smem,
                      st, tk, tv, p);
}

size_t decode_fused_smem(int nkv, int ring_kb, int B) {
  const bool deep = ring_kb == kFusedRingDeep;
  switch (nkv) {
    case 1: return deep ? FusedCfg<1, kFusedRingDeep>::smem_bytes(B) : FusedCfg<1, kFusedRing>::smem_bytes(B);
    case 2: return deep ? FusedCfg<2, kFusedRingDeep>::smem_bytes(B) : FusedCfg<2, kFusedRing>::smem_bytes(B);
    case 4: return deep ? FusedCfg<4, kFusedRingDeep>::smem_bytes(B) : FusedCfg<4, kFusedRing>::smem_bytes(B);
    default: return 0;
  }
}


cudaError_t launch_decode_fused(const CUtensorMap& tk, const CUtensorMap& tv,
                                const FusedParams& p, int ring_kb, int grid, cudaStream_t st) {
  const bool deep = ring_kb == kFusedRingDeep;
  if (!deep && ring_kb != kFusedRing) return cudaErrorInvalidValue;
  switch (p.n_kv) {
    case 1: return deep ? launch_fused_cfg<1, kFusedRingDeep>(tk, tv, p, grid, st)
                        : launch_fused_cfg<1, kFusedRing>(tk, tv, p, grid, st);
    case 2: return deep ? launch_fused_cfg<2, kFusedRingDeep>(tk, tv, p, grid, st)
                        : launch_fused_cfg<2, kFusedRing>(tk, tv, p, grid, st);
    case 4: return deep ? launch_fused_cfg<4, kFusedRingDeep>(tk, tv, p, grid, st)
                        : launch_fused_cfg<4, kFusedRing>(tk, tv, p, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_merge_exchange(const FusedParams& p, int grid, int groups, cudaStream_t st) {
  if (p.B <= 0) return cudaSuccess;
  if (groups == kMaxMergeGroups)
    return launch_pdl_f(merge_exchange_kernel<kMaxMergeGroups>, dim3(grid),
                        dim3(64 * kMaxMergeGroups), 0, st, p);
  if (groups == 1) return launch_pdl_f(merge_exchange_kernel<1>, dim3(grid), dim3(64), 0, st, p);
  return cudaErrorInvalidValue;
}

}  // namespace tg
