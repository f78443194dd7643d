// tg_kernels.h -- host-side launchers of the kernels in tg_kernels.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "tg_shared.h"

namespace tg {

cudaError_t launch_rope(const RopeParams& p, cudaStream_t st);

// Tensor-core split-KV decode over a bf16 cache with head_dim 64, n_kv in
// {1, 2, 4} and at most 8 query heads per KV head.  tk / tv are 2-D TMA
// maps of the whole cache ({n_kv*64, rows}, box {64, 64}, 128B swizzle).
cudaError_t launch_decode_mma(const CUtensorMap& tk, const CUtensorMap& tv,
                              const DecodeParams& p, int grid, cudaStream_t st);
size_t decode_mma_smem(int nkv, int B);
int mma_threads(int nkv);

// CUDA-core decode (fp32 or bf16 cache, any head_dim / group the limits in
// tg_backend.cu allow).
cudaError_t launch_decode_generic(const DecodeParams& p, int dtype, int grid,
                                  cudaStream_t st);
size_t decode_generic_smem(int B, int n_head, int n_kv, int hd);
int decode_generic_blocks_per_sm(int dtype, size_t smem);

// Caches of at most kSmallMaxRows positions, head_dim 64, at most 8 query
// heads per KV head, mode 0 only: a cluster of p.split (1, 2, 4 or 8) CTAs
// per (sequence, KV head), writes p.out directly (no merge launch).
constexpr int kSmallMaxRows = 1024;
cudaError_t launch_decode_small(const DecodeParams& p, int dtype, cudaStream_t st);
size_t decode_small_smem(int group, int max_ctx, int split);

cudaError_t launch_merge(const MergeParams& p, cudaStream_t st);

// Copies of a call's packed host inputs from page-locked staging (through
// its device address) into their device slots, issued by a kernel so that
// the kernels of a batch follow one another with programmatic overlap (a
// copy node or an event wait between two kernels removes it).
constexpr int kStageMaxRuns = 8;
struct StageRun {
  const uint4* src;
  uint4* dst;
  int n16;  // 16-byte words
};
struct StageParams {
  StageRun run[kStageMaxRuns];
  int n_runs;
};
cudaError_t launch_stage_copy(const StageParams& p, int total16, cudaStream_t st);
// Deferred host outputs of a batch: entry e copies `bytes` from device
// memory `src` to `dst` (the device address of page-locked host memory).
// The entry list itself lives in page-locked memory (read through its
// device address before the grid-dependency wait); one CTA per entry.
struct StoreEntry {
  void* dst;
  const void* src;
  unsigned long long bytes;
};
cudaError_t launch_store_out(const StoreEntry* list, int n, cudaStream_t st);
// Raises the shared-memory limit of the tensor-core decode (n_kv 1, 2, 4) and
// the CUDA-core decode (fp32, bf16) on the current device to what max_seqs
// sequences can need, so that later launches change no kernel attribute.
cudaError_t prepare_decode_kernels(int max_seqs);
cudaError_t launch_gather_merge(const GatherMergeParams& p, cudaStream_t st);
cudaError_t launch_elem(int op, float* data, const float* aux, int dim,
                        cudaStream_t st);
cudaError_t launch_fill_normal(void* out, size_t n, int dtype, uint64_t seed,
                               int num_sms, cudaStream_t st);
cudaError_t launch_convert_rows(void* dst, const float* src, size_t n,
                                int dtype, int num_sms, cudaStream_t st);

// Fused decode step (tg_decode_fused.cu): bf16 cache, head_dim 64,
// n_kv in {1, 2, 4}, at most 8 query heads per KV head.
// ring_kb: K/V ring per CTA, kFusedRing or kFusedRingDeep.
constexpr int kFusedRing = 128;
constexpr int kFusedRingDeep = 192;
cudaError_t launch_decode_fused(const CUtensorMap& tk, const CUtensorMap& tv,
                                const FusedParams& p, int ring_kb, int grid, cudaStream_t st);
// groups: 1 (64 threads per item, many items) or 4 (256 threads, few items or
// the persistent peer-exchange grid).
constexpr int kMergeGroupsWide = 4;
cudaError_t launch_merge_exchange(const FusedParams& p, int grid, int groups, cudaStream_t st);
size_t decode_fused_smem(int nkv, int ring_kb, int B);

// Prefill (tg_prefill.cu).  The attention kernel needs a bf16 cache with
// head_dim 64 and S a positive length; tq is a 3-D map of the rotated bf16 q
// ({64, n_head, B*S}, box {64, 1, 128}), tk / tv 2-D maps of the cache with
// 128-row boxes.
cudaError_t launch_prefill_rope(const PrefillRopeParams& p, cudaStream_t st);
cudaError_t launch_prefill_attn(const CUtensorMap& tq, const CUtensorMap& tk,
                                const CUtensorMap& tv, const PrefillParams& p, int grid,
                                cudaStream_t st);
size_t prefill_attn_smem();

// Q/K/V projection (tg_qkv.cu), cols a multiple of 32 up to qkv_max_cols().
// Batches of kQkvGemmMinB or more (cols up to qkv_gemm_max_cols()) take the
// batched kernel with kQkvGemmRows rows per CTA (qkv_use_gemm), others
// kQkvRows; p.tiles must follow the kernel launch_qkv picks.
cudaError_t launch_qkv(const QkvParams& p, cudaStream_t st);
size_t qkv_smem(int cols);
int qkv_max_cols();
int qkv_gemm_max_cols();
bool qkv_use_gemm(int B, int cols);
// Rows per CTA of the kernel launch_qkv picks for (B, cols): the tensor-core
// kernel (128) for batches of kQkvGemmMinB+ with cols up to
// qkv_tc_max_cols(), else the CUDA-core batched kernel or the GEMV.
int qkv_tc_max_cols();
// Cluster width (1 to 8 CTAs splitting the columns) of a tensor-core
// projection launch of `tiles` row tiles x sequence groups on device dev,
// from the device's resident-cluster count; 0 if none fits.
int qkv_tc_split(int tiles, int cols, int dev);
// Fixes the cluster width of later launches (1 to 8, clamped to the chunk
// count) or restores the automatic choice (0); -1 for other values.
int set_qkv_tc_split(int split);
bool qkv_use_tc(int B, int cols);
int qkv_rows_per_cta(int B, int cols);

}  // namespace tg
