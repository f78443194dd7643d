// tg_noalloc.cu -- decode attention that allocates no device memory.
//
// Some callers cannot call cudaMalloc at the point where they run attention:
// code recording a CUDA graph in global capture mode (where allocation calls
// are refused), runtimes that hand out a fixed pool and forbid the driver
// allocator after start-up, or an allocator hook that must not re-enter
// itself.  tg_attention_noalloc serves them: the caller passes device
// buffers for inputs and outputs, and the scratch the split-KV decode needs
// (partial softmax records, the tile schedule, the device error word) lives
// in one file-scope __device__ array of fixed size, g_noalloc_scratch, that
// every GPU which loads the library holds until the process exits.
//
// The entry point calls no cudaMalloc / cudaFree or any allocating routine.
// Its first call on a device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture.  Every call shares the array and it
// keeps the last call's contents: the error word is cleared at the start of
// each call, the schedule and the partial records are rewritten before they
// are read.  Calls whose GPU work overlaps (different streams, different
// threads) race on the array.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/tg_cuda_backend.h"
#include "tg_internal.h"
#include "tg_kernels.h"
#include "tg_shared.h"

namespace {

// Layout of the array: partial records, then the tile prefix, then the
// error word.  4 MiB of records hold 2 slots x G CTAs of n_head*(hd+2)
// floats; the grid is narrowed when a shape would need more.
constexpr size_t kPartBytes = size_t(4) << 20;
constexpr int kMaxSeqs = TG_NOALLOC_MAX_SEQS;
constexpr size_t kSchedBytes = (size_t(kMaxSeqs + 1) * 4 + 255) & ~size_t(255);
constexpr size_t kScratchBytes = kPartBytes + kSchedBytes + 256;
constexpr int kMaxDevices = 64;

static_assert(kScratchBytes == TG_NOALLOC_SCRATCH_BYTES, "scratch size stated in the header");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
unsigned char* g_scratch_addr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};

int err(int code, const char* fmt, ...) {
  char buf[384];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return tg::set_last_error(code, buf);
}

// Once per device, with that device current: the array's device address
// (host code must not use the symbol itself), the SM count, and the
// shared-memory limits of every kernel variant this entry point can launch,
// raised to what TG_NOALLOC_MAX_SEQS sequences need, so that a later call
// with another dtype, shape or batch changes no kernel attribute.
int setup(int dev, unsigned char** scratch, int* sms) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return err(TG_ERR_CUDA, "cudaGetSymbolAddress(g_noalloc_scratch): %s",
                 cudaGetErrorString(e));
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return err(TG_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    e = tg::prepare_decode_kernels(kMaxSeqs);
    if (e != cudaSuccess)
      return err(TG_ERR_CUDA, "tg_attention_noalloc: kernel set-up: %s", cudaGetErrorString(e));
    g_sms[dev] = n;
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
  }
  *scratch = g_scratch_addr[dev];
  *sms = g_sms[dev];
  return TG_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

extern "C" TG_API int tg_attention_noalloc(void* cuda_stream, const float* q, const void* k_cache,
                                           const void* v_cache, int dtype, int n_seqs,
                                           int max_ctx, int n_head, int n_kv_head, int head_dim,
                                           const int32_t* past_len, float* out,
                                           int* device_status) {
  if (!q || !k_cache || !v_cache || !past_len || !out)
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: null buffer");
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 7)
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: q and out must be 8-byte aligned");
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16)
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: dtype %d", dtype);
  if (n_head <= 0 || n_kv_head <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 128 ||
      n_head % n_kv_head || n_head * head_dim > 4096 || n_kv_head * head_dim > 1024 ||
      (n_kv_head * head_dim) % 8)
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: unsupported shape %d/%d/%d", n_head,
               n_kv_head, head_dim);
  if (n_seqs < 1 || n_seqs > kMaxSeqs)
    return err(TG_ERR_INVALID_ARG,
               "tg_attention_noalloc: n_seqs %d outside [1, %d], the size of its fixed "
               "scratch schedule",
               n_seqs, kMaxSeqs);
  if (max_ctx < 1 || (long long)n_seqs * max_ctx >= (1LL << 31))
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: max_ctx %d", max_ctx);
  const int rf = tg::record_floats(n_head, head_dim);
  const int max_grid = (int)(kPartBytes / (2 * (size_t)rf * 4));
  if (max_grid < 1)
    return err(TG_ERR_INVALID_ARG, "tg_attention_noalloc: record of %d floats exceeds scratch",
               rf);

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return err(TG_ERR_NO_DEVICE, "tg_attention_noalloc: no current device");
  unsigned char* scratch = nullptr;
  int sms = 0;
  int rc = setup(dev, &scratch, &sms);
  if (rc != TG_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  float* part = reinterpret_cast<float*>(scratch);
  int* sched = reinterpret_cast<int*>(scratch + kPartBytes);
  int* dev_err = reinterpret_cast<int*>(scratch + kPartBytes + kSchedBytes);

  tg::DecodeParams p{};
  p.q = q;
  p.out = out;
  p.past_len = past_len;
  p.k = k_cache;
  p.v = v_cache;
  p.part = part;
  p.sched = sched;
  p.err = dev_err;
  p.row0 = 0;
  p.B = n_seqs;
  p.n_head = n_head;
  p.n_kv = n_kv_head;
  p.head_dim = head_dim;
  p.group = n_head / n_kv_head;
  p.max_ctx = max_ctx;
  p.shard_start = 0;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  p.mode = 0;
  p.aligned16 = ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) %
                     16 == 0)
                    ? 1
                    : 0;

  bool mma = dtype == TG_DTYPE_BF16 && head_dim == 64 &&
             (n_kv_head == 1 || n_kv_head == 2 || n_kv_head == 4) &&
             n_head / n_kv_head <= 8 && encoder() != nullptr;
  int grid = 0;
  size_t smem = 0;
  alignas(64) CUtensorMap tk, tv;
  if (mma) {
    const cuuint64_t gdim[2] = {(cuuint64_t)n_kv_head * 64, (cuuint64_t)n_seqs * max_ctx};
    const cuuint64_t gstride[1] = {(cuuint64_t)n_kv_head * 64 * 2};
    const cuuint32_t box[2] = {64, 64};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r1 = encoder()(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(k_cache),
                            gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CUresult r2 = encoder()(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(v_cache),
                            gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    // Caches that are not 16-byte aligned have no TMA descriptor: the
    // CUDA-core kernel takes them.
    if (r1 != CUDA_SUCCESS || r2 != CUDA_SUCCESS) mma = false;
  }
  if (mma) {
    smem = tg::decode_mma_smem(n_kv_head, n_seqs);
    grid = sms;
  } else {
    smem = tg::decode_generic_smem(n_seqs, n_head, n_kv_head, head_dim);
    int per_sm = tg::decode_generic_blocks_per_sm(dtype, smem);
    if (per_sm > 4) per_sm = 4;
    grid = sms * per_sm;
  }
  if (smem > 227 * 1024)
    return err(TG_ERR_INVALID_ARG,
               "tg_attention_noalloc: %d sequences of shape %d/%d/%d need %zu KB of shared "
               "memory (at most 227)",
               n_seqs, n_head, n_kv_head, head_dim, (smem + 1023) / 1024);
  if (grid > max_grid) grid = max_grid;

  e = cudaMemsetAsync(dev_err, 0, sizeof(int), st);
  if (e == cudaSuccess)
    e = mma ? tg::launch_decode_mma(tk, tv, p, grid, st)
            : tg::launch_decode_generic(p, dtype, grid, st);
  if (e == cudaSuccess) {
    tg::MergeParams m{};
    m.part = part;
    m.sched = sched;
    m.out = out;
    m.B = n_seqs;
    m.n_head = n_head;
    m.head_dim = head_dim;
    m.G = grid;
    m.mode = 0;
    e = tg::launch_merge(m, st);
  }
  if (e == cudaSuccess && device_status)
    e = cudaMemcpyAsync(device_status, dev_err, sizeof(int), cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess)
    return err(TG_ERR_CUDA, "tg_attention_noalloc: %s", cudaGetErrorString(e));
  return TG_OK;
}
