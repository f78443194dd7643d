// tg_backend.cu -- host side of the C ABI declared in include/tg_cuda_backend.h.
//
// Replaces the dispatch layer of the reference's Metal backend for the
// attention hot path (metal_backend.hpp:114-191 batches, :354-453 elem /
// rope / attention ops, metal_backend.cpp:21-89 init).  One tg_context per
// device and host thread: a CUDA stream, a device error word, scratch for
// split-KV partial records, RoPE cos/sin tables built with the host libm,
// device mirrors of host arrays for the reference-compatible ops, and an
// optional NCCL communicator (loaded with dlopen) for split-KV decode.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <dlfcn.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/tg_cuda_backend.h"
#include "tg_kernels.h"
#include "tg_shared.h"

#define TG_VERSION "tmac_gguf.cpp_b200 0.1.0"

namespace {

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

#define TG_CUDA(call)                                                        \
  do {                                                                       \
    cudaError_t e_ = (call);                                                 \
    if (e_ != cudaSuccess)                                                   \
      return fail(e_ == cudaErrorMemoryAllocation ? TG_ERR_OUT_OF_MEMORY     \
                                                  : TG_ERR_CUDA,             \
                  "%s failed: %s", #call, cudaGetErrorString(e_));           \
  } while (0)

#define TG_TRY(expr)          \
  do {                        \
    int rc_ = (expr);         \
    if (rc_ != TG_OK) return rc_; \
  } while (0)

// ------------------------------------------------------------ NCCL (dlopen)

struct NcclApi {
  void* lib = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int,
                                     ncclConfig_t*) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool ok = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static bool tried = false;
  if (tried) return api;
  tried = true;
  // Reuse the NCCL a host framework already loaded (same soname), else the
  // system one.
  const char* names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char* n : names) {
    api.lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
    if (api.lib) break;
  }
  if (!api.lib) return api;
  auto sym = [&](const char* s) { return dlsym(api.lib, s); };
  api.GetUniqueId = (decltype(api.GetUniqueId))sym("ncclGetUniqueId");
  api.CommInitRankConfig = (decltype(api.CommInitRankConfig))sym("ncclCommInitRankConfig");
  api.AllGather = (decltype(api.AllGather))sym("ncclAllGather");
  api.CommDestroy = (decltype(api.CommDestroy))sym("ncclCommDestroy");
  api.CommAbort = (decltype(api.CommAbort))sym("ncclCommAbort");
  api.CommGetAsyncError = (decltype(api.CommGetAsyncError))sym("ncclCommGetAsyncError");
  api.GetErrorString = (decltype(api.GetErrorString))sym("ncclGetErrorString");
  api.ok = api.GetUniqueId && api.CommInitRankConfig && api.AllGather &&
           api.CommDestroy && api.CommAbort && api.CommGetAsyncError &&
           api.GetErrorString;
  return api;
}

// ------------------------------------------------------------ TMA encode

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

constexpr float kLog2e = 1.4426950408889634f;

// Fused decode tuning (tg_set_decode_tuning): the K/V ring per CTA in KB
// (0 = automatic) and whether tiles may be loaded before the
// grid-dependency wait when that is safe (1) or never (0).
std::atomic<int> g_decode_ring{0};
std::atomic<int> g_decode_preload{0};

}  // namespace

// ================================================================ context

struct RopeTable {
  uint32_t base_bits = 0;
  int head_dim = 0;
  int len = 0;
  float* d = nullptr;  // [len][head_dim/2][cos, sin]
};

struct Region {
  char* host = nullptr;
  size_t bytes = 0;
  char* dev = nullptr;
  int flags = TG_REGION_MIRROR;
  bool transient = true;  // created by an op: lives until the batch ends
  bool fresh = false;     // device copy current for this batch
  size_t dirty_lo = 0, dirty_hi = 0;  // byte range written by device ops
};

struct PendingCopy {
  void* host;
  const void* dev;
  size_t bytes;
};

struct tg_context {
  int device = 0;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  // Inside a batch, host inputs move on this stream and `stream` waits for
  // them through copy_done (created at the first batched call).
  cudaStream_t copy_stream = nullptr;
  cudaEvent_t copy_done = nullptr;
  int* d_err = nullptr;
  int* h_err = nullptr;  // page-locked copy of d_err, read after a stream wait

  float* part = nullptr;     size_t part_cap = 0;    // floats
  int* sched = nullptr;      size_t sched_cap = 0;   // ints
  float* records = nullptr;  size_t rec_cap = 0;     // floats
  float* recv = nullptr;     size_t recv_cap = 0;    // floats

  char* arena = nullptr;     size_t arena_cap = 0, arena_off = 0;
  uint16_t* qbf = nullptr;   size_t qbf_cap = 0;     // prefill: rotated bf16 q
  uint16_t* vh = nullptr;     size_t vh_cap = 0;   // prefill: fp16 copy of v
  float* qx = nullptr;        size_t qx_cap = 0;   // decode from x: rotated q
  float* cx = nullptr;        size_t cx_cap = 0;   // attention block: context
  std::vector<PendingCopy> pending;  // device -> host copies of staged outputs
  // Page-locked host outputs of the current batch: kernels write device
  // slots, and one store kernel moves them to the host at tg_batch_end.
  struct DeferredStore {
    void* host;
    void* alias;  // device address of `host`
    const void* dev;
    size_t bytes;
  };
  std::vector<DeferredStore> dstores;
  // Host inputs of the current call, moved to the arena by commit_inputs.
  struct PackEntry {
    char* dev;
    const char* host;
    size_t bytes;
  };
  std::vector<PackEntry> pack;

  char* hpin = nullptr;      size_t hpin_cap = 0, hpin_off = 0;
  char* hpin_dev = nullptr;  // device address of the current pinned block
  std::vector<char*> hpin_old;  // outgrown pinned blocks, freed at the next sync
  std::vector<void*> graveyard;      // device buffers freed at the next sync

  std::vector<RopeTable> tables;
  std::map<uintptr_t, Region> regions;
  bool in_batch = false;
  bool capturing = false;    // a CUDA graph capture is open on the stream
  bool call_staged = false;  // the current call moved host data
  long long launches = 0;
  long long capture_launches0 = 0;

  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  int timeout_ms = 60000;


  // Peer-memory exchange of split-KV records (IPC-mapped receive buffers).
  bool p2p_ready = false, p2p_failed = false;
  int exchange_pref = TG_EXCHANGE_AUTO;  // tg_comm_set_exchange
  int exchange_used = TG_EXCHANGE_AUTO;  // last split-KV call
  int p2p_bcap = 0, p2p_rf = 0, p2p_heads = 0;
  unsigned long long* xchg_local = nullptr;  // peer-exchange receive words
  unsigned* xchg_ctl = nullptr;              // exchange epoch word (this GPU only)
  unsigned long long* xchg_peer[tg::kMaxPeers] = {};
  unsigned char* nccl_stage = nullptr;  // small device staging for handle exchange

  std::vector<tg_kv_cache*> caches;  // freed by tg_shutdown if still alive

  // Optional CUDA-event timing of each decode-attention kernel launch.
  int prof_on = 0;  // TG_PROFILE_* mask
  std::vector<cudaEvent_t> prof_ev;  // start/stop pairs
  size_t prof_used = 0;              // events recorded since the last read
  // Optional %globaltimer stamps of bf16 decode steps (TG_PROFILE_STAMPS):
  // one record of kStampRowsPerSm * num_sms rows per decode launch.
  unsigned long long* stamps = nullptr;
  int stamp_cap = 0, stamp_used = 0;

  long long wait_ns = 5000000000LL;  // bound of in-kernel waits (tg_comm_set_wait_limit_ms)

  // (cache, layer) pairs whose rows a kernel that lets its successor start
  // early (programmatic dependent launch) has written since the stream was
  // last known idle; layer -1 = every layer.  Such rows may still be in
  // flight when a later kernel starts, so the bf16 decode does not load
  // them before its grid-dependency wait.  pdl_unknown: work of unknown
  // extent (a graph launch) may still run.
  std::vector<std::pair<const tg_kv_cache*, int>> pdl_writes;
  std::vector<std::pair<const tg_kv_cache*, int>> pdl_saved;  // live set during a capture
  bool pdl_unknown = false, pdl_unknown_saved = false;
};

struct tg_graph {
  tg_context* ctx = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  long long kernels = 0;  // kernel launches recorded into the graph
};

struct tg_kv_cache {
  tg_context* ctx = nullptr;
  tg_kv_desc d{};
  size_t row_elems = 0, esize = 0, layer_elems = 0;
  void* k = nullptr;
  void* v = nullptr;
  bool tmap_ok = false;
  alignas(64) CUtensorMap tmk;
  alignas(64) CUtensorMap tmv;
  bool tmap128_ok = false;        // 128-row boxes for the prefill kernel
  alignas(64) CUtensorMap tmk128;
  alignas(64) CUtensorMap tmv128;
  int global_ctx = 0;
};

namespace {

int set_device(tg_context* ctx) {
  if (!ctx) return fail(TG_ERR_INVALID_ARG, "null context");
  TG_CUDA(cudaSetDevice(ctx->device));
  return TG_OK;
}

// Device-accessible without staging (device or managed memory).
bool is_device_ptr(const void* p) {
  if (!p) return false;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

void free_graveyard(tg_context* ctx) {
  for (void* p : ctx->graveyard) cudaFree(p);
  ctx->graveyard.clear();
  for (char* p : ctx->hpin_old) cudaFreeHost(p);
  ctx->hpin_old.clear();
}

template <typename T>
int ensure_buf(tg_context* ctx, T** buf, size_t* cap, size_t need) {
  if (need <= *cap) return TG_OK;
  if (ctx->capturing)
    return fail(TG_ERR_STATE,
                "scratch must be sized before graph capture: run the same call once first");
  size_t n = need < 1024 ? 1024 : need;
  n = n + n / 4;
  T* nb = nullptr;
  TG_CUDA(cudaMalloc(&nb, n * sizeof(T)));
  if (*buf) ctx->graveyard.push_back(*buf);
  *buf = nb;
  *cap = n;
  return TG_OK;
}

// Queues the copy of the device error word into its page-locked mirror
// behind the stream's work, so that the wait that follows also brings the
// word back (no second, synchronous copy after the wait).  Returns whether
// it was queued.
bool queue_error_read(tg_context* ctx) {
  if (!ctx->h_err || ctx->capturing) return false;
  if (cudaMemcpyAsync(ctx->h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost,
                      ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

// Reads and clears the device error word (stream must be idle).  queued:
// queue_error_read ran before the wait, so the mirror holds the word.
int check_device_error(tg_context* ctx, bool queued = false) {
  int h = 0;
  if (queued) {
    h = *reinterpret_cast<volatile int*>(ctx->h_err);
    *ctx->h_err = 0;
  } else {
    TG_CUDA(cudaMemcpy(&h, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  }
  if (h != 0) {
    TG_CUDA(cudaMemset(ctx->d_err, 0, sizeof(int)));
    const char* what = h == tg::kDevErrBadPos         ? "position outside the cache / RoPE table"
                       : h == tg::kDevErrWaitFull     ? "bounded wait for a K/V tile expired"
                       : h == tg::kDevErrWaitEmpty    ? "bounded wait for a free stage expired"
                       : h == tg::kDevErrPeerTimeout  ? "another GPU's softmax record did not arrive"
                           : "device error";
    return fail(TG_ERR_DEVICE, "kernel reported 0x%x: %s", h, what);
  }
  return TG_OK;
}

// Waits for the stream; with a communicator, polls NCCL's async error and
// aborts the communicator once the timeout passes.
// The stream has no work in flight: nothing written earlier can still be
// changing.
void stream_idle(tg_context* ctx) {
  if (ctx->capturing) return;
  ctx->pdl_writes.clear();
  ctx->pdl_unknown = false;
}

// Rows of (kv, layer) written by a kernel that may still be running when
// the next kernel starts (see tg_context::pdl_writes).
void note_pdl_write(tg_context* ctx, const tg_kv_cache* kv, int layer) {
  for (const auto& w : ctx->pdl_writes)
    if (w.first == kv && (w.second == layer || w.second == -1)) return;
  ctx->pdl_writes.emplace_back(kv, layer);
}

// True when no kernel that may still be running writes rows of (kv, layer),
// so the bf16 decode may load them before its grid-dependency wait.
bool preload_allowed(const tg_context* ctx, const tg_kv_cache* kv, int layer) {
  if (ctx->pdl_unknown || g_decode_preload == 0) return false;
  for (const auto& w : ctx->pdl_writes)
    if (w.first == kv && (w.second == layer || w.second == -1)) return false;
  return true;
}

int wait_stream(tg_context* ctx) {
  if (!ctx->comm) {
    TG_CUDA(cudaStreamSynchronize(ctx->stream));
    stream_idle(ctx);
    return TG_OK;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) {
      stream_idle(ctx);
      return TG_OK;
    }
    if (q != cudaErrorNotReady)
      return fail(TG_ERR_CUDA, "stream failed: %s", cudaGetErrorString(q));
    ncclResult_t ae = ncclSuccess;
    nccl().CommGetAsyncError(ctx->comm, &ae);
    const double ms = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
    if ((ae != ncclSuccess && ae != ncclInProgress) || ms > ctx->timeout_ms) {
      nccl().CommAbort(ctx->comm);
      ctx->comm = nullptr;
      ctx->world = 1;
      return fail(TG_ERR_COMM, "collective did not complete (%s, %.0f ms); communicator aborted",
                  ae != ncclSuccess ? nccl().GetErrorString(ae) : "timeout", ms);
    }
  }
}

// ------------------------------------------------ staging for host pointers

int arena_alloc(tg_context* ctx, size_t bytes, void** out) {
  bytes = (bytes + 255) & ~size_t(255);
  if (ctx->arena_off + bytes > ctx->arena_cap) {
    size_t n = ctx->arena_cap * 2;
    if (n < bytes * 2) n = bytes * 2;
    if (n < (size_t(1) << 20)) n = size_t(1) << 20;
    char* na = nullptr;
    TG_CUDA(cudaMalloc(&na, n));
    if (ctx->arena) ctx->graveyard.push_back(ctx->arena);
    ctx->arena = na;
    ctx->arena_cap = n;
    ctx->arena_off = 0;
  }
  *out = ctx->arena + ctx->arena_off;
  ctx->arena_off += bytes;
  return TG_OK;
}

// Inputs up to this size are packed; larger ones are copied on their own.
constexpr size_t kPackMaxBytes = size_t(1) << 20;


// Pinned host staging for packed inputs (linear; reset when the stream is
// idle, so a block is never rewritten while a copy from it may be pending).
int hpin_alloc(tg_context* ctx, size_t bytes, char** out) {
  bytes = (bytes + 255) & ~size_t(255);
  if (ctx->hpin_off + bytes > ctx->hpin_cap) {
    size_t n = ctx->hpin_cap * 2;
    if (n < bytes * 2) n = bytes * 2;
    if (n < (size_t(1) << 20)) n = size_t(1) << 20;
    char* nb = nullptr;
    TG_CUDA(cudaHostAlloc(&nb, n, cudaHostAllocDefault));
    void* nd = nullptr;
    if (cudaHostGetDevicePointer(&nd, nb, 0) != cudaSuccess) {
      cudaGetLastError();
      nd = nullptr;  // no device address: inputs move by copies only
    }
    if (ctx->hpin) ctx->hpin_old.push_back(ctx->hpin);
    ctx->hpin = nb;
    ctx->hpin_dev = static_cast<char*>(nd);
    ctx->hpin_cap = n;
    ctx->hpin_off = 0;
  }
  *out = ctx->hpin + ctx->hpin_off;
  ctx->hpin_off += bytes;
  return TG_OK;
}

// Where a pointer lives: device memory, page-locked host memory (with the
// device address of it), or pageable host memory.  One driver query.
struct PtrInfo {
  bool device = false;
  void* alias = nullptr;
};
PtrInfo classify(const void* p) {
  PtrInfo r;
  if (!p) return r;
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return r;
  }
  r.device = a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
  if (a.type == cudaMemoryTypeHost) r.alias = a.devicePointer;
  return r;
}

// A host input of the current call: gets its arena slot now; the bytes move
// at commit_inputs.
int pack_input(tg_context* ctx, const void* p, size_t bytes, void** dev) {
  if (ctx->capturing)
    return fail(TG_ERR_STATE, "host pointers cannot be used inside a graph capture");
  ctx->call_staged = true;
  void* d = nullptr;
  TG_TRY(arena_alloc(ctx, bytes, &d));
  ctx->pack.push_back({static_cast<char*>(d), static_cast<const char*>(p), bytes});
  *dev = d;
  return TG_OK;
}

// Moves the current call's host inputs to their arena slots: packed into
// page-locked staging on the CPU and moved by one copy-engine transfer per
// run of consecutive slots (measured faster end to end than a kernel that
// reads page-locked inputs over the host link).  Inside a batch the
// transfers run on a side stream that the compute stream waits for through
// an event, so no copy node sits between two kernels of the compute stream:
// a copy between kernels makes the next kernel wait for the previous one to
// end and for the copy, and loses its programmatic (PDL) overlap.  Arena
// slots are fresh within a batch and the stream is drained before they are
// reused, so the early copies overwrite nothing still in use.
// Inside a batch, small inputs (at most kStageKernelMax bytes in at most
// tg::kStageMaxRuns runs of the current pinned block) move by a staging
// kernel instead: copies on a side stream joined by an event still put the
// event wait between two kernels of the compute stream (the next kernel
// waits for the previous one to end), while a kernel keeps the chain
// kernel-to-kernel with its programmatic overlap.
constexpr size_t kStageKernelMax = 256 * 1024;

int commit_inputs(tg_context* ctx) {
  if (ctx->pack.empty()) return TG_OK;
  if (ctx->in_batch) {
    size_t total = 0;
    for (const auto& e : ctx->pack) total += (e.bytes + 255) & ~size_t(255);
    if (total <= kStageKernelMax) {
      std::vector<char*> stage(ctx->pack.size());
      for (size_t i = 0; i < ctx->pack.size(); ++i) {
        TG_TRY(hpin_alloc(ctx, ctx->pack[i].bytes, &stage[i]));
        std::memcpy(stage[i], ctx->pack[i].host, ctx->pack[i].bytes);
      }
      tg::StageParams sp{};
      bool ok = ctx->hpin_dev != nullptr;
      int total16 = 0;
      size_t i = 0;
      while (ok && i < ctx->pack.size()) {
        char* d0 = ctx->pack[i].dev;
        char* h0 = stage[i];
        size_t run = 0, j = i;
        for (; j < ctx->pack.size(); ++j) {
          if (ctx->pack[j].dev != d0 + run || stage[j] != h0 + run) break;
          run += (ctx->pack[j].bytes + 255) & ~size_t(255);
        }
        const size_t bytes = (size_t)(ctx->pack[j - 1].dev - d0) + ctx->pack[j - 1].bytes;
        if (sp.n_runs == tg::kStageMaxRuns || h0 < ctx->hpin ||
            h0 + bytes > ctx->hpin + ctx->hpin_cap) {
          ok = false;
          break;
        }
        // Slots are 256-byte aligned and padded: 16-byte words cover them.
        tg::StageRun& r = sp.run[sp.n_runs++];
        r.src = reinterpret_cast<const uint4*>(ctx->hpin_dev + (h0 - ctx->hpin));
        r.dst = reinterpret_cast<uint4*>(d0);
        r.n16 = (int)((bytes + 15) / 16);
        total16 += r.n16;
        i = j;
      }
      if (ok) {
        ctx->pack.clear();
        cudaError_t e = tg::launch_stage_copy(sp, total16, ctx->stream);
        if (e != cudaSuccess) return fail(TG_ERR_CUDA, "staging launch: %s", cudaGetErrorString(e));
        ctx->launches++;
        return TG_OK;
      }
      // Fall back to copies from the staging already filled.
      cudaStream_t cs = ctx->stream;
      if (!ctx->copy_stream) {
        TG_CUDA(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
        TG_CUDA(cudaEventCreateWithFlags(&ctx->copy_done, cudaEventDisableTiming));
      }
      cs = ctx->copy_stream;
      for (size_t k = 0; k < ctx->pack.size(); ++k)
        TG_CUDA(cudaMemcpyAsync(ctx->pack[k].dev, stage[k], ctx->pack[k].bytes,
                                cudaMemcpyHostToDevice, cs));
      ctx->pack.clear();
      TG_CUDA(cudaEventRecord(ctx->copy_done, cs));
      TG_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->copy_done, 0));
      return TG_OK;
    }
  }
  cudaStream_t cs = ctx->stream;
  if (ctx->in_batch) {
    if (!ctx->copy_stream) {
      TG_CUDA(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking));
      TG_CUDA(cudaEventCreateWithFlags(&ctx->copy_done, cudaEventDisableTiming));
    }
    cs = ctx->copy_stream;
  }
  std::vector<char*> stage(ctx->pack.size());
  for (size_t i = 0; i < ctx->pack.size(); ++i) {
    TG_TRY(hpin_alloc(ctx, ctx->pack[i].bytes, &stage[i]));
    std::memcpy(stage[i], ctx->pack[i].host, ctx->pack[i].bytes);
  }
  size_t i = 0;
  while (i < ctx->pack.size()) {
    char* d0 = ctx->pack[i].dev;
    char* h0 = stage[i];
    size_t run = 0, j = i;
    for (; j < ctx->pack.size(); ++j) {
      if (ctx->pack[j].dev != d0 + run || stage[j] != h0 + run) break;
      run += (ctx->pack[j].bytes + 255) & ~size_t(255);
    }
    const size_t bytes = (size_t)(ctx->pack[j - 1].dev - d0) + ctx->pack[j - 1].bytes;
    TG_CUDA(cudaMemcpyAsync(d0, h0, bytes, cudaMemcpyHostToDevice, cs));
    i = j;
  }
  ctx->pack.clear();
  if (cs != ctx->stream) {
    TG_CUDA(cudaEventRecord(ctx->copy_done, cs));
    TG_CUDA(cudaStreamWaitEvent(ctx->stream, ctx->copy_done, 0));
  }
  return TG_OK;
}

int stage_in(tg_context* ctx, const void* p, size_t bytes, const void** dev) {
  const PtrInfo pi = bytes ? classify(p) : PtrInfo{};
  if (!p || bytes == 0 || pi.device) {
    *dev = p;
    return TG_OK;
  }
  void* d = nullptr;
  if (bytes > kPackMaxBytes) {  // bulk data (cache rows): one copy of its own
    if (ctx->capturing)
      return fail(TG_ERR_STATE, "host pointers cannot be used inside a graph capture");
    ctx->call_staged = true;
    TG_TRY(commit_inputs(ctx));
    TG_TRY(arena_alloc(ctx, bytes, &d));
    TG_CUDA(cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, ctx->stream));
  } else {
    TG_TRY(pack_input(ctx, p, bytes, &d));
  }
  *dev = d;
  return TG_OK;
}

// Output (copy_in = false) or in/out (copy_in = true) buffer.  dev_in is
// what kernels read, *dev what they write.  Pinned host memory is written
// directly through its device alias when dev_in is given (the kernel takes
// separate in / out pointers); otherwise host buffers get an arena copy and
// a device->host copy when the call finishes.
int stage_out(tg_context* ctx, void* p, size_t bytes, bool copy_in, void** dev,
              const void** dev_in = nullptr) {
  const PtrInfo pi = bytes ? classify(p) : PtrInfo{};
  if (!p || bytes == 0 || pi.device) {
    *dev = p;
    if (dev_in) *dev_in = p;
    return TG_OK;
  }
  if (ctx->capturing)
    return fail(TG_ERR_STATE, "host pointers cannot be used inside a graph capture");
  ctx->call_staged = true;
  if (ctx->in_batch && pi.alias) {
    // Page-locked memory inside a batch: the kernels work on a device slot
    // (in place when copy_in) and the store kernel at tg_batch_end writes it
    // to the host, so that no kernel of the batch writes host memory.
    void* d = nullptr;
    if (copy_in) {
      TG_TRY(pack_input(ctx, p, bytes, &d));
    } else {
      TG_TRY(arena_alloc(ctx, bytes, &d));
    }
    ctx->dstores.push_back({p, pi.alias, d, bytes});
    *dev = d;
    if (dev_in) *dev_in = d;
    return TG_OK;
  }
  if (dev_in && pi.alias) {
    *dev = pi.alias;
    if (copy_in) {
      void* d = nullptr;
      TG_TRY(pack_input(ctx, p, bytes, &d));
      *dev_in = d;
    } else {
      *dev_in = pi.alias;
    }
    return TG_OK;
  }
  void* d = nullptr;
  if (copy_in) {
    TG_TRY(pack_input(ctx, p, bytes, &d));
  } else {
    TG_TRY(arena_alloc(ctx, bytes, &d));
  }
  ctx->pending.push_back({p, d, bytes});
  *dev = d;
  if (dev_in) *dev_in = d;
  return TG_OK;
}

// Moves the batch's deferred page-locked outputs to the host: one store
// kernel over an entry list in page-locked staging, or one copy per output
// when the staging has no device address.
int flush_deferred(tg_context* ctx) {
  if (ctx->dstores.empty()) return TG_OK;
  const size_t n = ctx->dstores.size();
  char* h = nullptr;
  if (n <= (1u << 20)) TG_TRY(hpin_alloc(ctx, n * sizeof(tg::StoreEntry), &h));
  if (h && ctx->hpin_dev) {
    tg::StoreEntry* e = reinterpret_cast<tg::StoreEntry*>(h);
    for (size_t i = 0; i < n; ++i)
      e[i] = tg::StoreEntry{ctx->dstores[i].alias, ctx->dstores[i].dev,
                            (unsigned long long)ctx->dstores[i].bytes};
    const tg::StoreEntry* de =
        reinterpret_cast<const tg::StoreEntry*>(ctx->hpin_dev + (h - ctx->hpin));
    ctx->dstores.clear();
    cudaError_t err = tg::launch_store_out(de, (int)n, ctx->stream);
    if (err != cudaSuccess)
      return fail(TG_ERR_CUDA, "output store launch: %s", cudaGetErrorString(err));
    ctx->launches++;
    return TG_OK;
  }
  for (const auto& d : ctx->dstores)
    TG_CUDA(cudaMemcpyAsync(d.host, d.dev, d.bytes, cudaMemcpyDeviceToHost, ctx->stream));
  ctx->dstores.clear();
  return TG_OK;
}

// Issues the device->host copies of staged outputs.  A call that moved host
// data waits for the stream (outside a batch) so that its host outputs are
// valid on return; a call on device pointers only stays asynchronous, like
// any stream-ordered CUDA work, and device-side errors surface at the next
// tg_synchronize / tg_batch_end.
int finish_call(tg_context* ctx) {
  TG_TRY(commit_inputs(ctx));
  const bool staged = ctx->call_staged;
  ctx->call_staged = false;
  for (const PendingCopy& c : ctx->pending)
    TG_CUDA(cudaMemcpyAsync(c.host, c.dev, c.bytes, cudaMemcpyDeviceToHost, ctx->stream));
  ctx->pending.clear();
  if (ctx->in_batch || !staged) return TG_OK;
  const bool queued = queue_error_read(ctx);
  TG_TRY(wait_stream(ctx));
  ctx->arena_off = 0;
  ctx->hpin_off = 0;
  free_graveyard(ctx);
  return check_device_error(ctx, queued);
}

// ------------------------------------------------ host-array mirrors

Region* find_region(tg_context* ctx, const char* p, size_t bytes) {
  auto it = ctx->regions.upper_bound(reinterpret_cast<uintptr_t>(p));
  if (it == ctx->regions.begin()) return nullptr;
  --it;
  Region& r = it->second;
  if (r.host <= p && p + bytes <= r.host + r.bytes) return &r;
  return nullptr;
}

int make_fresh(tg_context* ctx, Region& r) {
  if (r.fresh || (r.flags & TG_REGION_DEVICE_OWNED) || r.dirty_hi > r.dirty_lo)
    return TG_OK;
  TG_CUDA(cudaMemcpyAsync(r.dev, r.host, r.bytes, cudaMemcpyHostToDevice, ctx->stream));
  r.fresh = true;
  return TG_OK;
}

// Creates a mirror for [p, p+bytes), absorbing any mirrors it overlaps: the
// new device copy starts as the host contents, then every absorbed mirror
// whose device copy is newer (written or device-owned) is copied over it.
// Transient mirrors (made by ops for unregistered host arrays) live in the
// staging arena until the batch ends; registered ones own their memory.
int create_region(tg_context* ctx, char* p, size_t bytes, int flags, bool transient,
                  Region** out) {
  if (ctx->capturing)
    return fail(TG_ERR_STATE, "host arrays cannot be used inside a graph capture");
  char* lo = p;
  char* hi = p + bytes;
  std::vector<uintptr_t> absorbed;
  for (auto& kv : ctx->regions) {
    Region& r = kv.second;
    if (r.host < hi && p < r.host + r.bytes) {
      if (transient && !r.transient)
        return fail(TG_ERR_INVALID_ARG,
                    "host range [%p, +%zu) straddles the registered array at %p (+%zu)",
                    (void*)p, bytes, (void*)r.host, r.bytes);
      absorbed.push_back(kv.first);
      if (r.host < lo) lo = r.host;
      if (r.host + r.bytes > hi) hi = r.host + r.bytes;
      flags |= r.flags;
    }
  }
  Region nr;
  nr.host = lo;
  nr.bytes = (size_t)(hi - lo);
  nr.flags = flags;
  nr.transient = transient;
  if (transient) {
    void* d = nullptr;
    TG_TRY(arena_alloc(ctx, nr.bytes, &d));
    nr.dev = static_cast<char*>(d);
  } else {
    TG_CUDA(cudaMalloc(&nr.dev, nr.bytes));
  }
  TG_CUDA(cudaMemcpyAsync(nr.dev, nr.host, nr.bytes, cudaMemcpyHostToDevice, ctx->stream));
  nr.fresh = true;
  for (uintptr_t key : absorbed) {
    Region& r = ctx->regions[key];
    const bool dev_newer = (r.flags & TG_REGION_DEVICE_OWNED) || r.dirty_hi > r.dirty_lo;
    if (dev_newer)
      TG_CUDA(cudaMemcpyAsync(nr.dev + (r.host - nr.host), r.dev, r.bytes,
                              cudaMemcpyDeviceToDevice, ctx->stream));
    if (r.dirty_hi > r.dirty_lo) {
      const size_t a = (size_t)(r.host - nr.host) + r.dirty_lo;
      const size_t b = (size_t)(r.host - nr.host) + r.dirty_hi;
      if (nr.dirty_hi <= nr.dirty_lo) {
        nr.dirty_lo = a;
        nr.dirty_hi = b;
      } else {
        if (a < nr.dirty_lo) nr.dirty_lo = a;
        if (b > nr.dirty_hi) nr.dirty_hi = b;
      }
    }
    if (!r.transient) ctx->graveyard.push_back(r.dev);
    ctx->regions.erase(key);
  }
  auto res = ctx->regions.emplace(reinterpret_cast<uintptr_t>(nr.host), nr);
  *out = &res.first->second;
  return TG_OK;
}

// Creates the mirror of a host range if none covers it yet.  Compat ops
// call this for every argument before resolving any, so that a merge of
// overlapping mirrors cannot move an address that was already handed out.
int ensure_region(tg_context* ctx, const void* p, size_t bytes) {
  if (!p) return fail(TG_ERR_INVALID_ARG, "null pointer argument");
  if (is_device_ptr(p)) return TG_OK;
  char* hp = const_cast<char*>(static_cast<const char*>(p));
  if (find_region(ctx, hp, bytes)) return TG_OK;
  Region* r = nullptr;
  return create_region(ctx, hp, bytes, TG_REGION_MIRROR, true, &r);
}

// Device address for a compat-op argument.  write: the op writes the range.
int resolve(tg_context* ctx, const void* p, size_t bytes, bool write, char** dev) {
  if (!p) return fail(TG_ERR_INVALID_ARG, "null pointer argument");
  if (is_device_ptr(p)) {
    *dev = const_cast<char*>(static_cast<const char*>(p));
    return TG_OK;
  }
  char* hp = const_cast<char*>(static_cast<const char*>(p));
  Region* r = find_region(ctx, hp, bytes);
  if (!r) TG_TRY(create_region(ctx, hp, bytes, TG_REGION_MIRROR, true, &r));
  ctx->call_staged = true;
  TG_TRY(make_fresh(ctx, *r));
  const size_t off = (size_t)(hp - r->host);
  if (write && !(r->flags & TG_REGION_DEVICE_OWNED)) {
    if (r->dirty_hi <= r->dirty_lo) {
      r->dirty_lo = off;
      r->dirty_hi = off + bytes;
    } else {
      if (off < r->dirty_lo) r->dirty_lo = off;
      if (off + bytes > r->dirty_hi) r->dirty_hi = off + bytes;
    }
  }
  *dev = r->dev + off;
  return TG_OK;
}

// metal_batch_end analogue for mirrors: copy back written ranges.
int flush_regions(tg_context* ctx) {
  for (auto& kv : ctx->regions) {
    Region& r = kv.second;
    if (r.dirty_hi > r.dirty_lo)
      TG_CUDA(cudaMemcpyAsync(r.host + r.dirty_lo, r.dev + r.dirty_lo, r.dirty_hi - r.dirty_lo,
                              cudaMemcpyDeviceToHost, ctx->stream));
  }
  const bool queued = queue_error_read(ctx);
  TG_TRY(wait_stream(ctx));
  for (auto it = ctx->regions.begin(); it != ctx->regions.end();) {
    if (it->second.transient) {
      it = ctx->regions.erase(it);
    } else {
      it->second.dirty_lo = it->second.dirty_hi = 0;
      it->second.fresh = false;
      ++it;
    }
  }
  ctx->arena_off = 0;
  ctx->hpin_off = 0;
  ctx->call_staged = false;
  free_graveyard(ctx);
  return check_device_error(ctx, queued);
}

// End of a compat op: outside a batch, host arrays are written back and the
// stream is waited on; an op on device pointers only stays asynchronous.
int finish_compat(tg_context* ctx) {
  if (ctx->in_batch) return TG_OK;
  if (!ctx->call_staged) return TG_OK;
  return flush_regions(ctx);
}

// ------------------------------------------------ RoPE tables

// cos/sin for positions [0, len) exactly as apply_rope computes them
// (tmac_gguf.cpp:993-996): theta = 1/powf(base, (float)d/head_dim),
// freq = pos*theta, cosf/sinf -- evaluated here with the host libm so the
// device rotation reproduces the reference bit for bit.
int get_table(tg_context* ctx, float base, int head_dim, int need_len, RopeTable** out) {
  uint32_t bits;
  std::memcpy(&bits, &base, 4);
  RopeTable* t = nullptr;
  for (RopeTable& x : ctx->tables)
    if (x.base_bits == bits && x.head_dim == head_dim) t = &x;
  if (t && t->len >= need_len) {
    *out = t;
    return TG_OK;
  }
  if (ctx->capturing)
    return fail(TG_ERR_STATE, "RoPE table for position %d must exist before graph capture",
                need_len - 1);
  int len = 4096;
  while (len < need_len) len *= 2;
  const int half = head_dim / 2;
  std::vector<float> theta(half);
  for (int j = 0; j < half; ++j) theta[j] = 1.0f / powf(base, (float)(2 * j) / head_dim);
  std::vector<float> h((size_t)len * head_dim);
  for (int pos = 0; pos < len; ++pos) {
    float* row = h.data() + (size_t)pos * head_dim;
    for (int j = 0; j < half; ++j) {
      const float freq = pos * theta[j];
      row[2 * j] = cosf(freq);
      row[2 * j + 1] = sinf(freq);
    }
  }
  float* d = nullptr;
  TG_CUDA(cudaMalloc(&d, h.size() * sizeof(float)));
  TG_CUDA(cudaMemcpy(d, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice));
  if (!t) {
    ctx->tables.push_back(RopeTable());
    t = &ctx->tables.back();
    t->base_bits = bits;
    t->head_dim = head_dim;
  } else {
    ctx->graveyard.push_back(t->d);
  }
  t->len = len;
  t->d = d;
  *out = t;
  return TG_OK;
}

// The kernels move q, k and outputs as float2 / float4: device pointers must
// be 8-byte aligned (host pointers are staged into aligned buffers).
int check_align8(const void* p, const char* what) {
  if (p && (reinterpret_cast<uintptr_t>(p) & 7))
    return fail(TG_ERR_INVALID_ARG, "%s must be 8-byte aligned", what);
  return TG_OK;
}

int check_shape(int n_head, int n_kv, int hd) {
  if (n_head <= 0 || n_kv <= 0 || hd <= 0 || hd % 2 || hd > 128 || n_head % n_kv)
    return fail(TG_ERR_INVALID_ARG, "unsupported shape n_head=%d n_kv_head=%d head_dim=%d", n_head,
                n_kv, hd);
  if (n_head * hd > 4096 || n_kv * hd > 1024 || (n_kv * hd) % 8)
    return fail(TG_ERR_INVALID_ARG, "shape too large n_head=%d n_kv_head=%d head_dim=%d", n_head,
                n_kv, hd);
  return TG_OK;
}

bool mma_eligible(const tg_kv_cache* kv) {
  return kv->tmap_ok && kv->d.dtype == TG_DTYPE_BF16 && kv->d.head_dim == 64 &&
         (kv->d.n_kv_head == 1 || kv->d.n_kv_head == 2 || kv->d.n_kv_head == 4) &&
         kv->d.n_head / kv->d.n_kv_head <= 8;
}

int generic_grid(tg_context* ctx, int dtype, size_t smem) {
  int per_sm = tg::decode_generic_blocks_per_sm(dtype, smem);
  if (per_sm > 4) per_sm = 4;
  return ctx->num_sms * per_sm;
}

// CUDA-event timing of one launch of a profiled kernel class
// (tg_profile_enable): a start event before the launch and, through
// prof_end, a stop event after it.  Inside a capture the records become
// event nodes of the graph, re-recorded by every replay.
int prof_begin(tg_context* ctx, int kind, cudaEvent_t* ev_stop) {
  *ev_stop = nullptr;
  if (!(ctx->prof_on & kind)) return TG_OK;
  while (ctx->prof_ev.size() < ctx->prof_used + 2) {
    cudaEvent_t ev;
    TG_CUDA(cudaEventCreate(&ev));
    ctx->prof_ev.push_back(ev);
  }
  TG_CUDA(cudaEventRecordWithFlags(ctx->prof_ev[ctx->prof_used], ctx->stream,
                                   ctx->capturing ? cudaEventRecordExternal : 0));
  *ev_stop = ctx->prof_ev[ctx->prof_used + 1];
  ctx->prof_used += 2;
  return TG_OK;
}

int prof_end(tg_context* ctx, cudaEvent_t ev_stop) {
  if (ev_stop)
    TG_CUDA(cudaEventRecordWithFlags(ev_stop, ctx->stream,
                                     ctx->capturing ? cudaEventRecordExternal : 0));
  return TG_OK;
}

// Caches the one-CTA-per-(sequence, KV head) kernel takes: capacity at most
// kSmallMaxRows, head_dim 64, at most 8 query heads per KV head, whole cache.
bool small_eligible(const tg_kv_cache* kv) {
  const tg_kv_desc& d = kv->d;
  const int group = d.n_head / d.n_kv_head;
  return d.head_dim == 64 && group <= 8 && d.max_ctx <= tg::kSmallMaxRows &&
         d.shard_start == 0 && tg::decode_small_smem(group, d.max_ctx, 1) <= 227 * 1024;
}

// CTAs per (sequence, KV head) of the short-cache kernel: the largest of 8,
// 4, 2, 1 that keeps the launch within two CTAs per SM and gives every CTA
// at least 16 rows of a full cache (measured at config 2, 128 items: the
// 2-way split 0.38 ms per step, none 0.48 ms).
int small_split(const tg_context* ctx, const tg_kv_cache* kv, int B) {
  const long long items = (long long)B * kv->d.n_kv_head;
  int c = 8;
  while (c > 1 && (items * c > 2LL * ctx->num_sms || kv->d.max_ctx < 16 * c)) c >>= 1;
  return c;
}

// Core decode launch on device pointers.  mode 0 writes `out`; mode 1
// writes per-sequence records to ctx->records.
int run_decode(tg_context* ctx, const tg_kv_cache* kv, int layer, int B, const float* q,
               const int* past_dev, int past_scalar, float* out, int mode) {
  TG_TRY(commit_inputs(ctx));
  const tg_kv_desc& d = kv->d;
  TG_TRY(check_align8(q, "q"));
  TG_TRY(check_align8(out, "out"));
  const int rf = tg::record_floats(d.n_head, d.head_dim);
  tg::DecodeParams p{};
  p.q = q;
  p.out = out;
  p.past_len = past_dev;
  p.past_len_scalar = past_scalar;
  p.k = static_cast<const char*>(kv->k) + (size_t)layer * kv->layer_elems * kv->esize;
  p.v = static_cast<const char*>(kv->v) + (size_t)layer * kv->layer_elems * kv->esize;
  p.row0 = (long long)layer * d.n_seqs * d.max_ctx;
  p.B = B;
  p.n_head = d.n_head;
  p.n_kv = d.n_kv_head;
  p.head_dim = d.head_dim;
  p.group = d.n_head / d.n_kv_head;
  p.max_ctx = d.max_ctx;
  p.shard_start = d.shard_start;
  p.scale_log2 = kLog2e / sqrtf((float)d.head_dim);
  p.mode = mode;
  p.err = ctx->d_err;
  p.aligned16 = ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) % 16 == 0 &&
                 (kv->row_elems * kv->esize) % 16 == 0)
                    ? 1
                    : 0;

  // Short caches: one CTA per (sequence, KV head) does the whole attention
  // (no split, no merge launch).  The cache capacity decides, so the choice
  // holds for any positions, also inside a graph capture.
  if (mode == 0 && small_eligible(kv)) {
    p.split = small_split(ctx, kv, B);
    cudaEvent_t ev_small = nullptr;
    TG_TRY(prof_begin(ctx, TG_PROFILE_ATTENTION, &ev_small));
    cudaError_t e = tg::launch_decode_small(p, d.dtype, ctx->stream);
    if (e != cudaSuccess) return fail(TG_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
    ctx->launches++;
    return prof_end(ctx, ev_small);
  }
  const bool mma = mma_eligible(kv);
  int grid;
  size_t smem;
  if (mma) {
    smem = tg::decode_mma_smem(d.n_kv_head, B);
    grid = ctx->num_sms;
  } else {
    smem = tg::decode_generic_smem(B, d.n_head, d.n_kv_head, d.head_dim);
    grid = generic_grid(ctx, d.dtype, smem);
  }
  if (smem > 227 * 1024)
    return fail(TG_ERR_INVALID_ARG,
                "%d sequences of shape %d/%d/%d need %zu KB of shared memory (at most 227)", B,
                d.n_head, d.n_kv_head, d.head_dim, (smem + 1023) / 1024);
  TG_TRY(ensure_buf(ctx, &ctx->part, &ctx->part_cap, (size_t)2 * grid * rf));
  TG_TRY(ensure_buf(ctx, &ctx->sched, &ctx->sched_cap, (size_t)B + 1));
  if (mode == 1) TG_TRY(ensure_buf(ctx, &ctx->records, &ctx->rec_cap, (size_t)B * rf));
  p.part = ctx->part;
  p.sched = ctx->sched;
  p.records = ctx->records;

  cudaEvent_t ev_stop = nullptr;
  TG_TRY(prof_begin(ctx, TG_PROFILE_ATTENTION, &ev_stop));
  cudaError_t e = mma ? tg::launch_decode_mma(kv->tmk, kv->tmv, p, grid, ctx->stream)
                      : tg::launch_decode_generic(p, d.dtype, grid, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  TG_TRY(prof_end(ctx, ev_stop));

  tg::MergeParams m{};
  m.part = ctx->part;
  m.sched = ctx->sched;
  m.out = out;
  m.records = ctx->records;
  m.B = B;
  m.n_head = d.n_head;
  m.head_dim = d.head_dim;
  m.G = grid;
  m.mode = mode;
  e = tg::launch_merge(m, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "merge launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  return TG_OK;
}

// Short caches: RoPE of q and k, the new row's cache-write and attention in
// one launch of the short-cache kernel (q and k rotated in place).
int run_small_step(tg_context* ctx, const tg_kv_cache* kv, int layer, int B, float* q, float* k,
                   const float* v, const int* pos_dev, float* out, float* q_wb = nullptr,
                   float* k_wb = nullptr) {
  TG_TRY(commit_inputs(ctx));
  const tg_kv_desc& d = kv->d;
  TG_TRY(check_align8(q, "q"));
  TG_TRY(check_align8(k, "k_new"));
  TG_TRY(check_align8(out, "out"));
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, d.rope_base, d.head_dim, kv->global_ctx, &t));
  tg::DecodeParams p{};
  p.q = q;
  p.out = out;
  p.past_len = pos_dev;
  p.k = static_cast<const char*>(kv->k) + (size_t)layer * kv->layer_elems * kv->esize;
  p.v = static_cast<const char*>(kv->v) + (size_t)layer * kv->layer_elems * kv->esize;
  p.B = B;
  p.n_head = d.n_head;
  p.n_kv = d.n_kv_head;
  p.head_dim = d.head_dim;
  p.group = d.n_head / d.n_kv_head;
  p.max_ctx = d.max_ctx;
  p.shard_start = 0;
  p.scale_log2 = kLog2e / sqrtf((float)d.head_dim);
  p.mode = 0;
  p.err = ctx->d_err;
  p.aligned16 = ((reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) % 16 == 0 &&
                 (kv->row_elems * kv->esize) % 16 == 0)
                    ? 1
                    : 0;
  p.rope = 1;
  p.q_io = q;
  p.k_io = k;
  p.q_wb = q_wb;
  p.k_wb = k_wb;
  p.v_new = v;
  p.cs = t->d;
  p.table_len = kv->global_ctx;
  p.k_cache = const_cast<void*>(p.k);
  p.v_cache = const_cast<void*>(p.v);
  p.split = small_split(ctx, kv, B);
  cudaEvent_t ev = nullptr;
  TG_TRY(prof_begin(ctx, TG_PROFILE_ATTENTION, &ev));
  cudaError_t e = tg::launch_decode_small(p, d.dtype, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "decode launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  note_pdl_write(ctx, kv, layer);
  return prof_end(ctx, ev);
}

int run_rope(tg_context* ctx, const tg_kv_cache* kv, int layer, int B, float* q, float* k,
             const float* v, const int* pos_dev) {
  TG_TRY(commit_inputs(ctx));
  const tg_kv_desc& d = kv->d;
  TG_TRY(check_align8(q, "q"));
  TG_TRY(check_align8(k, "k_new"));
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, d.rope_base, d.head_dim, kv->global_ctx, &t));
  tg::RopeParams rp{};
  rp.q = q;
  rp.k = k;
  rp.v = v;
  rp.pos = pos_dev;
  rp.cs = t->d;
  rp.table_len = kv->global_ctx;
  rp.k_cache = static_cast<char*>(kv->k) + (size_t)layer * kv->layer_elems * kv->esize;
  rp.v_cache = static_cast<char*>(kv->v) + (size_t)layer * kv->layer_elems * kv->esize;
  rp.B = B;
  rp.n_head = d.n_head;
  rp.n_kv = d.n_kv_head;
  rp.head_dim = d.head_dim;
  rp.max_ctx = d.max_ctx;
  rp.shard_start = d.shard_start;
  rp.dtype = d.dtype;
  rp.err = ctx->d_err;
  cudaError_t e = tg::launch_rope(rp, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "rope launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  note_pdl_write(ctx, kv, layer);
  return TG_OK;
}

// All-gather `bytes` per rank through NCCL on the context stream and wait.
int nccl_allgather_bytes(tg_context* ctx, const void* dsend, void* drecv, size_t bytes) {
  ncclResult_t r = nccl().AllGather(dsend, drecv, bytes, ncclUint8, ctx->comm, ctx->stream);
  if (r == ncclInProgress) {
    const auto t0 = std::chrono::steady_clock::now();
    do {
      nccl().CommGetAsyncError(ctx->comm, &r);
      const double ms = std::chrono::duration<double, std::milli>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
      if (r == ncclInProgress && ms > ctx->timeout_ms) break;
    } while (r == ncclInProgress);
  }
  if (r != ncclSuccess)
    return fail(TG_ERR_COMM, "ncclAllGather: %s",
                r == ncclInProgress ? "timeout" : nccl().GetErrorString(r));
  return wait_stream(ctx);
}

void p2p_release(tg_context* ctx) {
  if (!ctx->p2p_ready && !ctx->xchg_local) return;
  cudaStreamSynchronize(ctx->stream);
  for (int r = 0; r < tg::kMaxPeers; ++r) {
    if (ctx->xchg_peer[r]) cudaIpcCloseMemHandle(ctx->xchg_peer[r]);
    ctx->xchg_peer[r] = nullptr;
  }
  cudaFree(ctx->xchg_local);
  cudaFree(ctx->xchg_ctl);
  ctx->xchg_local = nullptr;
  ctx->xchg_ctl = nullptr;
  ctx->p2p_ready = false;
  ctx->p2p_bcap = 0;
}

// Collective: every rank of the communicator calls this with the same B.
// Allocates this GPU's receive words [2][world][B][n_head][kXchgWords],
// shares their IPC handle over NCCL, maps every peer's, and agrees with all
// ranks whether peer memory can be used (otherwise all ranks use the NCCL
// path).
int ensure_p2p(tg_context* ctx, int B, int n_head, int rf) {
  if (ctx->p2p_failed) return TG_ERR_UNSUPPORTED;
  if (ctx->p2p_ready && B <= ctx->p2p_bcap && rf == ctx->p2p_rf && n_head == ctx->p2p_heads)
    return TG_OK;
  if (ctx->capturing)
    return fail(TG_ERR_STATE, "peer buffers must be set up before graph capture");
  if (ctx->world > tg::kMaxPeers) {
    ctx->p2p_failed = true;
    return TG_ERR_UNSUPPORTED;
  }
  TG_TRY(wait_stream(ctx));
  p2p_release(ctx);
  const int W = ctx->world;
  const size_t xbytes = (size_t)2 * W * B * n_head * tg::kXchgWords * sizeof(unsigned long long);
  TG_CUDA(cudaMalloc(&ctx->xchg_local, xbytes));
  TG_CUDA(cudaMalloc(&ctx->xchg_ctl, 64 * sizeof(unsigned)));
  TG_CUDA(cudaMemsetAsync(ctx->xchg_local, 0, xbytes, ctx->stream));
  TG_CUDA(cudaMemsetAsync(ctx->xchg_ctl, 0, 64 * sizeof(unsigned), ctx->stream));
  if (!ctx->nccl_stage) TG_CUDA(cudaMalloc(&ctx->nccl_stage, 2 * 128 * (tg::kMaxPeers + 1)));
  cudaIpcMemHandle_t hx;
  TG_CUDA(cudaIpcGetMemHandle(&hx, ctx->xchg_local));
  const size_t hb = sizeof(hx);
  TG_CUDA(cudaMemcpyAsync(ctx->nccl_stage, &hx, hb, cudaMemcpyHostToDevice, ctx->stream));
  TG_TRY(nccl_allgather_bytes(ctx, ctx->nccl_stage, ctx->nccl_stage + hb, hb));
  std::vector<unsigned char> all((size_t)W * hb);
  TG_CUDA(cudaMemcpy(all.data(), ctx->nccl_stage + hb, all.size(), cudaMemcpyDeviceToHost));
  unsigned char ok = 1;
  for (int r = 0; r < W && ok; ++r) {
    if (r == ctx->rank) continue;
    cudaIpcMemHandle_t pr;
    std::memcpy(&pr, all.data() + r * hb, sizeof(pr));
    void* a = nullptr;
    if (cudaIpcOpenMemHandle(&a, pr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    }
    ctx->xchg_peer[r] = static_cast<unsigned long long*>(a);
  }
  // Consensus: peer memory only if every rank mapped every peer.  This
  // exchange also orders every rank's zeroing before any peer store.
  TG_CUDA(cudaMemcpyAsync(ctx->nccl_stage, &ok, 1, cudaMemcpyHostToDevice, ctx->stream));
  TG_TRY(nccl_allgather_bytes(ctx, ctx->nccl_stage, ctx->nccl_stage + 128, 1));
  std::vector<unsigned char> oks(W);
  TG_CUDA(cudaMemcpy(oks.data(), ctx->nccl_stage + 128, W, cudaMemcpyDeviceToHost));
  for (int r = 0; r < W; ++r)
    if (!oks[r]) ok = 0;
  if (!ok) {
    p2p_release(ctx);
    ctx->p2p_failed = true;
    return TG_ERR_UNSUPPORTED;
  }
  ctx->p2p_ready = true;
  ctx->p2p_bcap = B;
  ctx->p2p_rf = rf;
  ctx->p2p_heads = n_head;
  return TG_OK;
}

// A short shard: at most 16 tiles of 64 rows per SM on average, so that a
// CTA can load a good part of its tiles before its grid-dependency wait.
bool short_shard(const tg_context* ctx, const tg_kv_cache* kv, int B) {
  return (long long)B * ((kv->d.max_ctx + 63) / 64) <= 16LL * ctx->num_sms;
}

// K/V ring per CTA of the bf16 decode: 128 KB unless tg_set_decode_tuning
// asks for the deep one (192 KB, when its shared memory fits).  Measured on
// B200s at 4 x 131072 rows: on one GPU 46.2 us per layer with 128 KB against
// 47.4 with 192; split over 8 GPUs 192 KB was 1-4 % slower too.
int fused_ring(const tg_context* ctx, const tg_kv_cache* kv, int B) {
  (void)ctx;
  if (g_decode_ring == tg::kFusedRingDeep &&
      tg::decode_fused_smem(kv->d.n_kv_head, tg::kFusedRingDeep, B) <= 227 * 1024)
    return tg::kFusedRingDeep;
  return tg::kFusedRing;
}

// The decode step on the tensor-core path (bf16 cache): the decode kernel
// and, PDL-chained behind it, the merge kernel.  mode 0: normalised output;
// 1: per-sequence records to `records`; 2: exchange with the other GPUs of
// the communicator (peer memory, set up by ensure_p2p) and output.
// preload: the caller checked with preload_allowed (before any launch of its
// own that writes the new rows) that the cache rows may be loaded before
// the decode kernel's grid-dependency wait.
int run_fused(tg_context* ctx, const tg_kv_cache* kv, int layer, int B, const float* q_in,
              float* q_out, float* k_io, const float* v_new, const int* pos, float* out,
              float* records, int mode, bool rope, bool new_row, float* k_out, bool preload) {
  TG_TRY(commit_inputs(ctx));
  const tg_kv_desc& d = kv->d;
  TG_TRY(check_align8(q_in, "q"));
  TG_TRY(check_align8(q_out, "q"));
  TG_TRY(check_align8(k_io, "k_new"));
  TG_TRY(check_align8(k_out, "k_new"));
  TG_TRY(check_align8(out, "out"));
  const int rf = tg::record_floats(d.n_head, d.head_dim);
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, d.rope_base, d.head_dim, kv->global_ctx, &t));
  const int grid = ctx->num_sms;
  const int ring = fused_ring(ctx, kv, B);
  const size_t smem = tg::decode_fused_smem(d.n_kv_head, ring, B);
  if (smem > 227 * 1024)
    return fail(TG_ERR_INVALID_ARG, "batch of %d sequences exceeds the shared-memory schedule", B);
  TG_TRY(check_align8(records, "records"));
  TG_TRY(ensure_buf(ctx, &ctx->part, &ctx->part_cap, (size_t)2 * grid * rf));
  TG_TRY(ensure_buf(ctx, &ctx->sched, &ctx->sched_cap, (size_t)B + 1));
  if (mode == 2) {  // records of sequences finished inside one CTA
    TG_TRY(ensure_buf(ctx, &ctx->records, &ctx->rec_cap, (size_t)B * rf));
    records = ctx->records;
  }
  tg::FusedParams p{};
  p.q_in = q_in;
  p.q_out = q_out;
  p.k_io = k_io;
  p.k_out = k_out ? k_out : k_io;
  p.v_new = v_new;
  p.pos = pos;
  p.cs = t->d;
  p.table_len = kv->global_ctx;
  p.kc_layer = reinterpret_cast<uint16_t*>(static_cast<char*>(kv->k) +
                                           (size_t)layer * kv->layer_elems * kv->esize);
  p.vc_layer = reinterpret_cast<uint16_t*>(static_cast<char*>(kv->v) +
                                           (size_t)layer * kv->layer_elems * kv->esize);
  p.out = out;
  p.records = records;
  p.part = ctx->part;
  p.sched = ctx->sched;
  p.err = ctx->d_err;
  p.row0 = (long long)layer * d.n_seqs * d.max_ctx;
  p.B = B;
  p.n_head = d.n_head;
  p.n_kv = d.n_kv_head;
  p.group = d.n_head / d.n_kv_head;
  p.max_ctx = d.max_ctx;
  p.shard_start = d.shard_start;
  p.scale_log2 = kLog2e / sqrtf((float)d.head_dim);
  p.mode = mode;
  p.rope = rope ? 1 : 0;
  p.new_row = new_row ? 1 : 0;
  p.grid = grid;
  // Merge kernel: one CTA per (sequence, head); in mode 2 a persistent grid
  // that stays resident beside the decode kernel (its CTAs wait on peers).
  const int items = B * d.n_head;
  const int mgrid = mode == 2 ? std::min(items, 2 * ctx->num_sms) : items;
  // Wide items (256 threads) when they are few; 64 threads when there are
  // more items than the GPU holds wide CTAs at once.
  const int mgroups = (mode == 2 || items <= 2 * ctx->num_sms) ? tg::kMergeGroupsWide : 1;
  // The previous layer's merge kernel is long-lived in these cases (few wide
  // items, or the peer exchange), which leaves the next decode kernel time
  // to prefetch its first tiles into L2 before its wait returns (measured:
  // -0.8 us per layer at 4 x 16384..131072 rows, +4 us at 256 x 4096).
  p.prefetch = mgroups == tg::kMergeGroupsWide ? 1 : 0;
  // Tile loads before the wait, when tg_set_decode_tuning allows them, on
  // short shards only: on long ones they only compete with the previous
  // layer's merge for memory (+1.2 us per layer at 4 x 131072 rows on one
  // GPU).  Off by default: measured 1-2 us per layer slower on the split
  // 8-GPU shards too.
  p.preload = (preload && short_shard(ctx, kv, B)) ? 1 : 0;
  p.wait_ns = ctx->wait_ns;
  if (mode == 2) {
    p.world = ctx->world;
    p.rank = ctx->rank;
    p.b_cap = ctx->p2p_bcap;
    p.xchg_local = ctx->xchg_local;
    for (int r = 0; r < ctx->world; ++r) p.xchg_peer[r] = ctx->xchg_peer[r];
    p.epoch = ctx->xchg_ctl;
  }
  if ((ctx->prof_on & TG_PROFILE_STAMPS) && ctx->stamps && ctx->stamp_used < ctx->stamp_cap) {
    p.stamps = ctx->stamps +
               (size_t)ctx->stamp_used * tg::kStampRowsPerSm * ctx->num_sms * tg::kStampsPerCta;
    ctx->stamp_used++;
  }
  cudaEvent_t ev_stop = nullptr;
  TG_TRY(prof_begin(ctx, TG_PROFILE_ATTENTION, &ev_stop));
  cudaError_t e = tg::launch_decode_fused(kv->tmk, kv->tmv, p, ring, grid, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "fused decode launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  if (new_row) note_pdl_write(ctx, kv, layer);
  TG_TRY(prof_end(ctx, ev_stop));
  e = tg::launch_merge_exchange(p, mgrid, mgroups, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "merge launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  return TG_OK;
}

// ------------------------------------------------ Q/K/V projection

size_t qrow_bytes(int wtype, int cols) {
  return (size_t)(cols / 32) * (size_t)tg::wtype_block_bytes(wtype);
}

int check_qkv_cols(int cols) {
  if (cols <= 0 || cols % 32)
    return fail(TG_ERR_INVALID_ARG, "cols %d must be a positive multiple of 32", cols);
  if (cols > tg::qkv_max_cols())
    return fail(TG_ERR_INVALID_ARG, "cols %d exceeds the projection kernel's %d", cols,
                tg::qkv_max_cols());
  return TG_OK;
}

int check_wtype(int t, const char* what) {
  if (t != TG_WTYPE_Q5_0 && t != TG_WTYPE_Q8_0)
    return fail(TG_ERR_UNSUPPORTED, "%s: weight type %d (only Q5_0 = 6 and Q8_0 = 8)", what, t);
  return TG_OK;
}

// Blocks hold 16-bit fields: weight arrays must be 2-byte aligned.
int check_align2(const void* p, const char* what) {
  if (p && (reinterpret_cast<uintptr_t>(p) & 1))
    return fail(TG_ERR_INVALID_ARG, "%s must be 2-byte aligned", what);
  return TG_OK;
}

// Device address of a weight or bias array: device pointers pass through,
// registered host arrays use their mirror, other host arrays are staged
// for this call.
int weight_ptr(tg_context* ctx, const void* p, size_t bytes, const void** dev) {
  if (!p) {
    *dev = nullptr;
    return TG_OK;
  }
  if (is_device_ptr(p)) {
    *dev = p;
    return TG_OK;
  }
  if (find_region(ctx, static_cast<const char*>(p), bytes)) {
    char* d = nullptr;
    TG_TRY(resolve(ctx, p, bytes, false, &d));
    *dev = d;
    return TG_OK;
  }
  return stage_in(ctx, p, bytes, dev);
}

int run_qkv(tg_context* ctx, tg::QkvParams& p) {
  TG_TRY(commit_inputs(ctx));
  const int per = tg::qkv_rows_per_cta(p.B, p.cols);
  for (int m = 0; m < 3; ++m) p.tiles[m] = (p.rows[m] + per - 1) / per;
  p.err = ctx->d_err;
  cudaEvent_t ev_stop = nullptr;
  TG_TRY(prof_begin(ctx, TG_PROFILE_PROJECTION, &ev_stop));
  cudaError_t e = tg::launch_qkv(p, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "qkv launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  return prof_end(ctx, ev_stop);
}

// Mode-1 projection of one layer on device x / pos: bias, RoPE, cache-write,
// rotated q into dq_out.
int qkv_layer_core(tg_context* ctx, const tg_kv_cache* kv, int layer, int n,
                   const tg_qkv_weights* w, const float* dx, const int* dpos, float* dq_out) {
  const tg_kv_desc& d = kv->d;
  const int qrows = d.n_head * d.head_dim, krows = d.n_kv_head * d.head_dim;
  TG_TRY(check_qkv_cols(w->cols));
  TG_TRY(check_wtype(w->q_type, "w_q"));
  TG_TRY(check_wtype(w->k_type, "w_k"));
  TG_TRY(check_wtype(w->v_type, "w_v"));
  if (!w->w_q || !w->w_k || !w->w_v) return fail(TG_ERR_INVALID_ARG, "null weight pointer");
  const void *wq = nullptr, *wk = nullptr, *wv = nullptr;
  const void *bq = nullptr, *bk = nullptr, *bv = nullptr;
  TG_TRY(weight_ptr(ctx, w->w_q, (size_t)qrows * qrow_bytes(w->q_type, w->cols), &wq));
  TG_TRY(weight_ptr(ctx, w->w_k, (size_t)krows * qrow_bytes(w->k_type, w->cols), &wk));
  TG_TRY(weight_ptr(ctx, w->w_v, (size_t)krows * qrow_bytes(w->v_type, w->cols), &wv));
  TG_TRY(weight_ptr(ctx, w->b_q, (size_t)qrows * 4, &bq));
  TG_TRY(weight_ptr(ctx, w->b_k, (size_t)krows * 4, &bk));
  TG_TRY(weight_ptr(ctx, w->b_v, (size_t)krows * 4, &bv));
  TG_TRY(check_align2(wq, "w_q"));
  TG_TRY(check_align2(wk, "w_k"));
  TG_TRY(check_align2(wv, "w_v"));
  TG_TRY(check_align8(dq_out, "q_out"));
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, d.rope_base, d.head_dim, kv->global_ctx, &t));
  tg::QkvParams p{};
  const void* ws[3] = {wq, wk, wv};
  const void* bs[3] = {bq, bk, bv};
  const int types[3] = {w->q_type, w->k_type, w->v_type};
  const int rows[3] = {qrows, krows, krows};
  for (int m = 0; m < 3; ++m) {
    p.w[m] = static_cast<const uint8_t*>(ws[m]);
    p.bias[m] = static_cast<const float*>(bs[m]);
    p.wtype[m] = types[m];
    p.rows[m] = rows[m];
  }
  p.cols = w->cols;
  p.x = dx;
  p.B = n;
  p.mode = 1;
  p.q_out = dq_out;
  p.pos = dpos;
  p.cs = t->d;
  p.table_len = kv->global_ctx;
  p.head_dim = d.head_dim;
  p.k_cache = static_cast<char*>(kv->k) + (size_t)layer * kv->layer_elems * kv->esize;
  p.v_cache = static_cast<char*>(kv->v) + (size_t)layer * kv->layer_elems * kv->esize;
  p.dtype = d.dtype;
  p.max_ctx = d.max_ctx;
  p.shard_start = d.shard_start;
  TG_TRY(run_qkv(ctx, p));
  note_pdl_write(ctx, kv, layer);
  return TG_OK;
}

int check_kv_call(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs) {
  if (!ctx || !kv) return fail(TG_ERR_INVALID_ARG, "null context or cache");
  if (kv->ctx != ctx) return fail(TG_ERR_INVALID_ARG, "cache belongs to another context");
  if (layer < 0 || layer >= kv->d.n_layers)
    return fail(TG_ERR_INVALID_ARG, "layer %d outside [0, %d)", layer, kv->d.n_layers);
  if (n_seqs < 0 || n_seqs > kv->d.n_seqs)
    return fail(TG_ERR_INVALID_ARG, "n_seqs %d outside [0, %d]", n_seqs, kv->d.n_seqs);
  return set_device(ctx);
}

// Host position arrays are validated here; device ones by the kernels.
int check_host_pos(const int32_t* pos, int n, int limit, const char* what) {
  if (!pos || is_device_ptr(pos)) return TG_OK;
  for (int i = 0; i < n; ++i)
    if (pos[i] < 0 || pos[i] >= limit)
      return fail(TG_ERR_INVALID_ARG, "%s[%d] = %d outside [0, %d)", what, i, pos[i], limit);
  return TG_OK;
}

}  // namespace

// ================================================================ C ABI

extern "C" {

const char* tg_status_string(int s) {
  switch (s) {
    case TG_OK: return "ok";
    case TG_ERR_INVALID_ARG: return "invalid argument";
    case TG_ERR_CUDA: return "CUDA error";
    case TG_ERR_NO_DEVICE: return "no CUDA device";
    case TG_ERR_OUT_OF_MEMORY: return "out of device memory";
    case TG_ERR_UNSUPPORTED: return "unsupported";
    case TG_ERR_DEVICE: return "device-side error";
    case TG_ERR_COMM: return "communicator error";
    case TG_ERR_STATE: return "invalid call order";
    default: return "unknown status";
  }
}

const char* tg_last_error(void) { return t_err.c_str(); }
const char* tg_version(void) { return TG_VERSION; }

int tg_init(int device, tg_context** out) {
  if (!out) return fail(TG_ERR_INVALID_ARG, "null output pointer");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(TG_ERR_NO_DEVICE, "no CUDA device available");
  }
  if (device < 0 || device >= n)
    return fail(TG_ERR_INVALID_ARG, "device %d outside [0, %d)", device, n);
  TG_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  TG_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major < 10)
    return fail(TG_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device,
                prop.major, prop.minor);
  tg_context* c = new tg_context();
  c->device = device;
  c->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess ||
      cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess) {
    cudaError_t e = cudaGetLastError();
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return fail(TG_ERR_CUDA, "context setup failed: %s", cudaGetErrorString(e));
  }
  if (cudaHostAlloc(&c->h_err, sizeof(int), cudaHostAllocDefault) == cudaSuccess) {
    *c->h_err = 0;
  } else {
    cudaGetLastError();
    c->h_err = nullptr;  // the error word is then read by a synchronous copy
  }
  c->own_stream = true;
  *out = c;
  return TG_OK;
}

int tg_shutdown(tg_context* ctx) {
  if (!ctx) return TG_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  p2p_release(ctx);
  if (ctx->comm) {
    nccl().CommDestroy(ctx->comm);
    ctx->comm = nullptr;
  }
  cudaFree(ctx->nccl_stage);
  free_graveyard(ctx);
  for (tg_kv_cache* kv : ctx->caches) {
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
  }
  ctx->caches.clear();
  for (auto& kv : ctx->regions) cudaFree(kv.second.dev);
  for (RopeTable& t : ctx->tables) cudaFree(t.d);
  for (cudaEvent_t ev : ctx->prof_ev) cudaEventDestroy(ev);
  cudaFree(ctx->part);
  cudaFree(ctx->stamps);
  cudaFree(ctx->sched);
  cudaFree(ctx->records);
  cudaFree(ctx->recv);
  cudaFree(ctx->arena);
  if (ctx->hpin) cudaFreeHost(ctx->hpin);
  cudaFree(ctx->qbf);
  cudaFree(ctx->vh);
  cudaFree(ctx->qx);
  cudaFree(ctx->cx);
  cudaFree(ctx->d_err);
  if (ctx->h_err) cudaFreeHost(ctx->h_err);
  if (ctx->copy_stream) {
    cudaStreamSynchronize(ctx->copy_stream);
    cudaStreamDestroy(ctx->copy_stream);
  }
  if (ctx->copy_done) cudaEventDestroy(ctx->copy_done);
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
  return TG_OK;
}

int tg_set_stream(tg_context* ctx, void* stream) {
  TG_TRY(set_device(ctx));
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  ctx->stream = static_cast<cudaStream_t>(stream);
  ctx->own_stream = false;
  return TG_OK;
}

int tg_get_stream(tg_context* ctx, void** stream) {
  if (!ctx || !stream) return fail(TG_ERR_INVALID_ARG, "null argument");
  *stream = ctx->stream;
  return TG_OK;
}

int tg_device_sms(tg_context* ctx, int* out) {
  if (!ctx || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  *out = ctx->num_sms;
  return TG_OK;
}

int tg_batch_begin(tg_context* ctx) {
  TG_TRY(set_device(ctx));
  if (ctx->in_batch) return fail(TG_ERR_STATE, "batch already open");
  if (ctx->capturing) return fail(TG_ERR_STATE, "graph capture open");
  ctx->in_batch = true;
  ctx->dstores.clear();
  return TG_OK;
}

int tg_batch_end(tg_context* ctx) {
  TG_TRY(set_device(ctx));
  if (!ctx->in_batch) return fail(TG_ERR_STATE, "tg_batch_end without tg_batch_begin");
  ctx->in_batch = false;
  const int rc = flush_deferred(ctx);
  for (const PendingCopy& c : ctx->pending)
    TG_CUDA(cudaMemcpyAsync(c.host, c.dev, c.bytes, cudaMemcpyDeviceToHost, ctx->stream));
  ctx->pending.clear();
  const int rf = flush_regions(ctx);
  return rc != TG_OK ? rc : rf;
}

int tg_synchronize(tg_context* ctx) {
  TG_TRY(set_device(ctx));
  if (ctx->capturing) return fail(TG_ERR_STATE, "graph capture open");
  const bool queued = queue_error_read(ctx);
  TG_TRY(wait_stream(ctx));
  if (!ctx->in_batch) {
    ctx->arena_off = 0;
    ctx->hpin_off = 0;
    free_graveyard(ctx);
  }
  return check_device_error(ctx, queued);
}

int tg_graph_begin(tg_context* ctx) {
  TG_TRY(set_device(ctx));
  if (ctx->in_batch || ctx->capturing) return fail(TG_ERR_STATE, "batch or capture already open");
  TG_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  ctx->capturing = true;
  ctx->capture_launches0 = ctx->launches;
  // A graph starts once the work before its launch has finished: inside it
  // only its own kernels can be in flight.
  ctx->pdl_saved.swap(ctx->pdl_writes);
  ctx->pdl_writes.clear();
  ctx->pdl_unknown_saved = ctx->pdl_unknown;
  ctx->pdl_unknown = false;
  return TG_OK;
}

int tg_graph_end(tg_context* ctx, tg_graph** out) {
  TG_TRY(set_device(ctx));
  if (!ctx->capturing) return fail(TG_ERR_STATE, "tg_graph_end without tg_graph_begin");
  if (!out) return fail(TG_ERR_INVALID_ARG, "null output pointer");
  ctx->capturing = false;
  ctx->pdl_writes.swap(ctx->pdl_saved);  // nothing captured has run
  ctx->pdl_saved.clear();
  ctx->pdl_unknown = ctx->pdl_unknown_saved;
  cudaGraph_t g = nullptr;
  TG_CUDA(cudaStreamEndCapture(ctx->stream, &g));
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
  if (e != cudaSuccess) {
    cudaGraphDestroy(g);
    return fail(TG_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(e));
  }
  tg_graph* tgg = new tg_graph();
  tgg->ctx = ctx;
  tgg->graph = g;
  tgg->exec = ex;
  tgg->kernels = ctx->launches - ctx->capture_launches0;
  ctx->launches = ctx->capture_launches0;  // recorded, not run
  *out = tgg;
  return TG_OK;
}

int tg_graph_launch(tg_context* ctx, tg_graph* g) {
  TG_TRY(set_device(ctx));
  if (!g || g->ctx != ctx) return fail(TG_ERR_INVALID_ARG, "graph of another context");
  TG_CUDA(cudaGraphLaunch(g->exec, ctx->stream));
  ctx->launches += g->kernels;
  ctx->pdl_unknown = true;  // its kernels' writes are not tracked here
  return TG_OK;
}

int tg_graph_destroy(tg_graph* g) {
  if (!g) return TG_OK;
  cudaSetDevice(g->ctx->device);
  cudaStreamSynchronize(g->ctx->stream);
  cudaGraphExecDestroy(g->exec);
  cudaGraphDestroy(g->graph);
  delete g;
  return TG_OK;
}

int tg_register_host(tg_context* ctx, void* host_ptr, size_t bytes, int flags) {
  TG_TRY(set_device(ctx));
  if (!host_ptr || bytes == 0) return fail(TG_ERR_INVALID_ARG, "empty host range");
  if (is_device_ptr(host_ptr)) return fail(TG_ERR_INVALID_ARG, "pointer is device memory");
  Region* r = nullptr;
  TG_TRY(create_region(ctx, static_cast<char*>(host_ptr), bytes, flags, false, &r));
  if (!ctx->in_batch) return flush_regions(ctx);
  return TG_OK;
}

int tg_unregister_host(tg_context* ctx, void* host_ptr) {
  TG_TRY(set_device(ctx));
  auto it = ctx->regions.find(reinterpret_cast<uintptr_t>(host_ptr));
  if (it == ctx->regions.end() || it->second.transient)
    return fail(TG_ERR_INVALID_ARG, "pointer is not the start of a registered array");
  if (ctx->in_batch) return fail(TG_ERR_STATE, "cannot unregister inside a batch");
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
  cudaFree(it->second.dev);
  ctx->regions.erase(it);
  return TG_OK;
}

int tg_region_sync(tg_context* ctx, void* host_ptr, size_t bytes, int to_device) {
  TG_TRY(set_device(ctx));
  Region* r = find_region(ctx, static_cast<char*>(host_ptr), bytes);
  if (!r) return fail(TG_ERR_INVALID_ARG, "range is not inside a registered region");
  const size_t off = (size_t)(static_cast<char*>(host_ptr) - r->host);
  if (to_device)
    TG_CUDA(cudaMemcpyAsync(r->dev + off, host_ptr, bytes, cudaMemcpyHostToDevice, ctx->stream));
  else
    TG_CUDA(cudaMemcpyAsync(host_ptr, r->dev + off, bytes, cudaMemcpyDeviceToHost, ctx->stream));
  if (ctx->in_batch) return TG_OK;
  TG_TRY(wait_stream(ctx));
  return TG_OK;
}

// ------------------------------------------------ reference-compatible ops

int tg_rope_op(tg_context* ctx, float* data, int n_heads, int head_dim, int pos, float base) {
  TG_TRY(set_device(ctx));
  if (!data || n_heads <= 0 || head_dim <= 0 || head_dim % 2 || pos < 0)
    return fail(TG_ERR_INVALID_ARG, "rope_op: bad arguments (n_heads=%d head_dim=%d pos=%d)",
                n_heads, head_dim, pos);
  char* d = nullptr;
  TG_TRY(resolve(ctx, data, (size_t)n_heads * head_dim * 4, true, &d));
  TG_TRY(check_align8(d, "data"));
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, base, head_dim, pos + 1, &t));
  tg::RopeParams rp{};
  rp.q = reinterpret_cast<float*>(d);
  rp.pos_scalar = pos;
  rp.cs = t->d;
  rp.table_len = t->len;
  rp.B = 1;
  rp.n_head = n_heads;
  rp.n_kv = 1;
  rp.head_dim = head_dim;
  rp.err = ctx->d_err;
  cudaError_t e = tg::launch_rope(rp, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "rope launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  return finish_compat(ctx);
}

int tg_elem_op(tg_context* ctx, int op, float* data, const float* aux, int dim) {
  TG_TRY(set_device(ctx));
  if (op == 1)
    return fail(TG_ERR_UNSUPPORTED, "elem_op op 1 (SiLU x up) belongs to the FFN, not this path");
  if (op != 0 && op != 2) return fail(TG_ERR_INVALID_ARG, "elem_op: unknown op %d", op);
  if (!data || !aux || dim < 0) return fail(TG_ERR_INVALID_ARG, "elem_op: bad arguments");
  if (dim == 0) return TG_OK;
  char *dd = nullptr, *da = nullptr;
  TG_TRY(ensure_region(ctx, aux, (size_t)dim * 4));
  TG_TRY(ensure_region(ctx, data, (size_t)dim * 4));
  TG_TRY(resolve(ctx, aux, (size_t)dim * 4, false, &da));
  TG_TRY(resolve(ctx, data, (size_t)dim * 4, true, &dd));
  cudaError_t e = tg::launch_elem(op, reinterpret_cast<float*>(dd),
                                  reinterpret_cast<const float*>(da), dim, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "elem launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  return finish_compat(ctx);
}

int tg_attention_op(tg_context* ctx, const float* Q, const float* K_cache, const float* V_cache,
                    float* output, int n_head, int n_kv_head, int head_dim, int past_len) {
  TG_TRY(set_device(ctx));
  TG_TRY(check_shape(n_head, n_kv_head, head_dim));
  if (past_len < 0) return fail(TG_ERR_INVALID_ARG, "attention_op: past_len %d < 0", past_len);
  const size_t qbytes = (size_t)n_head * head_dim * 4;
  const size_t cbytes = (size_t)(past_len + 1) * n_kv_head * head_dim * 4;
  char *dq = nullptr, *dk = nullptr, *dv = nullptr, *dout = nullptr;
  TG_TRY(ensure_region(ctx, Q, qbytes));
  TG_TRY(ensure_region(ctx, K_cache, cbytes));
  TG_TRY(ensure_region(ctx, V_cache, cbytes));
  TG_TRY(ensure_region(ctx, output, qbytes));
  TG_TRY(resolve(ctx, Q, qbytes, false, &dq));
  TG_TRY(resolve(ctx, K_cache, cbytes, false, &dk));
  TG_TRY(resolve(ctx, V_cache, cbytes, false, &dv));
  TG_TRY(resolve(ctx, output, qbytes, true, &dout));
  // A one-sequence, one-layer view of the caller's fp32 cache.
  tg_kv_cache view;
  view.ctx = ctx;
  view.d.n_layers = 1;
  view.d.n_seqs = 1;
  view.d.max_ctx = past_len + 1;
  view.d.n_head = n_head;
  view.d.n_kv_head = n_kv_head;
  view.d.head_dim = head_dim;
  view.d.dtype = TG_DTYPE_F32;
  view.row_elems = (size_t)n_kv_head * head_dim;
  view.esize = 4;
  view.layer_elems = view.row_elems * (past_len + 1);
  view.k = dk;
  view.v = dv;
  view.global_ctx = past_len + 1;
  TG_TRY(run_decode(ctx, &view, 0, 1, reinterpret_cast<const float*>(dq), nullptr, past_len,
                    reinterpret_cast<float*>(dout), 0));
  return finish_compat(ctx);
}

// ------------------------------------------------ KV caches

int tg_kv_create(tg_context* ctx, const tg_kv_desc* desc, tg_kv_cache** out) {
  TG_TRY(set_device(ctx));
  if (!desc || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  const tg_kv_desc& d = *desc;
  TG_TRY(check_shape(d.n_head, d.n_kv_head, d.head_dim));
  if (d.n_layers <= 0 || d.n_seqs <= 0 || d.max_ctx <= 0 || d.shard_start < 0)
    return fail(TG_ERR_INVALID_ARG, "kv_create: bad sizes");
  if (d.dtype != TG_DTYPE_F32 && d.dtype != TG_DTYPE_BF16)
    return fail(TG_ERR_INVALID_ARG, "kv_create: dtype %d", d.dtype);
  const long long rows = (long long)d.n_layers * d.n_seqs * d.max_ctx;
  if (rows >= (1LL << 31)) return fail(TG_ERR_INVALID_ARG, "kv_create: %lld rows is too many", rows);
  if (!(d.rope_base > 0.f)) return fail(TG_ERR_INVALID_ARG, "kv_create: rope_base must be > 0");
  tg_kv_cache* kv = new tg_kv_cache();
  kv->ctx = ctx;
  kv->d = d;
  kv->row_elems = (size_t)d.n_kv_head * d.head_dim;
  kv->esize = d.dtype == TG_DTYPE_F32 ? 4 : 2;
  kv->layer_elems = kv->row_elems * (size_t)d.n_seqs * d.max_ctx;
  kv->global_ctx = d.global_ctx > 0 ? d.global_ctx : d.shard_start + d.max_ctx;
  if (kv->global_ctx < d.shard_start + d.max_ctx) kv->global_ctx = d.shard_start + d.max_ctx;
  const size_t bytes = kv->layer_elems * d.n_layers * kv->esize;
  if (cudaMalloc(&kv->k, bytes) != cudaSuccess || cudaMalloc(&kv->v, bytes) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
    return fail(TG_ERR_OUT_OF_MEMORY, "kv_create: %zu bytes per cache", bytes);
  }
  cudaMemsetAsync(kv->k, 0, bytes, ctx->stream);
  cudaMemsetAsync(kv->v, 0, bytes, ctx->stream);
  if (d.dtype == TG_DTYPE_BF16 && d.head_dim == 64) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (enc) {
      cuuint64_t gdim[2] = {(cuuint64_t)kv->row_elems, (cuuint64_t)rows};
      cuuint64_t gstride[1] = {(cuuint64_t)(kv->row_elems * 2)};
      cuuint32_t box[2] = {64, 64};
      cuuint32_t estr[2] = {1, 1};
      CUresult r1 = enc(&kv->tmk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv->k, gdim, gstride, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      CUresult r2 = enc(&kv->tmv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv->v, gdim, gstride, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      kv->tmap_ok = (r1 == CUDA_SUCCESS && r2 == CUDA_SUCCESS);
      cuuint32_t box128[2] = {64, 128};
      CUresult r3 = enc(&kv->tmk128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv->k, gdim, gstride,
                        box128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      CUresult r4 = enc(&kv->tmv128, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kv->v, gdim, gstride,
                        box128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      kv->tmap128_ok = (r3 == CUDA_SUCCESS && r4 == CUDA_SUCCESS);
    }
  }
  RopeTable* t = nullptr;
  int rc = get_table(ctx, d.rope_base, d.head_dim, kv->global_ctx, &t);
  if (rc != TG_OK) {
    cudaFree(kv->k);
    cudaFree(kv->v);
    delete kv;
    return rc;
  }
  if (cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaError_t e = cudaGetLastError();
    return fail(TG_ERR_CUDA, "kv_create: %s", cudaGetErrorString(e));
  }
  ctx->caches.push_back(kv);
  *out = kv;
  return TG_OK;
}

int tg_kv_destroy(tg_kv_cache* kv) {
  if (!kv) return TG_OK;
  cudaSetDevice(kv->ctx->device);
  if (cudaStreamSynchronize(kv->ctx->stream) == cudaSuccess) stream_idle(kv->ctx);
  auto& cs = kv->ctx->caches;
  for (size_t i = 0; i < cs.size(); ++i)
    if (cs[i] == kv) {
      cs.erase(cs.begin() + i);
      break;
    }
  cudaFree(kv->k);
  cudaFree(kv->v);
  delete kv;
  return TG_OK;
}

int tg_kv_reset(tg_kv_cache* kv) {
  if (!kv) return fail(TG_ERR_INVALID_ARG, "null cache");
  TG_TRY(set_device(kv->ctx));
  const size_t bytes = kv->layer_elems * kv->d.n_layers * kv->esize;
  TG_CUDA(cudaMemsetAsync(kv->k, 0, bytes, kv->ctx->stream));
  TG_CUDA(cudaMemsetAsync(kv->v, 0, bytes, kv->ctx->stream));
  if (kv->ctx->in_batch) return TG_OK;
  return tg_synchronize(kv->ctx);
}

int tg_kv_layer_ptrs(tg_kv_cache* kv, int layer, void** k, void** v) {
  if (!kv || layer < 0 || layer >= kv->d.n_layers)
    return fail(TG_ERR_INVALID_ARG, "bad cache or layer");
  const size_t off = (size_t)layer * kv->layer_elems * kv->esize;
  if (k) *k = static_cast<char*>(kv->k) + off;
  if (v) *v = static_cast<char*>(kv->v) + off;
  return TG_OK;
}

int tg_kv_fill_normal(tg_kv_cache* kv, uint64_t seed) {
  if (!kv) return fail(TG_ERR_INVALID_ARG, "null cache");
  tg_context* ctx = kv->ctx;
  TG_TRY(set_device(ctx));
  const size_t n = kv->layer_elems * kv->d.n_layers;
  cudaError_t e = tg::launch_fill_normal(kv->k, n, kv->d.dtype, seed, ctx->num_sms, ctx->stream);
  if (e == cudaSuccess)
    e = tg::launch_fill_normal(kv->v, n, kv->d.dtype, seed ^ 0x5bd1e995ULL, ctx->num_sms,
                               ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "fill launch: %s", cudaGetErrorString(e));
  ctx->launches += 2;
  if (ctx->in_batch) return TG_OK;
  return tg_synchronize(ctx);
}

int tg_kv_write_rows(tg_kv_cache* kv, int layer, int seq, int row0, int n_rows,
                     const float* k_rows, const float* v_rows) {
  if (!kv) return fail(TG_ERR_INVALID_ARG, "null cache");
  tg_context* ctx = kv->ctx;
  TG_TRY(check_kv_call(ctx, kv, layer, kv->d.n_seqs));
  if (seq < 0 || seq >= kv->d.n_seqs || row0 < 0 || n_rows < 0 || row0 + n_rows > kv->d.max_ctx)
    return fail(TG_ERR_INVALID_ARG, "kv_write_rows: rows [%d, %d) of seq %d out of range", row0,
                row0 + n_rows, seq);
  if (n_rows == 0) return TG_OK;
  const size_t n = (size_t)n_rows * kv->row_elems;
  const size_t off = ((size_t)layer * kv->layer_elems +
                      ((size_t)seq * kv->d.max_ctx + row0) * kv->row_elems) * kv->esize;
  const void* src[2] = {k_rows, v_rows};
  void* dst[2] = {static_cast<char*>(kv->k) + off, static_cast<char*>(kv->v) + off};
  for (int i = 0; i < 2; ++i) {
    if (!src[i]) continue;
    const void* ds = nullptr;
    TG_TRY(stage_in(ctx, src[i], n * 4, &ds));
    TG_TRY(commit_inputs(ctx));
    cudaError_t e = tg::launch_convert_rows(dst[i], static_cast<const float*>(ds), n,
                                            kv->d.dtype, ctx->num_sms, ctx->stream);
    if (e != cudaSuccess) return fail(TG_ERR_CUDA, "convert launch: %s", cudaGetErrorString(e));
    ctx->launches++;
  }
  return finish_call(ctx);
}

int tg_kv_read_rows(tg_kv_cache* kv, int layer, int seq, int row0, int n_rows, void* k_out,
                    void* v_out) {
  if (!kv) return fail(TG_ERR_INVALID_ARG, "null cache");
  tg_context* ctx = kv->ctx;
  TG_TRY(check_kv_call(ctx, kv, layer, kv->d.n_seqs));
  if (seq < 0 || seq >= kv->d.n_seqs || row0 < 0 || n_rows < 0 || row0 + n_rows > kv->d.max_ctx)
    return fail(TG_ERR_INVALID_ARG, "kv_read_rows: rows out of range");
  const size_t bytes = (size_t)n_rows * kv->row_elems * kv->esize;
  const size_t off = ((size_t)layer * kv->layer_elems +
                      ((size_t)seq * kv->d.max_ctx + row0) * kv->row_elems) * kv->esize;
  if (k_out)
    TG_CUDA(cudaMemcpyAsync(k_out, static_cast<char*>(kv->k) + off, bytes, cudaMemcpyDefault,
                            ctx->stream));
  if (v_out)
    TG_CUDA(cudaMemcpyAsync(v_out, static_cast<char*>(kv->v) + off, bytes, cudaMemcpyDefault,
                            ctx->stream));
  if (ctx->in_batch) return TG_OK;
  return tg_synchronize(ctx);
}

// ------------------------------------------------ batched decode

int tg_rope_cache_write(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, float* q,
                        float* k_new, const float* v_new, const int32_t* pos) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!pos) return fail(TG_ERR_INVALID_ARG, "null pos");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(pos, n_seqs, kv->global_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  void *dq = nullptr, *dk = nullptr;
  const void *dv = nullptr, *dp = nullptr;
  TG_TRY(stage_out(ctx, q, (size_t)n_seqs * d.n_head * d.head_dim * 4, true, &dq));
  TG_TRY(stage_out(ctx, k_new, (size_t)n_seqs * kv->row_elems * 4, true, &dk));
  TG_TRY(stage_in(ctx, v_new, (size_t)n_seqs * kv->row_elems * 4, &dv));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(run_rope(ctx, kv, layer, n_seqs, static_cast<float*>(dq), static_cast<float*>(dk),
                  static_cast<const float*>(dv), static_cast<const int*>(dp)));
  return finish_call(ctx);
}

int tg_attention_batched(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, const float* q,
                         const int32_t* past_len, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !past_len || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(past_len, n_seqs, kv->d.shard_start + kv->d.max_ctx, "past_len"));
  const size_t qb = (size_t)n_seqs * kv->d.n_head * kv->d.head_dim * 4;
  const void *dq = nullptr, *dp = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, q, qb, &dq));
  TG_TRY(stage_in(ctx, past_len, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout));
  if (mma_eligible(kv))
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, static_cast<const float*>(dq), nullptr, nullptr,
                     nullptr, static_cast<const int*>(dp), static_cast<float*>(dout), nullptr,
                     0, false, false, nullptr, preload_allowed(ctx, kv, layer)));
  else
    TG_TRY(run_decode(ctx, kv, layer, n_seqs, static_cast<const float*>(dq),
                      static_cast<const int*>(dp), 0, static_cast<float*>(dout), 0));
  return finish_call(ctx);
}

int tg_decode_layer(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, float* q,
                    float* k_new, const float* v_new, const int32_t* pos, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !k_new || !v_new || !pos || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(pos, n_seqs, kv->d.shard_start + kv->d.max_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  const size_t qb = (size_t)n_seqs * d.n_head * d.head_dim * 4;
  const size_t kb = (size_t)n_seqs * kv->row_elems * 4;
  void *dq = nullptr, *dk = nullptr, *dout = nullptr;
  const void *dv = nullptr, *dp = nullptr, *dq_in = nullptr, *dk_in = nullptr, *dout_in = nullptr;
  // The tensor-core and short-cache paths read staged copies and write
  // page-locked host outputs directly (no device->host copy between two
  // kernels of a batch); the CUDA-core path works in place.
  const bool split_io = mma_eligible(kv) || small_eligible(kv);
  TG_TRY(stage_out(ctx, q, qb, true, &dq, split_io ? &dq_in : nullptr));
  TG_TRY(stage_out(ctx, k_new, kb, true, &dk, split_io ? &dk_in : nullptr));
  TG_TRY(stage_in(ctx, v_new, kb, &dv));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout, split_io ? &dout_in : nullptr));
  if (split_io && mma_eligible(kv)) {
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, static_cast<const float*>(dq_in),
                     static_cast<float*>(dq), const_cast<float*>(static_cast<const float*>(dk_in)),
                     static_cast<const float*>(dv), static_cast<const int*>(dp),
                     static_cast<float*>(dout), nullptr, 0, true, true, static_cast<float*>(dk),
                     preload_allowed(ctx, kv, layer)));
    return finish_call(ctx);
  }
  if (small_eligible(kv)) {
    TG_TRY(run_small_step(ctx, kv, layer, n_seqs, const_cast<float*>(static_cast<const float*>(dq_in)),
                          const_cast<float*>(static_cast<const float*>(dk_in)),
                          static_cast<const float*>(dv), static_cast<const int*>(dp),
                          static_cast<float*>(dout), static_cast<float*>(dq),
                          static_cast<float*>(dk)));
    return finish_call(ctx);
  }
  TG_TRY(run_rope(ctx, kv, layer, n_seqs, static_cast<float*>(dq), static_cast<float*>(dk),
                  static_cast<const float*>(dv), static_cast<const int*>(dp)));
  TG_TRY(run_decode(ctx, kv, layer, n_seqs, static_cast<const float*>(dq),
                    static_cast<const int*>(dp), 0, static_cast<float*>(dout), 0));
  return finish_call(ctx);
}

// ------------------------------------------------ Q/K/V projection

namespace {
// hidden[s] += W_o ctx[s] on device x / hidden (mode 2 of the projection
// kernel); W_o resolved by weight_ptr.
int attn_output_core(tg_context* ctx, int n, int wtype, const void* w_o, int rows, int cols,
                     const float* dctx, float* dhidden) {
  TG_TRY(check_wtype(wtype, "w_o"));
  TG_TRY(check_qkv_cols(cols));
  if (rows <= 0) return fail(TG_ERR_INVALID_ARG, "attn_output: rows %d", rows);
  const void* dw = nullptr;
  TG_TRY(weight_ptr(ctx, w_o, (size_t)rows * qrow_bytes(wtype, cols), &dw));
  TG_TRY(check_align2(dw, "w_o"));
  tg::QkvParams p{};
  p.w[0] = static_cast<const uint8_t*>(dw);
  p.wtype[0] = p.wtype[1] = p.wtype[2] = wtype;
  p.rows[0] = rows;
  p.y[0] = dhidden;
  p.cols = cols;
  p.x = dctx;
  p.B = n;
  p.mode = 2;
  return run_qkv(ctx, p);
}
}  // namespace

int tg_attn_output(tg_context* ctx, int n_seqs, int wtype, const void* w_o, int rows, int cols,
                   const float* context, float* hidden) {
  TG_TRY(set_device(ctx));
  if (n_seqs < 0 || !w_o || !context || !hidden)
    return fail(TG_ERR_INVALID_ARG, "attn_output: bad arguments");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_wtype(wtype, "w_o"));
  TG_TRY(check_qkv_cols(cols));
  if (rows <= 0) return fail(TG_ERR_INVALID_ARG, "attn_output: rows %d", rows);
  const void* dc = nullptr;
  void* dh = nullptr;
  TG_TRY(stage_in(ctx, context, (size_t)n_seqs * cols * 4, &dc));
  TG_TRY(stage_out(ctx, hidden, (size_t)n_seqs * rows * 4, true, &dh));
  TG_TRY(attn_output_core(ctx, n_seqs, wtype, w_o, rows, cols, static_cast<const float*>(dc),
                          static_cast<float*>(dh)));
  return finish_call(ctx);
}

int tg_set_decode_tuning(int ring_kb, int preload) {
  if ((ring_kb != 0 && ring_kb != tg::kFusedRing && ring_kb != tg::kFusedRingDeep) ||
      (preload != 0 && preload != 1))
    return fail(TG_ERR_INVALID_ARG, "decode tuning: ring_kb %d (0, 128, 192), preload %d (0, 1)",
                ring_kb, preload);
  g_decode_ring = ring_kb;
  g_decode_preload = preload;
  return TG_OK;
}

int tg_set_projection_split(int split) {
  if (tg::set_qkv_tc_split(split) != 0)
    return fail(TG_ERR_INVALID_ARG, "projection split %d: 0 to 8", split);
  return TG_OK;
}

int tg_fused_qkv_op(tg_context* ctx, const uint8_t* W_q, const uint8_t* W_k, const uint8_t* W_v,
                    const float* x, float* y_q, float* y_k, float* y_v, int q_rows, int k_rows,
                    int v_rows, int cols, int v_is_q8) {
  TG_TRY(set_device(ctx));
  if (q_rows < 0 || k_rows < 0 || v_rows < 0)
    return fail(TG_ERR_INVALID_ARG, "fused_qkv_op: negative row count");
  TG_TRY(check_qkv_cols(cols));
  const uint8_t* W[3] = {W_q, W_k, W_v};
  float* Y[3] = {y_q, y_k, y_v};
  const int R[3] = {q_rows, k_rows, v_rows};
  const int T[3] = {TG_WTYPE_Q5_0, TG_WTYPE_Q5_0, v_is_q8 ? TG_WTYPE_Q8_0 : TG_WTYPE_Q5_0};
  if (!x) return fail(TG_ERR_INVALID_ARG, "fused_qkv_op: null x");
  for (int m = 0; m < 3; ++m)
    if (R[m] > 0 && (!W[m] || !Y[m]))
      return fail(TG_ERR_INVALID_ARG, "fused_qkv_op: null weight or output");
  if (R[0] + R[1] + R[2] == 0) return TG_OK;
  // Every mirror first, then the addresses (see ensure_region).
  TG_TRY(ensure_region(ctx, x, (size_t)cols * 4));
  for (int m = 0; m < 3; ++m) {
    if (!R[m]) continue;
    TG_TRY(ensure_region(ctx, W[m], (size_t)R[m] * qrow_bytes(T[m], cols)));
    TG_TRY(ensure_region(ctx, Y[m], (size_t)R[m] * 4));
  }
  tg::QkvParams p{};
  char* dx = nullptr;
  TG_TRY(resolve(ctx, x, (size_t)cols * 4, false, &dx));
  for (int m = 0; m < 3; ++m) {
    p.wtype[m] = T[m];
    if (!R[m]) continue;
    char *dw = nullptr, *dy = nullptr;
    TG_TRY(resolve(ctx, W[m], (size_t)R[m] * qrow_bytes(T[m], cols), false, &dw));
    TG_TRY(resolve(ctx, Y[m], (size_t)R[m] * 4, true, &dy));
    TG_TRY(check_align2(dw, "weights"));
    p.w[m] = reinterpret_cast<const uint8_t*>(dw);
    p.y[m] = reinterpret_cast<float*>(dy);
    p.rows[m] = R[m];
  }
  p.cols = cols;
  p.x = reinterpret_cast<const float*>(dx);
  p.B = 1;
  p.mode = 0;
  TG_TRY(run_qkv(ctx, p));
  return finish_compat(ctx);
}

int tg_matmul_q(tg_context* ctx, int wtype, int rows, int cols, const uint8_t* w, const float* x,
                float* y) {
  TG_TRY(set_device(ctx));
  TG_TRY(check_wtype(wtype, "matmul_q"));
  TG_TRY(check_qkv_cols(cols));
  if (rows < 0) return fail(TG_ERR_INVALID_ARG, "matmul_q: negative rows");
  if (!w || !x || !y) return fail(TG_ERR_INVALID_ARG, "matmul_q: null argument");
  if (rows == 0) return TG_OK;
  const size_t wb = (size_t)rows * qrow_bytes(wtype, cols);
  TG_TRY(ensure_region(ctx, w, wb));
  TG_TRY(ensure_region(ctx, x, (size_t)cols * 4));
  TG_TRY(ensure_region(ctx, y, (size_t)rows * 4));
  char *dw = nullptr, *dx = nullptr, *dy = nullptr;
  TG_TRY(resolve(ctx, w, wb, false, &dw));
  TG_TRY(resolve(ctx, x, (size_t)cols * 4, false, &dx));
  TG_TRY(resolve(ctx, y, (size_t)rows * 4, true, &dy));
  TG_TRY(check_align2(dw, "weights"));
  tg::QkvParams p{};
  p.w[0] = reinterpret_cast<const uint8_t*>(dw);
  p.wtype[0] = p.wtype[1] = p.wtype[2] = wtype;
  p.rows[0] = rows;
  p.y[0] = reinterpret_cast<float*>(dy);
  p.cols = cols;
  p.x = reinterpret_cast<const float*>(dx);
  p.B = 1;
  p.mode = 0;
  TG_TRY(run_qkv(ctx, p));
  return finish_compat(ctx);
}

int tg_qkv_rope_cache_write(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                            const tg_qkv_weights* w, const float* x, const int32_t* pos,
                            float* q_out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!w || !x || !pos || !q_out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_qkv_cols(w->cols));
  TG_TRY(check_host_pos(pos, n_seqs, kv->global_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  const void *dx = nullptr, *dp = nullptr;
  void* dq = nullptr;
  TG_TRY(stage_in(ctx, x, (size_t)n_seqs * w->cols * 4, &dx));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, q_out, (size_t)n_seqs * d.n_head * d.head_dim * 4, false, &dq));
  TG_TRY(qkv_layer_core(ctx, kv, layer, n_seqs, w, static_cast<const float*>(dx),
                        static_cast<const int*>(dp), static_cast<float*>(dq)));
  return finish_call(ctx);
}

int tg_decode_layer_x(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                      const tg_qkv_weights* w, const float* x, const int32_t* pos, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!w || !x || !pos || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_qkv_cols(w->cols));
  TG_TRY(check_host_pos(pos, n_seqs, kv->d.shard_start + kv->d.max_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  const size_t qb = (size_t)n_seqs * d.n_head * d.head_dim * 4;
  const void *dx = nullptr, *dp = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, x, (size_t)n_seqs * w->cols * 4, &dx));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout));
  TG_TRY(ensure_buf(ctx, &ctx->qx, &ctx->qx_cap, qb / 4));
  // Checked before the projection, which writes only the new rows (the
  // decode kernel loads the tiles holding them after its wait).
  const bool pre = preload_allowed(ctx, kv, layer);
  TG_TRY(qkv_layer_core(ctx, kv, layer, n_seqs, w, static_cast<const float*>(dx),
                        static_cast<const int*>(dp), ctx->qx));
  if (mma_eligible(kv))
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, ctx->qx, nullptr, nullptr, nullptr,
                     static_cast<const int*>(dp), static_cast<float*>(dout), nullptr, 0, false,
                     false, nullptr, pre));
  else
    TG_TRY(run_decode(ctx, kv, layer, n_seqs, ctx->qx, static_cast<const int*>(dp), 0,
                      static_cast<float*>(dout), 0));
  return finish_call(ctx);
}

// ------------------------------------------------ split-KV

int tg_comm_unique_id(void* id_out, size_t id_bytes) {
  if (!id_out || id_bytes < sizeof(ncclUniqueId))
    return fail(TG_ERR_INVALID_ARG, "id buffer must hold %zu bytes", sizeof(ncclUniqueId));
  if (!nccl().ok) return fail(TG_ERR_COMM, "NCCL library not found");
  ncclUniqueId id;
  ncclResult_t r = nccl().GetUniqueId(&id);
  if (r != ncclSuccess) return fail(TG_ERR_COMM, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
  std::memcpy(id_out, &id, sizeof(id));
  return TG_OK;
}

int tg_comm_init(tg_context* ctx, const void* id, int rank, int world, int timeout_ms) {
  TG_TRY(set_device(ctx));
  if (!id || world < 1 || rank < 0 || rank >= world)
    return fail(TG_ERR_INVALID_ARG, "comm_init: rank %d world %d", rank, world);
  if (ctx->comm) return fail(TG_ERR_STATE, "communicator already initialised");
  if (!nccl().ok) return fail(TG_ERR_COMM, "NCCL library not found");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // initialisation is polled with a deadline below
  ncclComm_t comm = nullptr;
  ncclResult_t r = nccl().CommInitRankConfig(&comm, world, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress)
    return fail(TG_ERR_COMM, "ncclCommInitRankConfig: %s", nccl().GetErrorString(r));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t ae = ncclInProgress;
    nccl().CommGetAsyncError(comm, &ae);
    if (ae == ncclSuccess) break;
    const double ms = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now() - t0)
                          .count();
    if (ae != ncclInProgress || ms > timeout_ms) {
      nccl().CommAbort(comm);
      return fail(TG_ERR_COMM, "communicator init failed (%s after %.0f ms)",
                  ae == ncclInProgress ? "timeout" : nccl().GetErrorString(ae), ms);
    }
  }
  ctx->comm = comm;
  ctx->rank = rank;
  ctx->world = world;
  ctx->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  return TG_OK;
}

int tg_comm_set_exchange(tg_context* ctx, int exchange) {
  if (!ctx) return fail(TG_ERR_INVALID_ARG, "null context");
  if (exchange < TG_EXCHANGE_AUTO || exchange > TG_EXCHANGE_NCCL)
    return fail(TG_ERR_INVALID_ARG, "exchange %d is not TG_EXCHANGE_AUTO / PEER / NCCL", exchange);
  ctx->exchange_pref = exchange;
  return TG_OK;
}

int tg_comm_set_wait_limit_ms(tg_context* ctx, int ms) {
  if (!ctx) return fail(TG_ERR_INVALID_ARG, "null context");
  if (ms <= 0) return fail(TG_ERR_INVALID_ARG, "wait limit %d ms must be positive", ms);
  ctx->wait_ns = (long long)ms * 1000000LL;
  return TG_OK;
}

int tg_comm_exchange(tg_context* ctx, int* exchange) {
  if (!ctx || !exchange) return fail(TG_ERR_INVALID_ARG, "null argument");
  *exchange = ctx->exchange_used;
  return TG_OK;
}

int tg_comm_destroy(tg_context* ctx) {
  TG_TRY(set_device(ctx));
  if (!ctx->comm) return TG_OK;
  cudaStreamSynchronize(ctx->stream);
  p2p_release(ctx);
  ctx->p2p_failed = false;
  ctx->exchange_used = TG_EXCHANGE_AUTO;
  nccl().CommDestroy(ctx->comm);
  ctx->comm = nullptr;
  ctx->world = 1;
  ctx->rank = 0;
  return TG_OK;
}

namespace {
// dq / dk are read; dq_out / dk_out receive the rotated q / k (the same
// buffers unless the caller's pinned host memory is written directly, which
// only the tensor-core path does).
int splitkv_core(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, float* dq,
                 float* dk, const float* dv, const int* dp, float* dout, bool rope_new,
                 bool preload, float* dq_out = nullptr, float* dk_out = nullptr) {
  TG_TRY(commit_inputs(ctx));
  if (!dq_out) dq_out = dq;
  if (!dk_out) dk_out = dk;
  const tg_kv_desc& d = kv->d;
  const int rf = tg::record_floats(d.n_head, d.head_dim);
  const bool fused = mma_eligible(kv);
  if (fused && ctx->world == 1)  // one GPU: no exchange at all
    return run_fused(ctx, kv, layer, n_seqs, dq, rope_new ? dq_out : nullptr,
                     rope_new ? dk : nullptr, dv, dp, dout, nullptr, 0, rope_new, rope_new,
                     rope_new ? dk_out : nullptr, preload);
  if (ctx->world > 1 && ctx->exchange_pref != TG_EXCHANGE_NCCL) {
    const int rc = fused ? ensure_p2p(ctx, n_seqs, d.n_head, rf) : TG_ERR_UNSUPPORTED;
    if (rc == TG_OK) {
      ctx->exchange_used = TG_EXCHANGE_PEER;
      return run_fused(ctx, kv, layer, n_seqs, dq, rope_new ? dq_out : nullptr,
                       rope_new ? dk : nullptr, dv, dp, dout, nullptr, 2, rope_new, rope_new,
                       rope_new ? dk_out : nullptr, preload);
    }
    if (rc != TG_ERR_UNSUPPORTED) return rc;
    if (ctx->exchange_pref == TG_EXCHANGE_PEER)
      return fail(TG_ERR_UNSUPPORTED,
                  "peer-memory exchange needs a bf16 tensor-core cache and peer access "
                  "between every pair of GPUs");
    t_err.clear();  // no peer memory between these GPUs: NCCL all-gather below
  }
  if (ctx->world > 1) ctx->exchange_used = TG_EXCHANGE_NCCL;
  // Records of this shard, all-gathered over NCCL, merged on every rank.
  TG_TRY(ensure_buf(ctx, &ctx->records, &ctx->rec_cap, (size_t)n_seqs * rf));
  if (fused) {
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, dq, rope_new ? dq_out : nullptr,
                     rope_new ? dk : nullptr, dv, dp, nullptr, ctx->records, 1, rope_new,
                     rope_new, rope_new ? dk_out : nullptr, preload));
  } else {
    if (dq_out != dq || dk_out != dk)
      return fail(TG_ERR_STATE, "separate q / k outputs need the tensor-core path");
    if (rope_new) TG_TRY(run_rope(ctx, kv, layer, n_seqs, dq, dk, dv, dp));
    TG_TRY(run_decode(ctx, kv, layer, n_seqs, dq, dp, 0, nullptr, 1));
  }
  const size_t count = (size_t)n_seqs * rf;
  TG_TRY(ensure_buf(ctx, &ctx->recv, &ctx->recv_cap, count * ctx->world));
  if (ctx->world > 1) {
    ncclResult_t r = nccl().AllGather(ctx->records, ctx->recv, count, ncclFloat32, ctx->comm,
                                      ctx->stream);
    if (r == ncclInProgress) {
      const auto t0 = std::chrono::steady_clock::now();
      do {
        nccl().CommGetAsyncError(ctx->comm, &r);
        const double ms = std::chrono::duration<double, std::milli>(
                              std::chrono::steady_clock::now() - t0)
                              .count();
        if (r == ncclInProgress && ms > ctx->timeout_ms) break;
      } while (r == ncclInProgress);
    }
    if (r != ncclSuccess) {
      nccl().CommAbort(ctx->comm);
      ctx->comm = nullptr;
      ctx->world = 1;
      return fail(TG_ERR_COMM, "ncclAllGather: %s; communicator aborted",
                  r == ncclInProgress ? "timeout" : nccl().GetErrorString(r));
    }
  } else {
    TG_CUDA(cudaMemcpyAsync(ctx->recv, ctx->records, count * 4, cudaMemcpyDeviceToDevice,
                            ctx->stream));
  }
  tg::GatherMergeParams g{};
  g.records = ctx->recv;
  g.out = dout;
  g.world = ctx->world;
  g.B = n_seqs;
  g.n_head = d.n_head;
  g.head_dim = d.head_dim;
  TG_TRY(commit_inputs(ctx));
  cudaError_t e = tg::launch_gather_merge(g, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "gather merge: %s", cudaGetErrorString(e));
  ctx->launches++;
  return TG_OK;
}
}  // namespace

int tg_attention_splitkv(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                         const float* q, const int32_t* past_len, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !past_len || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(past_len, n_seqs, kv->global_ctx, "past_len"));
  const size_t qb = (size_t)n_seqs * kv->d.n_head * kv->d.head_dim * 4;
  const void *dq = nullptr, *dp = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, q, qb, &dq));
  TG_TRY(stage_in(ctx, past_len, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout));
  TG_TRY(splitkv_core(ctx, kv, layer, n_seqs, const_cast<float*>(static_cast<const float*>(dq)),
                      nullptr, nullptr, static_cast<const int*>(dp), static_cast<float*>(dout),
                      false, preload_allowed(ctx, kv, layer)));
  return finish_call(ctx);
}

int tg_attention_records(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                         const float* q, const int32_t* past_len, float* records) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !past_len || !records) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(past_len, n_seqs, kv->global_ctx, "past_len"));
  const int rf = tg::record_floats(kv->d.n_head, kv->d.head_dim);
  const size_t qb = (size_t)n_seqs * kv->d.n_head * kv->d.head_dim * 4;
  const void *dq = nullptr, *dp = nullptr;
  void* drec = nullptr;
  TG_TRY(stage_in(ctx, q, qb, &dq));
  TG_TRY(stage_in(ctx, past_len, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, records, (size_t)n_seqs * rf * 4, false, &drec));
  if (mma_eligible(kv)) {
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, static_cast<const float*>(dq), nullptr, nullptr,
                     nullptr, static_cast<const int*>(dp), nullptr, static_cast<float*>(drec), 1,
                     false, false, nullptr, preload_allowed(ctx, kv, layer)));
    return finish_call(ctx);
  }
  TG_TRY(ensure_buf(ctx, &ctx->records, &ctx->rec_cap, (size_t)n_seqs * rf));
  TG_TRY(run_decode(ctx, kv, layer, n_seqs, static_cast<const float*>(dq),
                    static_cast<const int*>(dp), 0, nullptr, 1));
  TG_CUDA(cudaMemcpyAsync(drec, ctx->records, (size_t)n_seqs * rf * 4, cudaMemcpyDeviceToDevice,
                          ctx->stream));
  return finish_call(ctx);
}

int tg_merge_records(tg_context* ctx, int n_parts, int n_seqs, int n_head, int head_dim,
                     const float* records, float* out) {
  TG_TRY(set_device(ctx));
  if (n_parts <= 0 || n_seqs < 0 || !records || !out)
    return fail(TG_ERR_INVALID_ARG, "merge_records: bad arguments");
  TG_TRY(check_shape(n_head, 1, head_dim));
  if (n_seqs == 0) return TG_OK;
  const int rf = tg::record_floats(n_head, head_dim);
  const void* drec = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, records, (size_t)n_parts * n_seqs * rf * 4, &drec));
  TG_TRY(stage_out(ctx, out, (size_t)n_seqs * n_head * head_dim * 4, false, &dout));
  tg::GatherMergeParams g{};
  g.records = static_cast<const float*>(drec);
  g.out = static_cast<float*>(dout);
  g.world = n_parts;
  g.B = n_seqs;
  g.n_head = n_head;
  g.head_dim = head_dim;
  TG_TRY(commit_inputs(ctx));
  cudaError_t e = tg::launch_gather_merge(g, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "gather merge: %s", cudaGetErrorString(e));
  ctx->launches++;
  return finish_call(ctx);
}

int tg_decode_layer_splitkv(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, float* q,
                            float* k_new, const float* v_new, const int32_t* pos, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !k_new || !v_new || !pos || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_host_pos(pos, n_seqs, kv->global_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  const size_t qb = (size_t)n_seqs * d.n_head * d.head_dim * 4;
  const size_t kb = (size_t)n_seqs * kv->row_elems * 4;
  void *dq = nullptr, *dk = nullptr, *dout = nullptr;
  const void *dv = nullptr, *dp = nullptr, *dq_in = nullptr, *dk_in = nullptr, *dout_in = nullptr;
  // The tensor-core path reads staged copies and writes pinned host outputs
  // directly; the others work in place.
  const bool split_io = mma_eligible(kv);
  TG_TRY(stage_out(ctx, q, qb, true, &dq, split_io ? &dq_in : nullptr));
  TG_TRY(stage_out(ctx, k_new, kb, true, &dk, split_io ? &dk_in : nullptr));
  TG_TRY(stage_in(ctx, v_new, kb, &dv));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout, split_io ? &dout_in : nullptr));
  if (!split_io) {
    dq_in = dq;
    dk_in = dk;
  }
  TG_TRY(splitkv_core(ctx, kv, layer, n_seqs, const_cast<float*>(static_cast<const float*>(dq_in)),
                      const_cast<float*>(static_cast<const float*>(dk_in)),
                      static_cast<const float*>(dv), static_cast<const int*>(dp),
                      static_cast<float*>(dout), true, preload_allowed(ctx, kv, layer),
                      static_cast<float*>(dq), static_cast<float*>(dk)));
  return finish_call(ctx);
}

int tg_decode_layer_splitkv_x(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                              const tg_qkv_weights* w, const float* x, const int32_t* pos,
                              float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!w || !x || !pos || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_qkv_cols(w->cols));
  TG_TRY(check_host_pos(pos, n_seqs, kv->global_ctx, "pos"));
  const tg_kv_desc& d = kv->d;
  const size_t qb = (size_t)n_seqs * d.n_head * d.head_dim * 4;
  const void *dx = nullptr, *dp = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, x, (size_t)n_seqs * w->cols * 4, &dx));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, out, qb, false, &dout));
  TG_TRY(ensure_buf(ctx, &ctx->qx, &ctx->qx_cap, qb / 4));
  const bool pre = preload_allowed(ctx, kv, layer);
  // Every rank projects q (replicated); only the shard holding pos[s]
  // writes the k / v row.
  TG_TRY(qkv_layer_core(ctx, kv, layer, n_seqs, w, static_cast<const float*>(dx),
                        static_cast<const int*>(dp), ctx->qx));
  TG_TRY(splitkv_core(ctx, kv, layer, n_seqs, ctx->qx, nullptr, nullptr,
                      static_cast<const int*>(dp), static_cast<float*>(dout), false, pre));
  return finish_call(ctx);
}

namespace {
int attention_block(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                    const tg_qkv_weights* w, int o_type, const void* w_o, const float* x,
                    const int32_t* pos, float* hidden, bool split) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!w || !w_o || !x || !pos || !hidden) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0) return TG_OK;
  TG_TRY(check_qkv_cols(w->cols));
  TG_TRY(check_host_pos(pos, n_seqs, split ? kv->global_ctx : kv->d.shard_start + kv->d.max_ctx,
                        "pos"));
  const tg_kv_desc& d = kv->d;
  const int qdim = d.n_head * d.head_dim;
  const size_t qb = (size_t)n_seqs * qdim * 4;
  const void *dx = nullptr, *dp = nullptr;
  void* dh = nullptr;
  TG_TRY(stage_in(ctx, x, (size_t)n_seqs * w->cols * 4, &dx));
  TG_TRY(stage_in(ctx, pos, (size_t)n_seqs * 4, &dp));
  TG_TRY(stage_out(ctx, hidden, qb, true, &dh));
  TG_TRY(ensure_buf(ctx, &ctx->qx, &ctx->qx_cap, qb / 4));
  TG_TRY(ensure_buf(ctx, &ctx->cx, &ctx->cx_cap, qb / 4));
  const bool pre = preload_allowed(ctx, kv, layer);
  TG_TRY(qkv_layer_core(ctx, kv, layer, n_seqs, w, static_cast<const float*>(dx),
                        static_cast<const int*>(dp), ctx->qx));
  if (split) {
    TG_TRY(splitkv_core(ctx, kv, layer, n_seqs, ctx->qx, nullptr, nullptr,
                        static_cast<const int*>(dp), ctx->cx, false, pre));
  } else if (mma_eligible(kv)) {
    TG_TRY(run_fused(ctx, kv, layer, n_seqs, ctx->qx, nullptr, nullptr, nullptr,
                     static_cast<const int*>(dp), ctx->cx, nullptr, 0, false, false, nullptr, pre));
  } else {
    TG_TRY(run_decode(ctx, kv, layer, n_seqs, ctx->qx, static_cast<const int*>(dp), 0, ctx->cx,
                      0));
  }
  TG_TRY(attn_output_core(ctx, n_seqs, o_type, w_o, qdim, qdim, ctx->cx,
                          static_cast<float*>(dh)));
  return finish_call(ctx);
}
}  // namespace

int tg_attention_block(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                       const tg_qkv_weights* w, int o_type, const void* w_o, const float* x,
                       const int32_t* pos, float* hidden) {
  return attention_block(ctx, kv, layer, n_seqs, w, o_type, w_o, x, pos, hidden, false);
}

int tg_attention_block_splitkv(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs,
                               const tg_qkv_weights* w, int o_type, const void* w_o,
                               const float* x, const int32_t* pos, float* hidden) {
  return attention_block(ctx, kv, layer, n_seqs, w, o_type, w_o, x, pos, hidden, true);
}

// ------------------------------------------------ prefill

int tg_prefill_layer(tg_context* ctx, tg_kv_cache* kv, int layer, int n_seqs, int S,
                     const float* q, const float* k, const float* v, float* out) {
  TG_TRY(check_kv_call(ctx, kv, layer, n_seqs));
  if (!q || !k || !v || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  if (n_seqs == 0 || S == 0) return TG_OK;
  const tg_kv_desc& d = kv->d;
  if (d.dtype != TG_DTYPE_BF16 || d.head_dim != 64 || !kv->tmap128_ok)
    return fail(TG_ERR_UNSUPPORTED, "prefill needs a bf16 cache with head_dim 64");
  if (d.shard_start != 0) return fail(TG_ERR_UNSUPPORTED, "prefill on a split-KV shard");
  if (S < 0 || S > d.max_ctx)
    return fail(TG_ERR_INVALID_ARG, "prefill length %d outside [1, %d]", S, d.max_ctx);
  if ((long long)n_seqs * S * d.n_head >= (1LL << 31))
    return fail(TG_ERR_INVALID_ARG, "prefill of %d x %d positions is too large", n_seqs, S);
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(TG_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
  const size_t qd = (size_t)d.n_head * d.head_dim, kd = kv->row_elems;
  const size_t rows = (size_t)n_seqs * S;
  const void *dq = nullptr, *dk = nullptr, *dv = nullptr;
  void* dout = nullptr;
  TG_TRY(stage_in(ctx, q, rows * qd * 4, &dq));
  TG_TRY(stage_in(ctx, k, rows * kd * 4, &dk));
  TG_TRY(stage_in(ctx, v, rows * kd * 4, &dv));
  TG_TRY(stage_out(ctx, out, rows * qd * 4, false, &dout));
  RopeTable* t = nullptr;
  TG_TRY(get_table(ctx, d.rope_base, d.head_dim, S, &t));
  TG_TRY(ensure_buf(ctx, &ctx->qbf, &ctx->qbf_cap, rows * qd));
  TG_TRY(ensure_buf(ctx, &ctx->vh, &ctx->vh_cap, rows * kd));

  tg::PrefillRopeParams rp{};
  rp.q = static_cast<const float*>(dq);
  rp.k = static_cast<const float*>(dk);
  rp.v = static_cast<const float*>(dv);
  rp.cs = t->d;
  rp.q_bf16 = ctx->qbf;
  rp.k_cache = reinterpret_cast<uint16_t*>(static_cast<char*>(kv->k) +
                                           (size_t)layer * kv->layer_elems * kv->esize);
  rp.v_cache = reinterpret_cast<uint16_t*>(static_cast<char*>(kv->v) +
                                           (size_t)layer * kv->layer_elems * kv->esize);
  rp.B = n_seqs;
  rp.S = S;
  rp.n_head = d.n_head;
  rp.n_kv = d.n_kv_head;
  rp.head_dim = d.head_dim;
  rp.max_ctx = d.max_ctx;
  rp.v_f16 = ctx->vh;
  TG_TRY(commit_inputs(ctx));
  cudaError_t e = tg::launch_prefill_rope(rp, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "prefill rope launch: %s", cudaGetErrorString(e));
  ctx->launches++;

  // Rotated q as {64, n_head, rows}: one box = 128 positions of one head.
  alignas(64) CUtensorMap tq;
  cuuint64_t gdim[3] = {64, (cuuint64_t)d.n_head, (cuuint64_t)rows};
  cuuint64_t gstride[2] = {128, (cuuint64_t)d.n_head * 128};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, ctx->qbf, gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TG_ERR_CUDA, "q tensor map rejected (%d)", (int)r);
  // fp16 v as {n_kv*64, rows}: one box = 128 positions of one KV head.
  alignas(64) CUtensorMap tvh;
  cuuint64_t vdim[2] = {(cuuint64_t)kd, (cuuint64_t)rows};
  cuuint64_t vstride[1] = {(cuuint64_t)kd * 2};
  cuuint32_t vbox[2] = {64, 128};
  cuuint32_t vestr[2] = {1, 1};
  r = enc(&tvh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ctx->vh, vdim, vstride, vbox, vestr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TG_ERR_CUDA, "v tensor map rejected (%d)", (int)r);
  tg::PrefillParams pp{};
  pp.out = static_cast<float*>(dout);
  pp.err = ctx->d_err;
  pp.row0 = (long long)layer * d.n_seqs * d.max_ctx;
  pp.B = n_seqs;
  pp.S = S;
  pp.n_head = d.n_head;
  pp.n_kv = d.n_kv_head;
  pp.group = d.n_head / d.n_kv_head;
  pp.max_ctx = d.max_ctx;
  pp.n_qt = (S + 127) / 128;
  pp.scale_log2 = kLog2e / sqrtf((float)d.head_dim);
  const long long items = (long long)n_seqs * d.n_head * ((pp.n_qt + 1) / 2);  // tile pairs
  const int grid = (int)(items < ctx->num_sms ? items : ctx->num_sms);
  cudaEvent_t ev_stop = nullptr;
  TG_TRY(prof_begin(ctx, TG_PROFILE_ATTENTION, &ev_stop));
  e = tg::launch_prefill_attn(tq, kv->tmk128, tvh, pp, grid, ctx->stream);
  if (e != cudaSuccess) return fail(TG_ERR_CUDA, "prefill attention launch: %s", cudaGetErrorString(e));
  ctx->launches++;
  TG_TRY(prof_end(ctx, ev_stop));
  return finish_call(ctx);
}

// ------------------------------------------------ introspection

int tg_launch_count(tg_context* ctx, long long* out) {
  if (!ctx || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  *out = ctx->launches;
  return TG_OK;
}

int tg_profile_enable(tg_context* ctx, int on) {
  TG_TRY(set_device(ctx));
  if (on < 0 || on > (TG_PROFILE_ATTENTION | TG_PROFILE_PROJECTION | TG_PROFILE_STAMPS))
    return fail(TG_ERR_INVALID_ARG, "profile_enable: unknown mask %d", on);
  if ((on & TG_PROFILE_STAMPS) && !ctx->stamps) {
    if (ctx->capturing) return fail(TG_ERR_STATE, "enable stamps before graph capture");
    const size_t words =
        (size_t)TG_STAMP_LAUNCHES * tg::kStampRowsPerSm * ctx->num_sms * tg::kStampsPerCta;
    TG_CUDA(cudaMalloc(&ctx->stamps, words * sizeof(unsigned long long)));
    TG_CUDA(cudaMemsetAsync(ctx->stamps, 0, words * sizeof(unsigned long long), ctx->stream));
    ctx->stamp_cap = TG_STAMP_LAUNCHES;
  }
  ctx->prof_on = on;
  if (on) {  // disabling keeps the record (a graph may replay it)
    ctx->prof_used = 0;
    if (on & TG_PROFILE_STAMPS) ctx->stamp_used = 0;
  }
  return TG_OK;
}

int tg_profile_read_stamps(tg_context* ctx, unsigned long long* out, size_t cap_words,
                           int* n_launches, int* rows) {
  TG_TRY(set_device(ctx));
  if (!out || !n_launches || !rows) return fail(TG_ERR_INVALID_ARG, "null argument");
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
  *n_launches = ctx->stamp_used;
  *rows = tg::kStampRowsPerSm * ctx->num_sms;
  size_t words = (size_t)ctx->stamp_used * (*rows) * tg::kStampsPerCta;
  if (words > cap_words) words = cap_words;
  if (words)
    TG_CUDA(cudaMemcpy(out, ctx->stamps, words * sizeof(unsigned long long),
                       cudaMemcpyDeviceToHost));
  return TG_OK;
}

int tg_profile_read(tg_context* ctx, double* total_ms, long long* launches) {
  TG_TRY(set_device(ctx));
  if (!total_ms || !launches) return fail(TG_ERR_INVALID_ARG, "null argument");
  TG_CUDA(cudaStreamSynchronize(ctx->stream));
  double sum = 0.0;
  for (size_t i = 0; i + 1 < ctx->prof_used; i += 2) {
    float ms = 0.f;
    TG_CUDA(cudaEventElapsedTime(&ms, ctx->prof_ev[i], ctx->prof_ev[i + 1]));
    sum += ms;
  }
  *total_ms = sum;
  *launches = (long long)(ctx->prof_used / 2);
  return TG_OK;
}

int tg_kv_uses_tensor_cores(tg_kv_cache* kv, int* out) {
  if (!kv || !out) return fail(TG_ERR_INVALID_ARG, "null argument");
  *out = mma_eligible(kv) ? 1 : 0;
  return TG_OK;
}

}  // extern "C"

namespace tg {
// Records the message tg_last_error() returns on this thread, for entry
// points implemented in other files of the library.
int set_last_error(int code, const char* msg) {
  t_err = msg;
  return code;
}

int context_device(tg_context* ctx, int* device) {
  if (!ctx || !device) return fail(TG_ERR_INVALID_ARG, "null context");
  *device = ctx->device;
  return TG_OK;
}
}  // namespace tg
