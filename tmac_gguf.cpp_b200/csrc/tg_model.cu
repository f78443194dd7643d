// tg_model.cu -- the TMAC model-file loader (host code over the device
// allocator): load_tmac (tmac_gguf.cpp:1372-1425) and get_tensor_info
// (:417-422) for device-resident weights.
//
// The reference reads every tensor into one 512 MB host "DDR" region.  Here
// the file is read twice: a first pass over the headers (seeking past the
// data) sizes one device allocation with every tensor at a 256-byte aligned
// offset; a second pass streams the data through two page-locked staging
// buffers into it, so that reading the next chunk from the file overlaps the
// host-to-device copy of the previous one.  The table keeps what load_tmac
// keeps (name truncated to 127 characters, rows, cols, type, n_bytes) plus
// the device address.  There is no size cap: a B200 holds far more than
// 512 MB.  Like load_tmac, the magic is read but not checked.
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <string>
#include <unordered_map>
#include <vector>

#include "tg_cuda_backend.h"
#include "tg_internal.h"

struct tg_model {
  tg_context* ctx = nullptr;
  int device = 0;
  char* dev = nullptr;
  size_t bytes = 0;
  struct Entry {
    char name[128];
    uint64_t rows, cols, n_bytes;
    uint32_t type;
    size_t offset;       // in the device allocation
    long long file_pos;  // of the data in the file
  };
  std::vector<Entry> tensors;
  std::unordered_map<std::string, size_t> index;  // first tensor of each name
};

namespace {

constexpr size_t kAlign = 256;
constexpr size_t kChunk = 32u << 20;  // staging chunk

int model_fail(int code, const char* msg, const char* arg) {
  char buf[512];
  snprintf(buf, sizeof(buf), "%s%s", msg, arg ? arg : "");
  return tg::set_last_error(code, buf);
}

bool read_exact(FILE* f, void* dst, size_t n) { return fread(dst, 1, n, f) == n; }

void fill_info(const tg_model* m, size_t i, tg_tensor_info* out) {
  const tg_model::Entry& e = m->tensors[i];
  out->name = e.name;
  out->rows = e.rows;
  out->cols = e.cols;
  out->n_bytes = e.n_bytes;
  out->type = e.type;
  out->data = m->dev + e.offset;
}

}  // namespace

extern "C" {

int tg_model_load_tmac(tg_context* ctx, const char* path, tg_model** out) {
  if (!ctx || !path || !out) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  *out = nullptr;
  int dev = 0;
  if (tg::context_device(ctx, &dev) != TG_OK) return TG_ERR_INVALID_ARG;
  if (cudaSetDevice(dev) != cudaSuccess) return model_fail(TG_ERR_CUDA, "model: cudaSetDevice", nullptr);
  FILE* f = fopen(path, "rb");
  if (!f) return model_fail(TG_ERR_INVALID_ARG, "model: cannot open ", path);
  tg_model* m = new tg_model;
  m->ctx = ctx;
  m->device = dev;
  int st = TG_OK;
  char* stage[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t s = nullptr;
  do {
    // Pass 1: headers.  A tensor header takes at least 36 bytes, which
    // bounds the count a file of this size can hold.
    long long file_size = -1;
    if (fseek(f, 0, SEEK_END) == 0) file_size = ftell(f);
    if (file_size < 0 || fseek(f, 0, SEEK_SET) != 0) {
      st = model_fail(TG_ERR_INVALID_ARG, "model: cannot seek in ", path);
      break;
    }
    uint8_t magic[4];
    uint64_t n = 0;
    if (!read_exact(f, magic, 4) || !read_exact(f, &n, 8) || n > (uint64_t)file_size / 36) {
      st = model_fail(TG_ERR_INVALID_ARG, "model: truncated header in ", path);
      break;
    }
    m->tensors.resize(n);
    size_t off = 0;
    for (uint64_t i = 0; i < n && st == TG_OK; ++i) {
      tg_model::Entry& e = m->tensors[i];
      uint64_t name_len = 0;
      if (!read_exact(f, &name_len, 8)) {
        st = model_fail(TG_ERR_INVALID_ARG, "model: truncated tensor header in ", path);
        break;
      }
      const uint64_t keep = name_len < 128 ? name_len : 127;
      memset(e.name, 0, sizeof(e.name));
      if (!read_exact(f, e.name, keep) ||
          (name_len > keep && fseek(f, (long)(name_len - keep), SEEK_CUR) != 0) ||
          !read_exact(f, &e.rows, 8) || !read_exact(f, &e.cols, 8) || !read_exact(f, &e.type, 4) ||
          !read_exact(f, &e.n_bytes, 8)) {
        st = model_fail(TG_ERR_INVALID_ARG, "model: truncated tensor header in ", path);
        break;
      }
      e.file_pos = ftell(f);
      if (fseek(f, (long)e.n_bytes, SEEK_CUR) != 0) {
        st = model_fail(TG_ERR_INVALID_ARG, "model: truncated tensor data in ", path);
        break;
      }
      e.offset = off;
      off += (e.n_bytes + kAlign - 1) / kAlign * kAlign;
    }
    if (st != TG_OK) break;
    // The data must really be there (fseek past the end succeeds).
    if (n > 0) {
      const tg_model::Entry& last = m->tensors.back();
      if (fseek(f, 0, SEEK_END) != 0 || ftell(f) < last.file_pos + (long long)last.n_bytes) {
        st = model_fail(TG_ERR_INVALID_ARG, "model: truncated tensor data in ", path);
        break;
      }
    }
    m->bytes = off;
    if (off && cudaMalloc(&m->dev, off) != cudaSuccess) {
      cudaGetLastError();
      st = model_fail(TG_ERR_OUT_OF_MEMORY, "model: device allocation failed for ", path);
      break;
    }
    // Pass 2: data, through two page-locked chunks.
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMallocHost(&stage[0], kChunk) != cudaSuccess ||
        cudaMallocHost(&stage[1], kChunk) != cudaSuccess ||
        cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      st = model_fail(TG_ERR_CUDA, "model: staging setup failed", nullptr);
      break;
    }
    int b = 0;
    bool used[2] = {false, false};
    for (uint64_t i = 0; i < n && st == TG_OK; ++i) {
      const tg_model::Entry& e = m->tensors[i];
      if (fseek(f, (long)e.file_pos, SEEK_SET) != 0) {
        st = model_fail(TG_ERR_INVALID_ARG, "model: seek failed in ", path);
        break;
      }
      for (uint64_t done_b = 0; done_b < e.n_bytes;) {
        const size_t len = (size_t)((e.n_bytes - done_b) < kChunk ? (e.n_bytes - done_b) : kChunk);
        if (used[b] && cudaEventSynchronize(done[b]) != cudaSuccess) {
          st = model_fail(TG_ERR_CUDA, "model: copy failed", nullptr);
          break;
        }
        if (!read_exact(f, stage[b], len)) {
          st = model_fail(TG_ERR_INVALID_ARG, "model: truncated tensor data in ", path);
          break;
        }
        if (cudaMemcpyAsync(m->dev + e.offset + done_b, stage[b], len, cudaMemcpyHostToDevice, s) !=
                cudaSuccess ||
            cudaEventRecord(done[b], s) != cudaSuccess) {
          st = model_fail(TG_ERR_CUDA, "model: copy failed", nullptr);
          break;
        }
        used[b] = true;
        b ^= 1;
        done_b += len;
      }
    }
    if (st == TG_OK && cudaStreamSynchronize(s) != cudaSuccess)
      st = model_fail(TG_ERR_CUDA, "model: copy failed", nullptr);
  } while (false);
  fclose(f);
  if (s) {
    cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
  }
  for (int i = 0; i < 2; ++i) {
    if (done[i]) cudaEventDestroy(done[i]);
    if (stage[i]) cudaFreeHost(stage[i]);
  }
  if (st != TG_OK) {
    cudaFree(m->dev);
    delete m;
    return st;
  }
  for (size_t i = 0; i < m->tensors.size(); ++i) m->index.emplace(m->tensors[i].name, i);
  *out = m;
  return TG_OK;
}

int tg_model_destroy(tg_model* m) {
  if (!m) return TG_OK;
  cudaSetDevice(m->device);
  cudaFree(m->dev);
  delete m;
  return TG_OK;
}

int tg_model_count(tg_model* m, int* n) {
  if (!m || !n) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  *n = (int)m->tensors.size();
  return TG_OK;
}

int tg_model_tensor_at(tg_model* m, int i, tg_tensor_info* out) {
  if (!m || !out) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  if (i < 0 || (size_t)i >= m->tensors.size())
    return model_fail(TG_ERR_INVALID_ARG, "model: tensor index out of range", nullptr);
  fill_info(m, (size_t)i, out);
  return TG_OK;
}

int tg_model_find(tg_model* m, const char* name, tg_tensor_info* out) {
  if (!m || !name || !out) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  memset(out, 0, sizeof(*out));
  auto it = m->index.find(name);
  if (it != m->index.end()) fill_info(m, it->second, out);
  return TG_OK;
}

int tg_model_read(tg_model* m, int i, void* dst, size_t bytes) {
  if (!m || !dst) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  if (i < 0 || (size_t)i >= m->tensors.size() || bytes > m->tensors[i].n_bytes)
    return model_fail(TG_ERR_INVALID_ARG, "model: bad tensor index or size", nullptr);
  cudaSetDevice(m->device);
  if (cudaMemcpy(dst, m->dev + m->tensors[i].offset, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return model_fail(TG_ERR_CUDA, "model: read failed", nullptr);
  }
  return TG_OK;
}

int tg_model_layer_attention(tg_model* m, int layer, tg_qkv_weights* w, const void** w_o,
                             int* o_type) {
  if (!m || !w) return model_fail(TG_ERR_INVALID_ARG, "model: null argument", nullptr);
  char name[128];
  tg_tensor_info q, k, v, bq, bk, bv, o;
  auto find = [&](const char* what, tg_tensor_info* t) {
    snprintf(name, sizeof(name), "blk.%d.%s", layer, what);
    tg_model_find(m, name, t);
  };
  find("attn_q.weight", &q);
  find("attn_k.weight", &k);
  find("attn_v.weight", &v);
  find("attn_q.bias", &bq);
  find("attn_k.bias", &bk);
  find("attn_v.bias", &bv);
  find("attn_output.weight", &o);
  if (!q.data || !k.data || !v.data)
    return model_fail(TG_ERR_INVALID_ARG, "model: missing attention weights of a layer", nullptr);
  if (q.cols != k.cols || q.cols != v.cols || q.cols > 0x7fffffff)
    return model_fail(TG_ERR_INVALID_ARG, "model: q/k/v weights disagree on their inputs", nullptr);
  memset(w, 0, sizeof(*w));
  w->q_type = (int)q.type;
  w->k_type = (int)k.type;
  w->v_type = (int)v.type;
  w->cols = (int)q.cols;
  w->w_q = q.data;
  w->w_k = k.data;
  w->w_v = v.data;
  // Biases are fp32 (type 0) when the model has them.
  w->b_q = bq.data && bq.type == 0 ? static_cast<const float*>(bq.data) : nullptr;
  w->b_k = bk.data && bk.type == 0 ? static_cast<const float*>(bk.data) : nullptr;
  w->b_v = bv.data && bv.type == 0 ? static_cast<const float*>(bv.data) : nullptr;
  if (w_o) *w_o = o.data;
  if (o_type) *o_type = o.data ? (int)o.type : -1;
  return TG_OK;
}

}  // extern "C"
