// tg_shared.h -- structures and index arithmetic shared by host and device
// code of the decode-attention path.
//
// Work decomposition ("flat tile space").  For one layer, sequence s
// attends over n_local(s) cache rows of this shard; they form
// ceil(n_local(s) / TILE) tiles.  The tiles of all sequences are laid end
// to end (tile_prefix[s] .. tile_prefix[s+1]) and CTA c of a G-CTA grid
// takes the contiguous range [c*T/G, (c+1)*T/G), T = tile_prefix[B], where
// G = min(launched CTAs, T) so that every range is non-empty.  A
// CTA's range therefore covers at most two partial sequences (its first and
// its last segment); every sequence in between is complete.  A complete
// segment is finished by its CTA; a partial one leaves a partial softmax
// record in slot 2c (first segment) or 2c+1 (last segment), and the merge
// kernel combines the records of each split sequence.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define TG_HD __host__ __device__ __forceinline__
#else
#define TG_HD inline
#endif

namespace tg {

// Device error word values (first error wins).
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrWaitFull = 0x101,   // consumer timed out waiting for a TMA tile
  kDevErrWaitEmpty = 0x102,  // producer timed out waiting for a free stage
  kDevErrBadPos = 0x103,     // position outside the RoPE table / cache
  kDevErrTooManySeqs = 0x104,
  kDevErrPeerTimeout = 0x105,  // a peer GPU's softmax record did not arrive in time
};

// Per-CTA %globaltimer stamps (ns) of a profiled decode step: decode CTAs
// {start, grid dependency released, tile loop done, end}, merge CTAs
// {start, grid dependency released, first record slice stored to the peers
// (mode 2), end}.  One record per decode launch:
// kStampRowsPerSm * num_sms rows of kStampsPerCta (decode CTAs first, the
// merge grid's CTAs from row num_sms on; rows of absent CTAs stay 0).
constexpr int kStampsPerCta = 4;
constexpr int kStampRowsPerSm = 3;

constexpr int kMaxPeers = 8;
// Words per (sequence, head) in the peer exchange: o[64], m, l.
constexpr int kXchgWords = 66;

constexpr float kNegBig = -1.0e30f;  // finite "minus infinity" for m

// Softmax record of one sequence (or one segment of it), all heads:
//   o[n_head][head_dim]  un-normalised sum of 2^(s*log2e - m) * V
//   m[n_head]            running max in log2 units (score * log2(e))
//   l[n_head]            sum of 2^(s*log2e - m)
TG_HD int record_floats(int n_head, int head_dim) {
  return n_head * (head_dim + 2);
}

// CTA that owns flat tile t (G CTAs, T tiles): the largest c with
// floor(c*T/G) <= t.
TG_HD int cta_of_tile(long long t, int G, long long T) {
  return (int)(((t + 1) * (long long)G - 1) / T);
}

TG_HD long long cta_tile_lo(int c, int G, long long T) {
  return (long long)c * T / G;
}

// Number of cache rows of this shard that sequence s attends over, given
// the global position of its current token (n_pos = past_len + 1 rows in
// total, the shard holds global rows [shard_start, shard_start + max_ctx)).
TG_HD int local_rows(int past_len, int shard_start, int max_ctx) {
  long long n = (long long)past_len + 1 - shard_start;
  if (n < 0) n = 0;
  if (n > max_ctx) n = max_ctx;
  return (int)n;
}

struct DecodeParams {
  const float* q;        // [B][n_head*head_dim], already rotated
  float* out;            // [B][n_head*head_dim] normalised output (mode 0)
  float* records;        // [B][record_floats] per-sequence records (mode 1)
  const int* past_len;   // [B] global position of each sequence's token
  const void* k;         // layer cache base, [B][max_ctx][n_kv*head_dim]
  const void* v;
  float* part;           // [2*G][record_floats] partial records
  int* sched;            // [B+1] tile prefix written by CTA 0
  int* err;              // device error word
  long long row0;        // TMA row of (this layer, sequence 0, row 0)
  int B, n_head, n_kv, head_dim, group;
  int max_ctx, shard_start;
  float scale_log2;      // log2(e) / sqrt(head_dim)
  int mode;              // 0: normalised output, 1: records (split-KV)
  int past_len_scalar;   // used for every sequence when past_len == null
  int aligned16;         // k and v rows start on 16-byte boundaries
  // Short-cache kernel only (rope != 0): RoPE of q and of the new k row at
  // the sequence's position and the new row's cache-write, fused in.
  int rope;
  float* q_io;           // [B][n_head*head_dim] raw q in, rotated q out
  float* k_io;           // [B][n_kv*head_dim] raw k in, rotated k out
  const float* v_new;    // [B][n_kv*head_dim]
  const float* cs;       // RoPE table [table_len][head_dim] (cos, sin pairs)
  int table_len;
  void* k_cache;         // layer base of the caches (writable views of k / v)
  void* v_cache;
  float* q_wb;           // where the rotated q / k go (null: back into q_io / k_io)
  float* k_wb;
  int split;             // short-cache kernel: CTAs (a cluster) per (sequence, KV head)
  int stage_v;           // short-cache kernel: V rows copied to shared memory with the K loads
};

TG_HD int past_of(const DecodeParams& p, int s) {
  return p.past_len ? p.past_len[s] : p.past_len_scalar;
}

struct MergeParams {
  const float* part;     // partial records of the decode launch
  const int* sched;      // [B+1] tile prefix of that launch
  float* out;            // mode 0
  float* records;        // mode 1
  int B, n_head, head_dim, G, mode;
};

// Final merge of per-rank records after the all-gather (split-KV).
struct GatherMergeParams {
  const float* records;  // [world][B][record_floats]
  float* out;            // [B][n_head*head_dim]
  int world, B, n_head, head_dim;
};

struct RopeParams {
  float* q;              // [B][n_head*head_dim], rotated in place (or null)
  float* k;              // [B][n_kv*head_dim], rotated in place (or null)
  const float* v;        // [B][n_kv*head_dim] (or null)
  const int* pos;        // [B] global positions (device) or null
  int pos_scalar;        // used when pos == null
  const float* cs;       // RoPE table [table_len][head_dim/2][2] = cos, sin
  int table_len;
  void* k_cache;         // layer cache base (null: no cache-write)
  void* v_cache;
  int B, n_head, n_kv, head_dim;
  int max_ctx, shard_start, dtype;  // dtype: 0 f32, 1 bf16
  int* err;
};

// Prefill: RoPE of positions 0..S-1 + bf16 rounding + cache rows.
struct PrefillRopeParams {
  const float* q;        // [B][S][n_head*head_dim] un-rotated
  const float* k;        // [B][S][n_kv*head_dim] un-rotated
  const float* v;        // [B][S][n_kv*head_dim]
  const float* cs;       // RoPE table
  uint16_t* q_bf16;      // [B][S][n_head][head_dim] rotated, bf16 bits
  uint16_t* k_cache;     // layer base of the bf16 cache
  uint16_t* v_cache;
  uint16_t* v_f16;       // [B][S][n_kv*head_dim] v in fp16 bits (the P.V operand)
  int B, S, n_head, n_kv, head_dim, max_ctx;
};

// Prefill: causal attention of positions 0..S-1 over cache rows 0..S-1.
struct PrefillParams {
  float* out;            // [B][S][n_head][64] fp32
  int* err;
  long long row0;        // TMA row of (this layer, sequence 0, row 0)
  int B, S, n_head, n_kv, group, max_ctx, n_qt;
  float scale_log2;
};

// Decode step of one layer in two launches (tg_decode_fused.cu): the decode
// kernel (RoPE, the new K/V row, split-KV attention) and the merge kernel
// (split sequences, the write-back of rotated q / k and, across GPUs, the
// exchange and merge of per-GPU softmax records over peer memory).
struct FusedParams {
  const float* q_in;       // [B][n_head*64] raw (rope) or already rotated
  float* q_out;            // rotated q written by the CTA finishing a sequence (or null)
  float* k_io;             // [B][n_kv*64] raw new k (new_row)
  float* k_out;            // [B][n_kv*64] rotated k (k_io, or a separate buffer)
  const float* v_new;      // [B][n_kv*64] new v (new_row)
  const int* pos;          // [B] global position of each sequence's current token
  const float* cs;         // RoPE table [table_len][64] (cos, sin pairs)
  int table_len;
  uint16_t* kc_layer;      // layer base of the bf16 caches (new-row writes)
  uint16_t* vc_layer;
  float* out;              // [B][n_head*64] normalised output (modes 0, 2)
  float* records;          // [B][record_floats] (mode 1)
  float* part;             // [2*G][record_floats] partial records
  int* sched;              // [B+1] tile prefix (written by CTA 0)
  int* err;
  long long row0;
  int B, n_head, n_kv, group, max_ctx, shard_start;
  float scale_log2;
  int mode;                // 0 output, 1 records, 2 peer exchange + output
  int rope, new_row;
  int grid;                // CTAs of the decode launch (merge kernel)
  int prefetch;            // L2 prefetch of tiles before the grid-dependency wait
  // Tiles may be loaded into the ring before the grid-dependency wait: no
  // kernel that can still be running writes this layer's cache rows, except
  // the new rows at pos[] when new_row == 0 (the tile holding such a row is
  // loaded after the wait).
  int preload;
  long long wait_ns;       // bound of the in-kernel waits for peer records
  unsigned long long* stamps;  // this launch's stamp record, or null
  // mode 2
  int world, rank, b_cap;  // receive buffers hold b_cap sequences
  // Receive words [2][world][b_cap][n_head][kXchgWords] on this GPU and
  // mapped from every peer: each word = (epoch tag << 32) | float bits.
  unsigned long long* xchg_local;
  unsigned long long* xchg_peer[kMaxPeers];
  unsigned* epoch;         // exchange launches on this GPU (advanced by the decode kernel)
};


// Q/K/V projection of one layer (tg_qkv.cu): y_m = W_m x (+ bias) for the
// three weight matrices m = 0 (q), 1 (k), 2 (v) and B input vectors, with
// weights in the model file's 32-element blocks (GGML Q5_0 / Q8_0).  Mode 0
// writes y_m; mode 2 adds W_m x to y_m (the attn_output matvec and its
// residual add); mode 1 is the layer step of tmac_gguf.cpp:1067-1091: bias,
// RoPE of q and k at pos[s], the k / v rows into the cache, rotated q out.
constexpr int kWTypeQ5_0 = 6;   // 22-byte blocks: fp16 d, 32 high bits, 16 nibble bytes
constexpr int kWTypeQ8_0 = 8;   // 34-byte blocks: fp16 d, 32 int8
constexpr int kQkvRows = 8;     // weight rows per CTA (one warp each)
constexpr int kQkvSeqs = 64;    // sequences per CTA (grid.y covers the batch)
constexpr int kQkvGemmRows = 16;  // batched path: rows per CTA (4 per warp)
constexpr int kQkvGemmMinB = 9;   // batches from this size take the batched path

TG_HD int wtype_block_bytes(int t) {
  return t == kWTypeQ5_0 ? 22 : (t == kWTypeQ8_0 ? 34 : 0);
}

struct QkvParams {
  const uint8_t* w[3];     // row-major rows of cols/32 blocks
  const float* bias[3];    // or null (a model without that bias)
  float* y[3];             // modes 0 / 2: [B][rows[m]]
  int wtype[3];
  int rows[3];             // 0 rows: matrix absent
  int tiles[3];            // CTAs of each matrix: ceil(rows / rows per CTA of the path)
  int cols;                // inputs, a multiple of 32
  const float* x;          // [B][cols]
  int B;
  int mode;
  // mode 1
  float* q_out;            // [B][rows[0]] rotated q
  float* k_out;            // optional [B][rows[1]]: the rotated k row
  float* v_out;            // optional [B][rows[2]]: the v row
  const int* pos;          // [B] global position of each sequence's token
  const float* cs;         // RoPE table [table_len][head_dim] (cos, sin pairs)
  int table_len, head_dim;
  void* k_cache;           // layer base of the caches, [n_seqs][max_ctx][rows[1]]
  void* v_cache;
  int dtype, max_ctx, shard_start;
  int* err;
};

}  // namespace tg
