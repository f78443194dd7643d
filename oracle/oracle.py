"""ctypes view of the CPU parity oracle -- TEST INFRASTRUCTURE ONLY.

Two libraries are wrapped here:

* ``liboracle.so``: the plain-C restatement (``tg_oracle.c``) of the
  reference's CPU hot path -- RoPE (tmac_gguf.cpp:990-1016), the KV
  cache-write (:1090-1091), the GQA decode attention (:1093-1128) and the
  quantized Q/K/V projection with its bias adds (:220-248, :311-328,
  :402-415, :476-513, :1046-1081) -- plus the seeded input generators
  shared by every test and benchmark.
* ``_ref/libref.so``: the reference's own lines of that path, compiled from
  the reference tree by ``oracle/Makefile``.  The restatement is pinned
  bit-for-bit against it (tests/test_oracle.py) and against the golden
  fixtures it produced (tests/golden/).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs may import
this module; the CUDA product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref.so")

# The reference's model shape (tmac_gguf.cpp:163-172) and RoPE base (:991).
N_HEAD, N_KV_HEAD, HEAD_DIM = 14, 2, 64
ROPE_BASE = 1000000.0

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")

# Weight types (tmac_gguf.cpp:177-182) and bytes per 32-element block.
TYPE_F32, TYPE_Q5_0, TYPE_Q8_0 = 0, 6, 8
BLOCK_BYTES = {TYPE_Q5_0: 22, TYPE_Q8_0: 34}

_lib = None
_ref = None


def build() -> None:
    """Compile liboracle.so (and _ref/libref.so when the reference tree is
    present) with oracle/Makefile."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        L.tgo_splitmix64.restype = C.c_uint64
        L.tgo_splitmix64.argtypes = [C.POINTER(C.c_uint64)]
        L.tgo_fill_normal.argtypes = [C.c_uint64, _f32p, C.c_size_t]
        L.tgo_fill_normal_bf16.argtypes = [C.c_uint64, _f32p, C.c_size_t]
        L.tgo_pack_bf16.argtypes = [_f32p, _u16p, C.c_size_t]
        L.tgo_round_bf16_inplace.argtypes = [_f32p, C.c_size_t]
        L.tgo_rope_heads.argtypes = [_f32p, C.c_int, C.c_int, C.c_int, C.c_float]
        L.tgo_apply_rope.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int,
                                     C.c_int, C.c_float]
        L.tgo_rope_cos_sin.argtypes = [C.c_int, C.c_int, C.c_float, _f32p]
        L.tgo_attention.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int,
                                    C.c_int, C.c_int, C.c_int, _f32p]
        L.tgo_decode_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                      C.c_int, C.c_int, C.c_int, C.c_int,
                                      C.c_float, _f32p]
        L.tgo_prefill_causal.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_int,
                                         C.c_int]
        L.tgo_attention_units_mt.restype = C.c_int
        L.tgo_attention_units_mt.argtypes = [
            C.c_int, C.c_void_p, C.c_size_t, C.POINTER(C.c_void_p),
            C.POINTER(C.c_void_p), _i32p, C.c_void_p, C.c_int, C.c_int,
            C.c_int, C.c_int]
        L.tgo_partial_head.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int,
                                       C.c_int, C.c_int, C.c_int, C.c_int,
                                       C.POINTER(C.c_float),
                                       C.POINTER(C.c_float), _f32p, _f32p]
        L.tgo_merge_partials.argtypes = [C.c_int, _f32p, _f32p, _f32p, C.c_int,
                                         _f32p]
        L.tgo_f16_to_f32.restype = C.c_float
        L.tgo_f16_to_f32.argtypes = [C.c_uint16]
        L.tgo_dequant.restype = C.c_float
        L.tgo_dequant.argtypes = [C.c_int, _u8p, C.c_uint64]
        L.tgo_matmul_q.argtypes = [C.c_int, _u8p, _f32p, _f32p, C.c_int, C.c_int]
        L.tgo_qkv_step.argtypes = [C.c_int, _u8p, C.c_int, _u8p, C.c_int, _u8p,
                                   C.c_void_p, C.c_void_p, C.c_void_p, _f32p,
                                   _f32p, _f32p, _f32p, C.c_int, C.c_int,
                                   C.c_int, C.c_int, C.c_int, C.c_float,
                                   C.c_void_p, C.c_void_p]
        L.tgo_fill_qblocks.argtypes = [C.c_int, C.c_uint64, _u8p, C.c_size_t,
                                       C.c_float]
        L.tgo_attn_output.argtypes = [C.c_int, _u8p, _f32p, _f32p, _f32p, C.c_int,
                                      C.c_int, C.c_void_p]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    """The reference's own hot-path build (oracle/_ref/libref.so)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(
                f"{REF_SO} is missing: build it with `make -C oracle ref "
                "REF_DIR=<checkout of the reference>`")
        R = C.CDLL(REF_SO)
        R.tgref_max_ctx.restype = C.c_int
        R.tgref_apply_rope.argtypes = [_f32p, _f32p, C.c_int]
        R.tgref_cache_write_attention.argtypes = [_f32p, _f32p, _f32p, _f32p,
                                                  _f32p, _f32p, C.c_int]
        R.tgref_decode_step.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p,
                                        _f32p, C.c_int]
        R.tgref_attention_units_mt.restype = C.c_int
        R.tgref_attention_units_mt.argtypes = [
            C.c_int, C.c_void_p, C.c_long, C.POINTER(C.c_void_p),
            C.POINTER(C.c_void_p), _i32p, C.c_void_p, C.c_int]
        R.tgref_f16_to_f32.restype = C.c_float
        R.tgref_f16_to_f32.argtypes = [C.c_uint16]
        R.tgref_matmul.argtypes = [C.c_int, _u8p, _f32p, _f32p, C.c_int, C.c_int]
        R.tgref_attention_block.restype = C.c_int
        R.tgref_attention_block.argtypes = [
            C.c_int, _u8p, C.c_int, _u8p, C.c_int, _u8p, C.c_void_p, C.c_void_p,
            C.c_void_p, C.c_int, _u8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
            _f32p, _f32p, _f32p, C.c_int]
        R.tgref_load_tmac.restype = C.c_int
        R.tgref_load_tmac.argtypes = [C.c_char_p]
        R.tgref_tmac_count.restype = C.c_int
        R.tgref_tmac_tensor.restype = C.c_int
        R.tgref_tmac_tensor.argtypes = [C.c_int, C.c_char_p, C.POINTER(C.c_uint64),
                                        C.POINTER(C.c_uint64), C.POINTER(C.c_uint32),
                                        C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        R.tgref_tmac_ddr.restype = C.c_void_p
        R.tgref_qkv_layer.restype = C.c_int
        R.tgref_qkv_layer.argtypes = [C.c_int, _u8p, C.c_int, _u8p, C.c_int, _u8p,
                                      C.c_void_p, C.c_void_p, C.c_void_p, _f32p,
                                      _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
                                      C.c_int]
        _ref = R
    return _ref


# ---------------------------------------------------------------- inputs

def normal(seed: int, n: int) -> np.ndarray:
    """N(0,1) float32 stream of length n from splitmix64 + Box-Muller."""
    out = np.empty(int(n), dtype=np.float32)
    lib().tgo_fill_normal(C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), out, out.size)
    return out


def normal_bf16(seed: int, n: int) -> np.ndarray:
    """The same stream rounded to bf16 (RNE) and widened to float32."""
    out = np.empty(int(n), dtype=np.float32)
    lib().tgo_fill_normal_bf16(C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), out,
                               out.size)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().tgo_round_bf16_inplace(y.reshape(-1), y.size)
    return y


def pack_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().tgo_pack_bf16(x.reshape(-1), out.reshape(-1), x.size)
    return out


def qblocks(wtype: int, seed: int, rows: int, cols: int,
            d_scale: float = 0.004) -> np.ndarray:
    """Synthetic weight rows of a block type: uint8 [rows, row_bytes]."""
    nb = rows * (cols // 32)
    out = np.empty(nb * BLOCK_BYTES[wtype], dtype=np.uint8)
    lib().tgo_fill_qblocks(wtype, C.c_uint64(seed & 0xFFFFFFFFFFFFFFFF), out, nb,
                           d_scale)
    return out.reshape(rows, -1)


def derive_seed(seed: int, layer: int, seq: int, tag: int = 0) -> int:
    """Independent sub-stream seed for (layer, sequence, tensor tag)."""
    return (seed ^ (layer << 32) ^ (seq << 8) ^ (tag << 56)) & 0xFFFFFFFFFFFFFFFF


# ---------------------------------------------------------------- oracle ops

def rope_heads(x: np.ndarray, n_heads: int, head_dim: int, pos: int,
               base: float = ROPE_BASE) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().tgo_rope_heads(y.reshape(-1), n_heads, head_dim, pos, base)
    return y


def rope_cos_sin(head_dim: int, pos: int, base: float = ROPE_BASE) -> np.ndarray:
    cs = np.empty(head_dim, dtype=np.float32)
    lib().tgo_rope_cos_sin(head_dim, pos, base, cs)
    return cs


def attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray,
              pos: int, n_head: int = N_HEAD, n_kv_head: int = N_KV_HEAD,
              head_dim: int = HEAD_DIM) -> np.ndarray:
    """tmac_gguf.cpp:1093-1128 over cache rows 0..pos."""
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1)
    k = np.ascontiguousarray(k_cache, dtype=np.float32).reshape(-1)
    v = np.ascontiguousarray(v_cache, dtype=np.float32).reshape(-1)
    assert k.size >= (pos + 1) * n_kv_head * head_dim
    out = np.empty(n_head * head_dim, dtype=np.float32)
    scores = np.empty(pos + 1, dtype=np.float32)
    lib().tgo_attention(q, k, v, out, n_head, n_kv_head, head_dim, pos, scores)
    return out


def decode_step(q, k_new, v_new, k_cache, v_cache, pos, n_head=N_HEAD,
                n_kv_head=N_KV_HEAD, head_dim=HEAD_DIM, base=ROPE_BASE):
    """RoPE + cache-write + attention (tmac_gguf.cpp:1087-1128).  q, k_new,
    k_cache and v_cache are updated in place; returns the context."""
    out = np.empty(n_head * head_dim, dtype=np.float32)
    scores = np.empty(pos + 1, dtype=np.float32)
    lib().tgo_decode_step(q, k_new, np.ascontiguousarray(v_new, np.float32),
                          k_cache.reshape(-1), v_cache.reshape(-1), out,
                          n_head, n_kv_head, head_dim, pos, base, scores)
    return out


def prefill_causal(q, k, v, n_head=N_HEAD, n_kv_head=N_KV_HEAD,
                   head_dim=HEAD_DIM, t_begin=0, t_end=None) -> np.ndarray:
    """Token-by-token causal attention (process_prompt, tmac_gguf.cpp:1621).
    Rows t_begin..t_end-1 of the output are computed; others stay zero."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    S = q.shape[0]
    t_end = S if t_end is None else t_end
    out = np.zeros((S, n_head * head_dim), dtype=np.float32)
    lib().tgo_prefill_causal(q.reshape(-1), k.reshape(-1), v.reshape(-1),
                             out.reshape(-1), S, n_head, n_kv_head, head_dim,
                             t_begin, t_end)
    return out


def _ptr(a):
    return None if a is None else np.ascontiguousarray(a, np.float32).ctypes.data


def matmul_q(wtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """matmul's CPU loop (tmac_gguf.cpp:508-512): y = W x, j-ordered sums."""
    y = np.empty(rows, dtype=np.float32)
    lib().tgo_matmul_q(wtype, np.ascontiguousarray(w, np.uint8).reshape(-1),
                       np.ascontiguousarray(x, np.float32).reshape(-1), y, rows, cols)
    return y


def dequant_rows(wtype: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """The dequantised weight matrix [rows, cols] (tmac_gguf.cpp:240-248,
    :311-328), element by element."""
    flat = np.ascontiguousarray(w, np.uint8).reshape(-1)
    L = lib()
    return np.array([L.tgo_dequant(wtype, flat, i) for i in range(rows * cols)],
                    dtype=np.float32).reshape(rows, cols)


def qkv_step(wq, wk, wv, bq, bk, bv, x, pos, q_type=TYPE_Q5_0, k_type=TYPE_Q5_0,
             v_type=TYPE_Q5_0, n_head=N_HEAD, n_kv_head=N_KV_HEAD, head_dim=HEAD_DIM,
             base=ROPE_BASE, k_cache=None, v_cache=None):
    """tmac_gguf.cpp:1046-1091 for one sequence: projections, bias adds,
    RoPE at pos and (when caches are given, updated in place) the
    cache-write.  Returns (q, k, v)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    cols = x.size
    qd, kd = n_head * head_dim, n_kv_head * head_dim
    q = np.empty(qd, np.float32)
    k = np.empty(kd, np.float32)
    v = np.empty(kd, np.float32)
    keep = [np.ascontiguousarray(b, np.float32) if b is not None else None
            for b in (bq, bk, bv)]
    lib().tgo_qkv_step(q_type, np.ascontiguousarray(wq, np.uint8).reshape(-1), k_type,
                       np.ascontiguousarray(wk, np.uint8).reshape(-1), v_type,
                       np.ascontiguousarray(wv, np.uint8).reshape(-1),
                       *[_ptr(b) for b in keep], x, q, k, v, n_head, n_kv_head,
                       head_dim, cols, pos, base,
                       None if k_cache is None else k_cache.ctypes.data,
                       None if v_cache is None else v_cache.ctypes.data)
    return q, k, v


def attn_output(o_type: int, wo, context, original_hidden) -> np.ndarray:
    """tmac_gguf.cpp:1129-1140: original_hidden + W_o context."""
    context = np.ascontiguousarray(context, np.float32).reshape(-1)
    h0 = np.ascontiguousarray(original_hidden, np.float32).reshape(-1)
    out = np.empty_like(h0)
    lib().tgo_attn_output(o_type, np.ascontiguousarray(wo, np.uint8).reshape(-1), context, h0,
                          out, h0.size, context.size, None)
    return out


def attention_units_mt(q: np.ndarray, k_list, v_list, pos, n_threads: int,
                       n_head=N_HEAD, n_kv_head=N_KV_HEAD, head_dim=HEAD_DIM):
    """Multi-threaded oracle over independent (sequence, layer) units."""
    n = len(k_list)
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(n, -1)
    out = np.empty_like(q)
    kp = (C.c_void_p * n)(*[k.ctypes.data for k in k_list])
    vp = (C.c_void_p * n)(*[v.ctypes.data for v in v_list])
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    rc = lib().tgo_attention_units_mt(n, q.ctypes.data, q.shape[1], kp, vp,
                                      pos, out.ctypes.data, n_head, n_kv_head,
                                      head_dim, n_threads)
    if rc != 0:
        raise RuntimeError("tgo_attention_units_mt failed")
    return out


# ---------------------------------------------------------------- reference

def ref_apply_rope(q: np.ndarray, k: np.ndarray, pos: int):
    """The reference's apply_rope (14 q heads, 2 kv heads, 64, base 1e6)."""
    q = np.ascontiguousarray(q, dtype=np.float32).copy()
    k = np.ascontiguousarray(k, dtype=np.float32).copy()
    ref().tgref_apply_rope(q.reshape(-1), k.reshape(-1), pos)
    return q, k


def ref_attention(q, k_cache, v_cache, pos):
    """The reference's tmac_gguf.cpp:1093-1128 (cache rows already hold the
    current token)."""
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(-1).copy()
    k = np.ascontiguousarray(k_cache, dtype=np.float32).reshape(-1).copy()
    v = np.ascontiguousarray(v_cache, dtype=np.float32).reshape(-1).copy()
    kd = N_KV_HEAD * HEAD_DIM
    out = np.empty(N_HEAD * HEAD_DIM, dtype=np.float32)
    k_row = np.ascontiguousarray(k[pos * kd:(pos + 1) * kd])
    v_row = np.ascontiguousarray(v[pos * kd:(pos + 1) * kd])
    ref().tgref_cache_write_attention(q, k_row, v_row, out, k, v, pos)
    return out


def ref_decode_step(q, k_new, v_new, k_cache, v_cache, pos):
    """The reference's decode step (tmac_gguf.cpp:1087-1128), in place on
    q, k_new and the caches; returns the context."""
    out = np.empty(N_HEAD * HEAD_DIM, dtype=np.float32)
    ref().tgref_decode_step(q, k_new, np.ascontiguousarray(v_new, np.float32),
                            out, k_cache.reshape(-1), v_cache.reshape(-1), pos)
    return out


def ref_attention_units_mt(q: np.ndarray, k_list, v_list, pos, n_threads: int):
    n = len(k_list)
    q = np.ascontiguousarray(q, dtype=np.float32).reshape(n, -1)
    out = np.empty_like(q)
    kp = (C.c_void_p * n)(*[k.ctypes.data for k in k_list])
    vp = (C.c_void_p * n)(*[v.ctypes.data for v in v_list])
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    rc = ref().tgref_attention_units_mt(n, q.ctypes.data, q.shape[1], kp, vp,
                                        pos, out.ctypes.data, n_threads)
    if rc != 0:
        raise RuntimeError("tgref_attention_units_mt failed")
    return out


def ref_matmul(wtype: int, w: np.ndarray, x: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """The reference's matmul (tmac_gguf.cpp:476-514, CPU loop)."""
    y = np.empty(rows, dtype=np.float32)
    ref().tgref_matmul(wtype, np.ascontiguousarray(w, np.uint8).reshape(-1),
                       np.ascontiguousarray(x, np.float32).reshape(-1), y, rows, cols)
    return y


def ref_qkv_layer(wq, wk, wv, bq, bk, bv, x, k_cache, v_cache, pos,
                  q_type=TYPE_Q5_0, k_type=TYPE_Q5_0, v_type=TYPE_Q5_0):
    """The reference's tmac_gguf.cpp:1045-1128 for one sequence (Qwen2-0.5B
    shape): returns (q, k, v, context); the caches are updated in place."""
    q = np.empty(N_HEAD * HEAD_DIM, np.float32)
    k = np.empty(N_KV_HEAD * HEAD_DIM, np.float32)
    v = np.empty(N_KV_HEAD * HEAD_DIM, np.float32)
    out = np.empty(N_HEAD * HEAD_DIM, np.float32)
    keep = [np.ascontiguousarray(b, np.float32) if b is not None else None
            for b in (bq, bk, bv)]
    rc = ref().tgref_qkv_layer(q_type, np.ascontiguousarray(wq, np.uint8).reshape(-1),
                               k_type, np.ascontiguousarray(wk, np.uint8).reshape(-1),
                               v_type, np.ascontiguousarray(wv, np.uint8).reshape(-1),
                               *[_ptr(b) for b in keep],
                               np.ascontiguousarray(x, np.float32).reshape(-1), q, k, v,
                               out, k_cache.reshape(-1), v_cache.reshape(-1), pos)
    if rc != 0:
        raise RuntimeError("tgref_qkv_layer failed")
    return q, k, v, out


def ref_attention_block(wq, wk, wv, bq, bk, bv, wo, x, original_hidden, k_cache, v_cache,
                        pos, q_type=TYPE_Q5_0, k_type=TYPE_Q5_0, v_type=TYPE_Q5_0,
                        o_type=TYPE_Q5_0):
    """The reference's tmac_gguf.cpp:1045-1140 for one sequence: returns
    (hidden, q, k, v, context); the caches are updated in place."""
    q = np.empty(N_HEAD * HEAD_DIM, np.float32)
    k = np.empty(N_KV_HEAD * HEAD_DIM, np.float32)
    v = np.empty(N_KV_HEAD * HEAD_DIM, np.float32)
    ctx = np.empty(N_HEAD * HEAD_DIM, np.float32)
    att = np.empty(N_HEAD * HEAD_DIM, np.float32)
    hid = np.empty(N_HEAD * HEAD_DIM, np.float32)
    keep = [np.ascontiguousarray(b, np.float32) if b is not None else None
            for b in (bq, bk, bv)]
    rc = ref().tgref_attention_block(
        q_type, np.ascontiguousarray(wq, np.uint8).reshape(-1), k_type,
        np.ascontiguousarray(wk, np.uint8).reshape(-1), v_type,
        np.ascontiguousarray(wv, np.uint8).reshape(-1), *[_ptr(b) for b in keep], o_type,
        np.ascontiguousarray(wo, np.uint8).reshape(-1),
        np.ascontiguousarray(x, np.float32).reshape(-1),
        np.ascontiguousarray(original_hidden, np.float32).reshape(-1), hid, q, k, v, ctx, att,
        k_cache.reshape(-1), v_cache.reshape(-1), pos)
    if rc != 0:
        raise RuntimeError("tgref_attention_block failed")
    return hid, q, k, v, ctx


def ref_load_tmac(path: str):
    """The reference's load_tmac (tmac_gguf.cpp:1372-1425): returns its
    status and the table it built, a list of (name, rows, cols, type,
    n_bytes, data bytes)."""
    R = ref()
    rc = R.tgref_load_tmac(path.encode())
    table = []
    ddr = R.tgref_tmac_ddr()
    for i in range(R.tgref_tmac_count() if rc == 0 else 0):
        name = C.create_string_buffer(128)
        rows, cols, nb, off = C.c_uint64(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        typ = C.c_uint32()
        R.tgref_tmac_tensor(i, name, C.byref(rows), C.byref(cols), C.byref(typ), C.byref(nb),
                            C.byref(off))
        data = C.string_at(ddr + off.value, nb.value)
        table.append((name.value.decode(), rows.value, cols.value, typ.value, nb.value, data))
    return rc, table
