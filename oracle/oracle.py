"""ctypes view of the CPU parity oracle -- TEST INFRASTRUCTURE ONLY.

Two libraries are wrapped here:

* ``liboracle.so``: the plain-C restatement (``tg_oracle.c``) of the
  reference's CPU hot path -- RoPE (tmac_gguf.cpp:990-1016), the KV
  cache-write (:1090-1091) and the GQA decode attention (:1093-1128) -- plus
  the seeded input generator shared by every test and benchmark.
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
                f"{REF_SO} is missing: build it with `make -C oracle ref` "
                "where the reference tree is mounted")
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
