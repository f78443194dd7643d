"""Seeded input builders shared by the golden-fixture script and the tests.

Every case is a pure function of (seed, shape), drawn from the oracle's
splitmix64 + Box-Muller stream, so a fixture only records its seeds and the
reference's outputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np

_ORACLE_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..",
                           "..", "oracle")
if _ORACLE_DIR not in sys.path:
    sys.path.insert(0, os.path.abspath(_ORACLE_DIR))
import oracle as O  # noqa: E402

KD = O.N_KV_HEAD * O.HEAD_DIM     # 128: one cache row (both KV heads)
QD = O.N_HEAD * O.HEAD_DIM        # 896: one query / context vector

# tensor tags for derive_seed
T_Q, T_KNEW, T_VNEW, T_KC, T_VC = 1, 2, 3, 4, 5


def decode_inputs(seed: int, pos: int, bf16: bool = False, seq: int = 0,
                  layer: int = 0):
    """Inputs of one decode step at position pos: un-roped q and k_new, v_new,
    and cache rows 0..pos-1 (row pos is written by the step).  Caches are
    allocated with pos+1 rows.  bf16=True rounds the cache rows and the new
    v row to bf16 (the roped k row is rounded by the step itself)."""
    gen = O.normal_bf16 if bf16 else O.normal
    q = O.normal(O.derive_seed(seed, layer, seq, T_Q), QD)
    k_new = O.normal(O.derive_seed(seed, layer, seq, T_KNEW), KD)
    v_new = gen(O.derive_seed(seed, layer, seq, T_VNEW), KD)
    k_cache = np.zeros((pos + 1, KD), dtype=np.float32)
    v_cache = np.zeros((pos + 1, KD), dtype=np.float32)
    if pos > 0:
        k_cache[:pos] = gen(O.derive_seed(seed, layer, seq, T_KC),
                            pos * KD).reshape(pos, KD)
        v_cache[:pos] = gen(O.derive_seed(seed, layer, seq, T_VC),
                            pos * KD).reshape(pos, KD)
    return q, k_new, v_new, k_cache, v_cache


def oracle_decode(seed: int, pos: int, bf16: bool = False, seq: int = 0,
                  layer: int = 0):
    """Run the oracle's decode step on decode_inputs.  For bf16 the roped k
    row is rounded to bf16 before it enters the cache, as the bf16 cache
    stores it.  Returns (q_roped, k_roped, v_new, k_cache, v_cache, ctx)."""
    q, k_new, v_new, kc, vc = decode_inputs(seed, pos, bf16, seq, layer)
    q = q.copy()
    k = k_new.copy()
    O.lib().tgo_apply_rope(q, k, O.N_HEAD, O.N_KV_HEAD, O.HEAD_DIM, pos,
                           O.ROPE_BASE)
    k_row = O.round_bf16(k) if bf16 else k
    kc[pos] = k_row
    vc[pos] = v_new
    ctx = O.attention(q, kc, vc, pos)
    return q, k, v_new, kc, vc, ctx


def prefill_raw(seed: int, S: int, seq: int = 0):
    """Un-rotated fp32 prefill inputs q [S][896], k/v [S][128] ~ N(0,1)."""
    q = O.normal(O.derive_seed(seed, 0, seq, T_Q), S * QD).reshape(S, QD)
    k = O.normal(O.derive_seed(seed, 0, seq, T_KNEW), S * KD).reshape(S, KD)
    v = O.normal(O.derive_seed(seed, 0, seq, T_VNEW), S * KD).reshape(S, KD)
    return q, k, v


def prefill_inputs(seed: int, S: int, seq: int = 0):
    """Prefill inputs: q/k/v ~ N(0,1), RoPE applied to q and k in binary32 at
    positions 0..S-1 with the reference formula, then all three rounded to
    bf16.  Returns float32 arrays q [S][896], k/v [S][128] (bf16 values)."""
    q, k, v = prefill_raw(seed, S, seq)
    q = q.copy()
    k = k.copy()
    for t in range(S):
        q[t] = O.rope_heads(q[t], O.N_HEAD, O.HEAD_DIM, t)
        k[t] = O.rope_heads(k[t], O.N_KV_HEAD, O.HEAD_DIM, t)
    return O.round_bf16(q), O.round_bf16(k), O.round_bf16(v)


# tensor tags of the Q/K/V projection inputs
T_WQ, T_WK, T_WV, T_BQ, T_BK, T_BV, T_X, T_WO, T_H = 21, 22, 23, 24, 25, 26, 27, 28, 29
# d scale per weight type: keeps |q|, |k|, |v| of order 1 for N(0,1) inputs.
D_SCALE = {O.TYPE_Q5_0: 0.004, O.TYPE_Q8_0: 0.0005}


def qkv_weights(seed: int, v_type: int = O.TYPE_Q5_0, bias: bool = True,
                layer: int = 0, cols: int = QD):
    """One layer's projection weights as the model file holds them: W_q
    (QD rows) and W_k (KD rows) in Q5_0, W_v (KD rows) in v_type, each row
    of `cols` inputs in 32-element blocks; fp32 biases ~ 0.1 N(0,1), or None
    (a model without biases).  Returns (wq, wk, wv, bq, bk, bv)."""
    wq = O.qblocks(O.TYPE_Q5_0, O.derive_seed(seed, layer, 0, T_WQ), QD, cols,
                   D_SCALE[O.TYPE_Q5_0])
    wk = O.qblocks(O.TYPE_Q5_0, O.derive_seed(seed, layer, 0, T_WK), KD, cols,
                   D_SCALE[O.TYPE_Q5_0])
    wv = O.qblocks(v_type, O.derive_seed(seed, layer, 0, T_WV), KD, cols,
                   D_SCALE[v_type])
    if not bias:
        return wq, wk, wv, None, None, None
    bq = (O.normal(O.derive_seed(seed, layer, 0, T_BQ), QD) * np.float32(0.1)).astype(np.float32)
    bk = (O.normal(O.derive_seed(seed, layer, 0, T_BK), KD) * np.float32(0.1)).astype(np.float32)
    bv = (O.normal(O.derive_seed(seed, layer, 0, T_BV), KD) * np.float32(0.1)).astype(np.float32)
    return wq, wk, wv, bq, bk, bv


def qkv_x(seed: int, n_seqs: int = 1, cols: int = QD, layer: int = 0):
    """Normed hidden states x [n_seqs][cols] ~ N(0,1)."""
    return O.normal(O.derive_seed(seed, layer, 0, T_X), n_seqs * cols).reshape(n_seqs, cols)


def attn_output_weight(seed: int, o_type: int = O.TYPE_Q5_0, layer: int = 0):
    """W_o (QD x QD) in o_type blocks."""
    return O.qblocks(o_type, O.derive_seed(seed, layer, 0, T_WO), QD, QD, D_SCALE[o_type])


def residual_in(seed: int, n_seqs: int = 1, layer: int = 0):
    """The residual stream entering the layer, [n_seqs][QD] ~ N(0,1)."""
    return O.normal(O.derive_seed(seed, layer, 0, T_H), n_seqs * QD).reshape(n_seqs, QD)
