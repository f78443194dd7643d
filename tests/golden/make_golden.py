"""Generate tests/golden/golden_ref.npz from the reference's own code.

The outputs come from oracle/_ref/libref.so, i.e. tmac_gguf.cpp:990-1016
(apply_rope) and :1090-1128 (cache-write + GQA attention) compiled from the
reference tree by oracle/Makefile.  golden_qkv.npz holds the reference's
layer step from the normed hidden state (:1045-1128: quantized Q/K/V
projections, bias adds, RoPE, cache-write, attention) and the attention
block (:1045-1140: the same followed by the attn_output matmul and the
residual add) with weights decoded by its own f16_to_f32 / dequant_q5_0 /
dequant_q8_0 / read_tensor / matmul (:220-415, :476-514).  Inputs are regenerated from the seeds
recorded in the file (tests/golden/cases.py), so the fixture stays small.

Run from the repository root where the reference tree is mounted:
    make -C oracle all && python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402
from cases import O  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_ref.npz")
OUT_QKV = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_qkv.npz")

ROPE_POS = [0, 1, 2, 17, 255, 4095, 131071]
DECODE_POS = [0, 1, 7, 15, 16, 17, 63, 64, 100, 255]
DECODE_POS_BF16 = [0, 16, 255, 1000]
PREFILL_S = 48
SEED = 20260601


def _sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main() -> None:
    R = O.ref()
    data = {"seed": np.int64(SEED)}

    # RoPE: the reference's apply_rope on seeded q / k at several positions.
    q0 = O.normal(O.derive_seed(SEED, 0, 0, 11), cases.QD)
    k0 = O.normal(O.derive_seed(SEED, 0, 0, 12), cases.KD)
    data["rope_pos"] = np.array(ROPE_POS, dtype=np.int32)
    data["rope_in_sha"] = np.array(_sha(q0, k0))
    rq, rk = [], []
    for pos in ROPE_POS:
        q, k = O.ref_apply_rope(q0, k0, pos)
        rq.append(q)
        rk.append(k)
    data["rope_q"] = np.stack(rq)
    data["rope_k"] = np.stack(rk)

    # Decode steps (fp32 cache): RoPE + cache-write + attention, reference.
    for tag, positions, bf16 in (("f32", DECODE_POS, False),
                                 ("bf16", DECODE_POS_BF16, True)):
        outs, qs, ks, shas = [], [], [], []
        for pos in positions:
            q, k_new, v_new, kc, vc = cases.decode_inputs(SEED, pos, bf16)
            shas.append(_sha(q, k_new, v_new, kc, vc))
            q = q.copy()
            k = k_new.copy()
            if bf16:
                # bf16 cache: the roped k row is stored rounded, so run the
                # reference's rope, round the row, then its cache-write +
                # attention on the rounded row.
                q, k = O.ref_apply_rope(q, k, pos)
                k_row = O.round_bf16(k)
                out = np.empty(cases.QD, dtype=np.float32)
                R.tgref_cache_write_attention(q, k_row, v_new, out,
                                              kc.reshape(-1), vc.reshape(-1),
                                              pos)
            else:
                out = O.ref_decode_step(q, k, v_new, kc, vc, pos)
            outs.append(out)
            qs.append(q)
            ks.append(k)
        data[f"dec_{tag}_pos"] = np.array(positions, dtype=np.int32)
        data[f"dec_{tag}_out"] = np.stack(outs)
        data[f"dec_{tag}_q"] = np.stack(qs)
        data[f"dec_{tag}_k"] = np.stack(ks)
        data[f"dec_{tag}_in_sha"] = np.array(shas)

    # Prefill: token-by-token causal attention through the reference code.
    q, k, v = cases.prefill_inputs(SEED, PREFILL_S)
    kc = np.zeros((PREFILL_S, cases.KD), dtype=np.float32)
    vc = np.zeros((PREFILL_S, cases.KD), dtype=np.float32)
    pout = np.empty((PREFILL_S, cases.QD), dtype=np.float32)
    for t in range(PREFILL_S):
        qt = q[t].copy()
        R.tgref_cache_write_attention(qt, np.ascontiguousarray(k[t]),
                                      np.ascontiguousarray(v[t]), pout[t],
                                      kc.reshape(-1), vc.reshape(-1), t)
    data["prefill_S"] = np.int32(PREFILL_S)
    data["prefill_in_sha"] = np.array(_sha(q, k, v))
    data["prefill_out"] = pout

    _save(OUT, data)


QKV_CASES = [  # (v weight type, biases present, position)
    (6, True, 0), (6, True, 5), (6, True, 63), (8, True, 17), (8, False, 40),
    (6, False, 1),
]


BLOCK_CASES = [  # (v type, attn_output type, biases present, position)
    (6, 6, 1, 9), (8, 8, 1, 33), (6, 8, 0, 2),
]


def main_qkv() -> None:
    data = {"seed": np.int64(SEED), "cases": np.array(QKV_CASES, dtype=np.int32)}
    outs = {k: [] for k in ("q", "k", "v", "ctx", "sha")}
    for i, (vt, bias, pos) in enumerate(QKV_CASES):
        wq, wk, wv, bq, bk, bv = cases.qkv_weights(SEED + i, vt, bias)
        x = cases.qkv_x(SEED + i)[0]
        kc = np.zeros((pos + 1, cases.KD), np.float32)
        vc = np.zeros((pos + 1, cases.KD), np.float32)
        if pos > 0:
            kc[:pos] = O.normal(O.derive_seed(SEED + i, 0, 0, cases.T_KC), pos * cases.KD).reshape(pos, -1)
            vc[:pos] = O.normal(O.derive_seed(SEED + i, 0, 0, cases.T_VC), pos * cases.KD).reshape(pos, -1)
        outs["sha"].append(_sha(wq, wk, wv, *(b for b in (bq, bk, bv) if b is not None), x, kc, vc))
        q, k, v, ctx = O.ref_qkv_layer(wq, wk, wv, bq, bk, bv, x, kc, vc, pos, v_type=vt)
        for key, val in (("q", q), ("k", k), ("v", v), ("ctx", ctx)):
            outs[key].append(val)
    for key in ("q", "k", "v", "ctx"):
        data[f"qkv_{key}"] = np.stack(outs[key])
    data["qkv_in_sha"] = np.array(outs["sha"])
    # The attention block (tmac_gguf.cpp:1045-1140): the layer step, then
    # hidden = original_hidden + attn_output . context.
    data["blk_cases"] = np.array(BLOCK_CASES, dtype=np.int32)
    hid, shas = [], []
    for i, (vt, ot, bias, pos) in enumerate(BLOCK_CASES):
        seed = SEED + 100 + i
        wq, wk, wv, bq, bk, bv = cases.qkv_weights(seed, vt, bias)
        wo = cases.attn_output_weight(seed, ot)
        x = cases.qkv_x(seed)[0]
        h0 = cases.residual_in(seed)[0]
        kc = np.zeros((pos + 1, cases.KD), np.float32)
        vc = np.zeros((pos + 1, cases.KD), np.float32)
        if pos > 0:
            kc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_KC), pos * cases.KD).reshape(pos, -1)
            vc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_VC), pos * cases.KD).reshape(pos, -1)
        shas.append(_sha(wq, wk, wv, *(b for b in (bq, bk, bv) if b is not None), wo, x, h0, kc, vc))
        h, *_ = O.ref_attention_block(wq, wk, wv, bq, bk, bv, wo, x, h0, kc, vc, pos,
                                      v_type=vt, o_type=ot)
        hid.append(h)
    data["blk_hidden"] = np.stack(hid)
    data["blk_in_sha"] = np.array(shas)
    _save(OUT_QKV, data)


def _save(path, data) -> None:
    """Write the fixture unless an identical one is already there."""
    if os.path.exists(path):
        old = np.load(path)
        if set(old.files) == set(data) and all(
                np.array_equal(old[k], np.asarray(data[k])) for k in data):
            print(f"{path} unchanged")
            return
    np.savez_compressed(path, **data)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
    main_qkv()
