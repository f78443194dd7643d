"""Generate tests/golden/golden_ref.npz from the reference's own code.

The outputs come from oracle/_ref/libref.so, i.e. tmac_gguf.cpp:990-1016
(apply_rope) and :1090-1128 (cache-write + GQA attention) compiled from the
reference tree by oracle/Makefile.  Inputs are regenerated from the seeds
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

    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
