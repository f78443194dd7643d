"""Writer of TMAC model files for the tests (test infrastructure only).

Layout as scripts/extract_tmac.py:6-23 documents it and load_tmac
(tmac_gguf.cpp:1372-1425) reads it: char magic[4] = "TMAC", uint64
n_tensors, then per tensor uint64 name_len, the name bytes, uint64 rows,
uint64 cols, uint32 type (GGUF type code), uint64 n_bytes and the data.
Every Q8_0 tensor is followed by its "<name>_row_max_abs" companion (rows x 1
float32, the largest |value| of each row), as the extractor writes it.
"""
from __future__ import annotations

import struct

import numpy as np

import cases
from cases import O


def write_tmac(path, tensors, magic=b"TMAC"):
    """tensors: iterable of (name, rows, cols, type, data bytes)."""
    tensors = list(tensors)
    with open(path, "wb") as f:
        f.write(magic)
        f.write(struct.pack("<Q", len(tensors)))
        for name, rows, cols, typ, data in tensors:
            nb = name.encode()
            f.write(struct.pack("<Q", len(nb)))
            f.write(nb)
            f.write(struct.pack("<QQIQ", rows, cols, typ, len(data)))
            f.write(bytes(data))


def row_max_abs(wtype, w, rows, cols):
    """Largest |dequantised value| of each row, float32 (for the companion)."""
    flat = np.ascontiguousarray(w, np.uint8).reshape(-1)
    L = O.lib()
    out = np.empty(rows, np.float32)
    for r in range(rows):
        out[r] = max(abs(L.tgo_dequant(wtype, flat, r * cols + j)) for j in range(cols))
    return out


def layer_tensors(seed, layer, v_type=O.TYPE_Q8_0, o_type=O.TYPE_Q5_0, bias=True):
    """The attention tensors of one layer, named as the model file names them
    (blk.N.attn_{q,k,v}.weight / .bias, blk.N.attn_output.weight), with rows
    = outputs and cols = inputs (read_tensor, tmac_gguf.cpp:402-407)."""
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(seed, v_type, bias, layer=layer)
    wo = cases.attn_output_weight(seed, o_type, layer=layer)
    QD, KD = cases.QD, cases.KD
    out = [(f"blk.{layer}.attn_q.weight", QD, QD, O.TYPE_Q5_0, wq.tobytes()),
           (f"blk.{layer}.attn_k.weight", KD, QD, O.TYPE_Q5_0, wk.tobytes()),
           (f"blk.{layer}.attn_v.weight", KD, QD, v_type, wv.tobytes())]
    if bias:
        out += [(f"blk.{layer}.attn_q.bias", QD, 1, O.TYPE_F32, bq.tobytes()),
                (f"blk.{layer}.attn_k.bias", KD, 1, O.TYPE_F32, bk.tobytes()),
                (f"blk.{layer}.attn_v.bias", KD, 1, O.TYPE_F32, bv.tobytes())]
    out.append((f"blk.{layer}.attn_output.weight", QD, QD, o_type, wo.tobytes()))
    with_aux = []
    for name, rows, cols, typ, data in out:
        with_aux.append((name, rows, cols, typ, data))
        if typ == O.TYPE_Q8_0:
            w = np.frombuffer(data, np.uint8)
            with_aux.append((name + "_row_max_abs", rows, 1, O.TYPE_F32,
                             row_max_abs(typ, w, rows, cols).tobytes()))
    return with_aux
