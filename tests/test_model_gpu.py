"""The TMAC loader of the library (tg_model_*): its device table against the
reference's own load_tmac (tmac_gguf.cpp:1372-1425), error statuses, and a
layer's attention weights from the file driving the attention block."""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _write(tmp_path, tensors):
    import tmac_file as T
    path = str(tmp_path / "model.tmac")
    T.write_tmac(path, tensors)
    return path


def test_load_tmac_matches_reference_loader(tg, backend, O, tmp_path):
    import tmac_file as T
    tensors = T.layer_tensors(21, 0) + T.layer_tensors(22, 1, bias=False)
    tensors.append(("m" * 150, 5, 1, O.TYPE_F32, bytes(range(20))))
    path = _write(tmp_path, tensors)
    m = tg.Model(backend, path)
    assert len(m) == len(tensors)
    if O.ref_available():
        rc, table = O.ref_load_tmac(path)
        assert rc == 0
    else:
        table = [(n[:127], r, c, t, len(d), bytes(d)) for n, r, c, t, d in tensors]
    for i, (name, rows, cols, typ, nb, data) in enumerate(table):
        info = m.tensor(i)
        assert info["name"] == name
        assert (info["rows"], info["cols"], info["type"], info["n_bytes"]) == (rows, cols, typ, nb)
        assert info["data"] % 256 == 0
        assert m.read(i) == data
    assert m.find("blk.0.attn_q.bias")["n_bytes"] == 896 * 4
    assert m.find("blk.1.attn_q.bias") is None          # a model without that bias
    assert m.find("m" * 127)["rows"] == 5
    m.destroy()


def test_load_tmac_errors(tg, backend, tmp_path):
    import tmac_file as T
    with pytest.raises(tg.TGError) as e:
        tg.Model(backend, str(tmp_path / "absent.tmac"))
    assert e.value.status == tg.TG_ERR_INVALID_ARG
    path = _write(tmp_path, T.layer_tensors(23, 0))
    size = os.path.getsize(path)
    for cut in (size - 100, 30, 8):
        with open(path, "r+b") as f:
            f.truncate(cut)
        with pytest.raises(tg.TGError) as e:
            tg.Model(backend, path)
        assert e.value.status == tg.TG_ERR_INVALID_ARG
    # a count no file of this size can hold
    with open(path, "wb") as f:
        f.write(b"TMAC" + (1 << 60).to_bytes(8, "little"))
    with pytest.raises(tg.TGError):
        tg.Model(backend, path)


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_layer_from_file_runs_attention_block(tg, backend, O, cases, tmp_path, bf16):
    """The attention block with a layer's weights from the file equals the
    block with the same weights handed over as arrays, bit for bit, and the
    weights' device copies equal the arrays."""
    import tmac_file as T
    tensors = T.layer_tensors(31, 0) + T.layer_tensors(32, 1, bias=False)
    m = tg.Model(backend, _write(tmp_path, tensors))
    positions = [5, 70, 0, 33]
    B = len(positions)
    dt = tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32
    outs = []
    for layer in (0, 1):
        w_file, wo_file, o_type = m.layer_attention(layer)
        assert o_type == O.TYPE_Q5_0 and wo_file
        wq, wk, wv, bq, bk, bv = cases.qkv_weights(31 + layer, O.TYPE_Q8_0, layer == 0,
                                                   layer=layer)
        wo = cases.attn_output_weight(31 + layer, O.TYPE_Q5_0, layer=layer)
        w_arr = tg.QKVWeights(wq, wk, wv, 896, v_type=O.TYPE_Q8_0, b_q=bq, b_k=bk, b_v=bv)
        assert (w_file.desc.b_q is None) == (layer == 1)
        res = []
        for w, w_o in ((w_file, wo_file), (w_arr, wo)):
            kv = tg.KVCache(backend, 1, B, 128, dtype=dt)
            kv.fill_normal(77)
            x = cases.qkv_x(41, B).copy()
            hid = cases.residual_in(42, B).copy()
            kv.attention_block(0, w, w_o, x, positions, hid, o_type=o_type)
            res.append(hid)
            kv.destroy()
        assert np.array_equal(res[0].view(np.uint32), res[1].view(np.uint32)), layer
        outs.append(res[0])
    assert not np.array_equal(outs[0], outs[1])
    m.destroy()
