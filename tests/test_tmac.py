"""TMAC model files: the test writer (tests/golden/tmac_file.py) against
the reference's own loader load_tmac (tmac_gguf.cpp:1372-1425, compiled
into oracle/_ref), on the CPU."""
from __future__ import annotations

import os

import pytest

pytestmark = pytest.mark.skipif("not __import__('oracle').ref_available()")


def test_writer_round_trips_through_reference_loader(tmp_path, O):
    import tmac_file as T
    tensors = T.layer_tensors(11, 0) + T.layer_tensors(12, 1, bias=False)
    tensors.append(("n" * 140, 3, 2, O.TYPE_F32, bytes(range(24))))   # name cut to 127
    path = str(tmp_path / "m.tmac")
    T.write_tmac(path, tensors)
    rc, table = O.ref_load_tmac(path)
    assert rc == 0 and len(table) == len(tensors)
    for (name, rows, cols, typ, nb, data), (wn, wr, wc, wt, wd) in zip(table, tensors):
        assert name == wn[:127]
        assert (rows, cols, typ, nb) == (wr, wc, wt, len(wd))
        assert data == bytes(wd)
    # the Q8_0 v weight is followed by its row_max_abs companion
    names = [t[0] for t in table]
    assert names[names.index("blk.0.attn_v.weight") + 1] == "blk.0.attn_v.weight_row_max_abs"


def test_reference_loader_rejects_truncated_file(tmp_path, O):
    import tmac_file as T
    path = str(tmp_path / "m.tmac")
    T.write_tmac(path, T.layer_tensors(13, 0))
    size = os.path.getsize(path)
    with open(path, "r+b") as f:
        f.truncate(size - 100)
    rc, _ = O.ref_load_tmac(path)
    assert rc == -1
