"""The C-ABI library loads and exports every entry point include/*.h
declares; calls that need no GPU behave as documented on a CPU-only host.
No test here launches GPU work."""
from __future__ import annotations

import ctypes as C
import glob
import os
import re
import subprocess

import pytest

from conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"^TG_API\s+[\w\s\*]+?\b(tg_\w+)\s*\(", txt, re.M))
    return names


@pytest.fixture(scope="module")
def built(tg):
    if not os.path.exists(tg.LIB_PATH):
        tg.build()
    return tg


def test_header_declares_entry_points():
    names = _declared()
    for n in ("tg_init", "tg_rope_op", "tg_elem_op", "tg_attention_op",
              "tg_batch_begin", "tg_batch_end", "tg_decode_layer",
              "tg_attention_splitkv"):
        assert n in names


def test_library_exports_every_declared_symbol(built):
    out = subprocess.run(["nm", "-D", "--defined-only", built.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (tg_\w+)", out))
    missing = _declared() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # and nothing undeclared leaks out of the C ABI
    assert exported - _declared() == set()


def test_python_binding_covers_header(built):
    assert set(built.exported_symbols()) == _declared()
    L = built.lib()
    for n in _declared():
        assert getattr(L, n) is not None


def test_status_strings_and_version(built):
    L = built.lib()
    assert L.tg_status_string(0) == b"ok"
    assert b"unsupported" in L.tg_status_string(5)
    assert L.tg_version().startswith(b"tmac_gguf.cpp_b200")


def test_init_without_gpu_reports_no_device(built):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = built.lib().tg_init(0, C.byref(h))
    assert rc == built.TG_ERR_NO_DEVICE
    assert h.value is None
    assert b"no CUDA device" in built.lib().tg_last_error()


def test_null_arguments_are_rejected(built):
    L = built.lib()
    assert L.tg_init(0, None) == built.TG_ERR_INVALID_ARG
    assert L.tg_comm_unique_id(None, 0) == built.TG_ERR_INVALID_ARG
    assert L.tg_launch_count(None, None) == built.TG_ERR_INVALID_ARG
    assert L.tg_shutdown(None) == built.TG_OK


def test_python_errors_carry_status(built):
    with pytest.raises(built.TGError) as ei:
        built._check(built.TG_ERR_STATE)
    assert ei.value.status == built.TG_ERR_STATE


def test_shard_ranges_cover_context(built):
    for ctx in (1, 7, 131072, 131071):
        for world in (1, 2, 3, 4, 8):
            got = [built.shard_range(ctx, world, r) for r in range(world)]
            assert sum(n for _, n in got) == ctx
            pos = 0
            for s, n in got:
                if n:
                    assert s == pos
                pos += n
