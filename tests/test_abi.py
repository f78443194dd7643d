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


def test_tuning_and_wait_limit_validate_arguments(built):
    L = built.lib()
    assert L.tg_set_decode_tuning(0, 0) == built.TG_OK
    assert L.tg_set_decode_tuning(128, 1) == built.TG_OK
    assert L.tg_set_decode_tuning(192, 0) == built.TG_OK
    assert L.tg_set_decode_tuning(64, 0) == built.TG_ERR_INVALID_ARG
    assert L.tg_set_decode_tuning(0, 2) == built.TG_ERR_INVALID_ARG
    assert L.tg_set_decode_tuning(0, 0) == built.TG_OK   # back to the defaults
    assert L.tg_comm_set_wait_limit_ms(None, 1000) == built.TG_ERR_INVALID_ARG
    n = C.c_int()
    assert L.tg_profile_read_stamps(None, None, 0, C.byref(n), C.byref(n)) == \
        built.TG_ERR_INVALID_ARG


def test_stamp_summary_reads_the_record_layout():
    """bench.py's in-step timing from per-CTA stamps: decode rows first,
    merge rows after the SM count, absent CTAs zero."""
    import numpy as np
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    n_sms, steps = 4, 3
    st = np.zeros((steps, 3 * n_sms, 4), np.uint64)
    for L in range(steps):
        t0 = 1_000_000 + 50_000 * L          # release of layer L, ns
        for c in range(n_sms):                # decode CTAs
            st[L, c] = (t0 - 5000 + 100 * c, t0 + 10 * c, t0 + 40_000 + 500 * c, t0 + 41_000 + 500 * c)
        for m in range(2):                    # two merge CTAs
            st[L, n_sms + m] = (t0 + 40_000, t0 + 43_000, 0, t0 + 45_000 + 100 * m)
    s = bench.stamp_summary(st, n_sms)
    assert s["steps"] == steps
    assert abs(s["tiles_us"] - 41.5) < 1e-9          # last tile at +41.5 us
    assert abs(s["launch_us"] - 45.1) < 1e-9         # last merge CTA at +45.1 us
    assert abs(s["tail_us"] - 3.6) < 1e-9
    assert abs(s["period_us"] - 50.0) < 1e-9
    assert abs(s["early_us"] - 5.0) < 1e-9
