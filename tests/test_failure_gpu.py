"""The library's own failure detection on one GPU (the reference only
prints and returns: metal_backend.cpp:23-27, tmac_gguf.cpp:1374-1409).

A communicator whose second rank never joins: tg_comm_init gives up with
TG_ERR_COMM after its timeout and the context keeps working.  The failure
is made on the host (a rank that never joins); no kernel waits on it.  The
device-side bound (a peer's records that never arrive, error 0x105) is
exercised by tests/splitkv_worker.py on two or more GPUs."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_comm_init_times_out_and_context_survives():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "10", "180", sys.executable,
           os.path.join(ROOT, "tests", "comm_timeout_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=240)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert "PASS" in r.stdout
