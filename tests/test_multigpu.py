"""Split-KV decode across every GPU of one box (skipped with fewer than 2):
small ragged cases and the BASELINE config-4 shape (4 x 131072 bf16
positions, one layer) against the oracle, under both record exchanges."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_splitkv_across_gpus():
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "splitkv_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
    print(r.stdout[-4000:], r.stderr[-4000:])
    assert r.returncode == 0
    assert "PASS" in r.stdout
