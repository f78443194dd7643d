"""One process joins a communicator of two ranks that the other rank never
joins: tg_comm_init must give up with TG_ERR_COMM after its timeout, and the
context must still run a decode step afterwards (checked against the
oracle).  Run by tests/test_failure_gpu.py; prints PASS on success."""
from __future__ import annotations

import os
import sys
import time

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, os.path.join(ROOT, "tests"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def main() -> int:
    import torch  # noqa: F401  (loads the NCCL the library then reuses)
    from conftest import load_package
    import cases
    tg = load_package()
    be = tg.CudaBackend(0)
    uid = tg.comm_unique_id()
    t0 = time.perf_counter()
    try:
        be.comm_init(uid, 0, 2, timeout_ms=2000)
        print("comm_init without the second rank succeeded")
        return 1
    except tg.TGError as e:
        dt = time.perf_counter() - t0
        print(f"comm_init failed after {dt:.2f} s: [{e.status}] {e.message}")
        if e.status != tg.TG_ERR_COMM or dt > 20:
            return 1
    # the context is still usable
    pos = [0, 100, 700]
    kv = tg.KVCache(be, 1, len(pos), 1024, dtype=tg.DTYPE_BF16)
    Q = np.zeros((3, cases.QD), np.float32)
    K = np.zeros((3, cases.KD), np.float32)
    V = np.zeros((3, cases.KD), np.float32)
    refs = []
    for i, p in enumerate(pos):
        q, k, v, kc, vc = cases.decode_inputs(31, p, True, seq=i)
        if p:
            kv.write_rows(0, i, 0, kc[:p], vc[:p])
        Q[i], K[i], V[i] = q, k, v
        refs.append(cases.oracle_decode(31, p, True, seq=i)[5])
    out = np.zeros_like(Q)
    kv.decode_layer(0, Q, K, V, np.array(pos, np.int32), out)
    err = max(float(np.abs(out[i] - refs[i]).max()) for i in range(3))
    print(f"decode after the failed init: max err {err:.2e}")
    kv.destroy()
    be.shutdown()
    if err > 2e-3:
        return 1
    print("PASS")
    return 0


if __name__ == "__main__":
    sys.exit(main())
