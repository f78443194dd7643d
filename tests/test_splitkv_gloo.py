"""The N>1 split-KV protocol on CPU ranks (gloo, world size 2 and 3).

Each rank takes its positions with the package's shard_range, builds the
per-shard softmax records in the layout the device kernels exchange
(o[n_head][hd] un-normalised, m[n_head] in log2 units, l[n_head]) with the
oracle's arithmetic, all-gathers them and merges them the way
gather_merge_kernel does; every rank must hold the oracle's result.  A
second test checks that a rank which never reaches the exchange makes the
others fail within the process-group timeout instead of waiting forever.
"""
from __future__ import annotations

import ctypes as C
import datetime
import math
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

LOG2E = 1.4426950408889634


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def shard_records(O, q, kc, vc, pos, start, length, n_head=14, n_kv=2, hd=64):
    """Records of one shard for one sequence (rows [start, start+length)
    intersected with 0..pos)."""
    rec = np.zeros(n_head * (hd + 2), np.float32)
    lo, hi = start, min(start + length, pos + 1)
    scores = np.empty(max(hi - lo, 1), np.float32)
    for h in range(n_head):
        if hi <= lo:
            rec[n_head * hd + h] = -1e30
            continue
        m, l = C.c_float(), C.c_float()
        o = np.empty(hd, np.float32)
        O.lib().tgo_partial_head(q, kc.reshape(-1), vc.reshape(-1), h, n_head, n_kv, hd,
                                 lo, hi, C.byref(m), C.byref(l), o, scores)
        rec[h * hd:(h + 1) * hd] = o
        rec[n_head * hd + h] = m.value * LOG2E  # natural -> log2 units
        rec[n_head * hd + n_head + h] = l.value
    return rec


def merge_records(recs, n_head=14, hd=64):
    """gather_merge_kernel's combine, in numpy (float64)."""
    qd = n_head * hd
    out = np.zeros(qd, np.float64)
    for h in range(n_head):
        m = np.array([r[qd + h] for r in recs], np.float64)
        l = np.array([r[qd + n_head + h] for r in recs], np.float64)
        M = m.max()
        w = np.exp2(m - M)
        o = sum(w[i] * recs[i][h * hd:(h + 1) * hd].astype(np.float64) for i in range(len(recs)))
        out[h * hd:(h + 1) * hd] = o / float((w * l).sum())
    return out


def _worker(rank, world, port, q_dir, mode):
    import sys
    import torch
    import torch.distributed as dist
    root = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
    for p in (root, os.path.join(root, "tests"), os.path.join(root, "tests", "golden")):
        sys.path.insert(0, p)
    from conftest import load_package
    import cases
    O = cases.O
    tg = load_package()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=8))
    result = {"ok": True, "err": None}
    try:
        if mode == "dead-peer" and rank == world - 1:
            return  # this rank never reaches the exchange (it exits)
        positions = [5000, 64, 1]
        gctx = max(positions) + 1
        start, length = tg.shard_range(gctx, world, rank)
        for i, p in enumerate(positions):
            q, _, _, kc, vc, ctx = cases.oracle_decode(123, p, seq=i)
            rec = torch.from_numpy(shard_records(O, q, kc, vc, p, start, length))
            got = [torch.zeros_like(rec) for _ in range(world)]
            dist.all_gather(got, rec)
            out = merge_records([g.numpy() for g in got])
            err = float(np.abs(out - ctx).max())
            if err > 1e-5:
                result = {"ok": False, "err": f"seq {i}: {err}"}
    except Exception as e:  # the dead-peer case lands here on live ranks
        result = {"ok": False, "err": f"{type(e).__name__}: {e}"}
    finally:
        np.save(os.path.join(q_dir, f"r{rank}.npy"), np.array([result], dtype=object),
                allow_pickle=True)
        if mode != "dead-peer":
            dist.destroy_process_group()


def _run(world, mode, tmp_path):
    port = _port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), mode))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    return [np.load(os.path.join(tmp_path, f"r{r}.npy"), allow_pickle=True)[0]
            for r in range(world)]


@pytest.mark.parametrize("world", [2, 3])
def test_splitkv_protocol_on_cpu_ranks(world, tmp_path):
    res = _run(world, "ok", tmp_path)
    assert all(r["ok"] for r in res), res


def test_dead_peer_fails_within_timeout(tmp_path):
    res = _run(2, "dead-peer", tmp_path)
    assert not res[0]["ok"]        # the live rank saw an error, not a hang
