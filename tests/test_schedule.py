"""Host-side check of the flat-tile split-KV schedule (csrc/tg_shared.h):
the index functions the kernels use are compiled here for the host and the
ownership / partial-slot bookkeeping of the decode and merge kernels is
replayed for many random batches."""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import tempfile

import numpy as np
import pytest

from conftest import PKG_DIR

SHIM = r"""
#include "tg_shared.h"
extern "C" {
int cta_of_tile(long long t, int G, long long T) { return tg::cta_of_tile(t, G, T); }
long long cta_tile_lo(int c, int G, long long T) { return tg::cta_tile_lo(c, G, T); }
int local_rows(int p, int s, int m) { return tg::local_rows(p, s, m); }
int record_floats(int h, int d) { return tg::record_floats(h, d); }
}
"""


@pytest.fixture(scope="module")
def sched():
    d = tempfile.mkdtemp()
    src = os.path.join(d, "shim.cpp")
    so = os.path.join(d, "shim.so")
    open(src, "w").write(SHIM)
    subprocess.run(["g++", "-O1", "-shared", "-fPIC", "-I",
                    os.path.join(PKG_DIR, "csrc"), src, "-o", so], check=True)
    L = C.CDLL(so)
    L.cta_of_tile.restype = C.c_int
    L.cta_of_tile.argtypes = [C.c_longlong, C.c_int, C.c_longlong]
    L.cta_tile_lo.restype = C.c_longlong
    L.cta_tile_lo.argtypes = [C.c_int, C.c_int, C.c_longlong]
    L.local_rows.argtypes = [C.c_int, C.c_int, C.c_int]
    return L


def test_local_rows(sched):
    assert sched.local_rows(0, 0, 256) == 1
    assert sched.local_rows(255, 0, 256) == 256
    assert sched.local_rows(99, 100, 50) == 0       # shard after the token
    assert sched.local_rows(120, 100, 50) == 21
    assert sched.local_rows(1000, 100, 50) == 50    # shard fully before
    assert sched.record_floats(14, 64) == 14 * 66


def _replay(sched, tiles, G):
    """Replays the kernels' bookkeeping; returns per-sequence slot lists
    written by the decode kernel and derived by the merge kernel."""
    prefix = np.concatenate([[0], np.cumsum(tiles)]).astype(np.int64)
    T = int(prefix[-1])
    B = len(tiles)
    G = min(G, T)  # the kernels' effective grid
    written = {s: [] for s in range(B)}
    complete = set()
    owner = np.full(T, -1)
    for c in range(G):
        lo, hi = sched.cta_tile_lo(c, G, T), sched.cta_tile_lo(c + 1, G, T)
        assert lo < hi  # no empty CTA in the effective grid
        owner[lo:hi] = c
        t = lo
        while t < hi:
            s = int(np.searchsorted(prefix, t, side="right") - 1)
            seg_hi = min(hi, int(prefix[s + 1]))
            if t == prefix[s] and seg_hi == prefix[s + 1]:
                complete.add(s)
            else:
                written[s].append(2 * c + (0 if t == lo else 1))
            t = seg_hi
    assert (owner >= 0).all()
    for t in range(T):
        assert sched.cta_of_tile(t, G, T) == owner[t]
    derived = {}
    for s in range(B):
        t0, t1 = int(prefix[s]), int(prefix[s + 1])
        if t1 == t0:
            continue
        c1, c2 = sched.cta_of_tile(t0, G, T), sched.cta_of_tile(t1 - 1, G, T)
        if c1 == c2:
            assert s in complete
            continue
        first = 2 * c1 + (0 if sched.cta_tile_lo(c1, G, T) == t0 else 1)
        derived[s] = [first] + [2 * (c1 + k) for k in range(1, c2 - c1 + 1)]
    return written, derived, complete


@pytest.mark.parametrize("seed", range(12))
def test_slots_agree_between_decode_and_merge(sched, seed):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 300))
    tiles = rng.integers(0, 70, size=B)
    if seed % 3 == 0:
        tiles[:] = 1                    # many tiny sequences
    if seed % 4 == 1:
        tiles[0] = 2048                 # one long sequence
    if tiles.sum() == 0:
        tiles[0] = 1
    G = int(rng.choice([1, 7, 148, 296, 592]))
    written, derived, complete = _replay(sched, tiles, G)
    for s in range(B):
        if tiles[s] == 0:
            continue
        if s in complete:
            assert written[s] == [] and s not in derived
        else:
            assert sorted(written[s]) == sorted(derived[s])
    all_slots = [x for v in written.values() for x in v]
    assert len(all_slots) == len(set(all_slots))


@pytest.mark.parametrize("tiles,G", [([3], 592), ([2], 592), ([1, 5, 2], 148),
                                     ([0, 4, 0, 9], 296), ([33], 32), ([7, 1], 8)])
def test_more_ctas_than_tiles(sched, tiles, G):
    """Short sequences on a large grid: every CTA of the effective grid owns
    tiles, so a split sequence's slots are all written."""
    tiles = np.array(tiles)
    written, derived, complete = _replay(sched, tiles, G)
    for s in range(len(tiles)):
        if tiles[s] and s not in complete:
            assert sorted(written[s]) == sorted(derived[s])


def test_long_context_split_counts(sched):
    # config 4 at one GPU: 4 sequences x 2048 tiles over 148 CTAs
    tiles = np.full(4, 131072 // 64)
    written, derived, _ = _replay(sched, tiles, 148)
    assert sum(len(v) for v in written.values()) <= 2 * 148
    assert all(len(derived[s]) >= 37 for s in range(4))
