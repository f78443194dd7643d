"""tg_attention_noalloc: decode attention without any device allocation.

Who needs it: a caller that cannot call cudaMalloc at the moment it runs
attention -- for example code recording a CUDA graph in global capture mode,
where allocation calls are refused, a runtime that owns a fixed memory pool
and forbids the driver allocator once it has started, or an allocator hook
that must not re-enter itself.  This entry point takes only the caller's
device buffers and keeps its split-KV scratch in a fixed array inside the
library.

The tests compare it with the regular entry point (tg_attention_batched on a
tg_kv_cache) through the C ABI, on two calls in a row, for a bf16 cache
(tensor-core kernel) and an fp32 cache (CUDA-core kernel), and with the
oracle on two calls of different batch sizes (one shape narrows the grid to
fit the fixed array), within the tolerances the other parity tests use; and
check that a position outside the cache reads 0x103 in the call's status.
Each test creates its own context so that the file passes alone in a fresh
process as well as after the rest of the suite.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = {"bf16": 2e-3, "f32": 1e-4}


@pytest.mark.parametrize("dtype_name", ["bf16", "f32"])
def test_noalloc_matches_regular_entry_point(tg, dtype_name):
    import torch
    dtype = tg.DTYPE_BF16 if dtype_name == "bf16" else tg.DTYPE_F32
    be = tg.CudaBackend(0)
    try:
        B, max_ctx = 6, 3000
        kv = tg.KVCache(be, 1, B, max_ctx, dtype=dtype)
        kv.fill_normal(4242)
        kptr, vptr = kv.layer_ptrs(0)
        g = torch.Generator(device="cuda")
        g.manual_seed(17)
        q = torch.randn(B, 896, device="cuda", generator=g)
        past = torch.tensor([0, 63, 64, 700, 2999, 1500], dtype=torch.int32, device="cuda")
        ref = torch.zeros(B, 896, device="cuda")
        kv.attention(0, q, past, ref)
        be.synchronize()
        stream = be.stream()
        status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        for call in range(2):  # the scratch keeps the previous call's contents
            out = torch.full((B, 896), float("nan"), device="cuda")
            tg.attention_noalloc(stream, q, kptr, vptr, dtype, B, max_ctx, past, out,
                                 device_status=status)
            be.synchronize()
            assert int(status.item()) == 0, call
            err = float((out - ref).abs().max().item())
            assert err <= TOL[dtype_name], (call, err)
        # sizes beyond the fixed scratch are refused with a clear error
        with pytest.raises(tg.TGError) as e:
            tg.attention_noalloc(stream, q, kptr, vptr, dtype, tg.NOALLOC_MAX_SEQS + 1,
                                 max_ctx, past, out)
        assert e.value.status == tg.TG_ERR_INVALID_ARG
        assert "n_seqs" in e.value.message
        kv.destroy()
    finally:
        be.shutdown()


# Shapes for the oracle checks: the Qwen2-0.5B head shape over a bf16 cache
# (tensor-core kernel), and 32 query / 4 KV heads of head_dim 128 over an fp32
# cache, whose softmax records (32 x 130 floats) let only 126 CTAs' partial
# records fit in the fixed array -- fewer than the GPU's SMs, so the call
# narrows its grid.
ORACLE_SHAPES = [("bf16", 14, 2, 64), ("f32", 32, 4, 128)]


def _seeded_cache(O, seed, B, max_ctx, n_kv, hd, bf16):
    gen = O.normal_bf16 if bf16 else O.normal
    k = gen(O.derive_seed(seed, 0, 0, 4), B * max_ctx * n_kv * hd).reshape(B, max_ctx, n_kv * hd)
    v = gen(O.derive_seed(seed, 0, 0, 5), B * max_ctx * n_kv * hd).reshape(B, max_ctx, n_kv * hd)
    return k, v


@pytest.mark.parametrize("dtype_name,n_head,n_kv,hd", ORACLE_SHAPES)
def test_noalloc_against_oracle(tg, O, dtype_name, n_head, n_kv, hd):
    """Both calls of a pair checked against the oracle's attention
    (tmac_gguf.cpp:1093-1128), the second with fewer sequences and other
    positions, so it reads the array with the first call's records in it."""
    import torch
    bf16 = dtype_name == "bf16"
    dtype = tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32
    be = tg.CudaBackend(0)
    try:
        B, max_ctx = 5, 2500
        kc, vc = _seeded_cache(O, 808, B, max_ctx, n_kv, hd, bf16)
        kv = tg.KVCache(be, 1, B, max_ctx, n_head=n_head, n_kv_head=n_kv, head_dim=hd,
                        dtype=dtype)
        for s in range(B):
            kv.write_rows(0, s, 0, kc[s], vc[s])
        kptr, vptr = kv.layer_ptrs(0)
        q = O.normal(O.derive_seed(809, 0, 0, 1), B * n_head * hd).reshape(B, n_head * hd)
        qd = torch.from_numpy(q).cuda()
        status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        stream = be.stream()
        for call, (nb, past) in enumerate([(5, [2499, 0, 64, 1234, 700]), (3, [17, 2048, 63])]):
            pd = torch.tensor(past, dtype=torch.int32, device="cuda")
            out = torch.full((nb, n_head * hd), float("nan"), device="cuda")
            tg.attention_noalloc(stream, qd, kptr, vptr, dtype, nb, max_ctx, pd, out,
                                 device_status=status, n_head=n_head, n_kv_head=n_kv,
                                 head_dim=hd)
            be.synchronize()
            assert int(status.item()) == 0, call
            got = out.cpu().numpy()
            for s in range(nb):
                ref = O.attention(q[s], kc[s], vc[s], past[s], n_head, n_kv, hd)
                err = float(np.abs(got[s] - ref).max())
                assert err <= TOL[dtype_name], (call, s, err)
        kv.destroy()
    finally:
        be.shutdown()


def test_noalloc_reports_bad_position(tg):
    """A position outside the cache is a device-side error: the call's
    status reads 0x103, the other sequences are still computed, and the next
    call (valid positions) reports 0 again."""
    import torch
    be = tg.CudaBackend(0)
    try:
        B, max_ctx = 3, 512
        kv = tg.KVCache(be, 1, B, max_ctx, dtype=tg.DTYPE_BF16)
        kv.fill_normal(99)
        kptr, vptr = kv.layer_ptrs(0)
        q = torch.randn(B, 896, device="cuda")
        good = torch.tensor([10, 300, 511], dtype=torch.int32, device="cuda")
        ref = torch.zeros(B, 896, device="cuda")
        kv.attention(0, q, good, ref)
        be.synchronize()
        status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        stream = be.stream()
        bad = torch.tensor([10, max_ctx, 511], dtype=torch.int32, device="cuda")
        out = torch.zeros(B, 896, device="cuda")
        tg.attention_noalloc(stream, q, kptr, vptr, tg.DTYPE_BF16, B, max_ctx, bad, out,
                             device_status=status)
        be.synchronize()
        assert int(status.item()) == 0x103
        for s in (0, 2):
            assert float((out[s] - ref[s]).abs().max().item()) <= TOL["bf16"]
        tg.attention_noalloc(stream, q, kptr, vptr, tg.DTYPE_BF16, B, max_ctx, good, out,
                             device_status=status)
        be.synchronize()
        assert int(status.item()) == 0
        assert float((out - ref).abs().max().item()) <= TOL["bf16"]
        kv.destroy()
    finally:
        be.shutdown()
