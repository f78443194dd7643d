"""tg_attention_noalloc: decode attention without any device allocation.

Who needs it: a caller that cannot call cudaMalloc at the moment it runs
attention -- for example code recording a CUDA graph in global capture mode,
where allocation calls are refused, a runtime that owns a fixed memory pool
and forbids the driver allocator once it has started, or an allocator hook
that must not re-enter itself.  This entry point takes only the caller's
device buffers and keeps its split-KV scratch in a fixed array inside the
library.

The test compares it with the regular entry point (tg_attention_batched on a
tg_kv_cache) through the C ABI, on two calls in a row, for a bf16 cache
(tensor-core kernel) and an fp32 cache (CUDA-core kernel), within the same
tolerances the other parity tests use.  It creates its own context so that it
passes alone in a fresh process as well as after the rest of the suite.
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
