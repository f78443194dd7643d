"""Causal prefill on the tcgen05 tensor cores vs the reference's
token-by-token prompt processing (process_prompt, tmac_gguf.cpp:1621-1658:
one decode step, i.e. tmac_gguf.cpp:1093-1128, per position) run by the
oracle on the same bf16-rounded, RoPE-rotated inputs.  Bar: max-abs 2e-3;
RoPE and the cache rows the prefill writes: bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3


def run_prefill(tg, backend, cases, S, B=1, seed=5, max_ctx=None):
    kv = tg.KVCache(backend, 1, B, max_ctx or max(S, 1), dtype=tg.DTYPE_BF16)
    raw = [cases.prefill_raw(seed, S, seq=i) for i in range(B)]
    q = np.ascontiguousarray(np.stack([r[0] for r in raw]))
    k = np.ascontiguousarray(np.stack([r[1] for r in raw]))
    v = np.ascontiguousarray(np.stack([r[2] for r in raw]))
    out = np.zeros((B, S, cases.QD), np.float32)
    kv.prefill(0, B, S, q, k, v, out)
    return kv, out


@pytest.mark.parametrize("S", [1, 2, 5, 127, 128, 129, 300])
def test_prefill_matches_token_by_token_oracle(tg, backend, O, cases, S):
    B = 2
    kv, out = run_prefill(tg, backend, cases, S, B=B)
    for i in range(B):
        qb, kb, vb = cases.prefill_inputs(5, S, seq=i)
        ref = O.prefill_causal(qb, kb, vb)
        err = float(np.abs(out[i] - ref).max())
        assert err <= TOL, (S, i, err)
        krow, vrow = kv.read_rows(0, i, 0, S)         # cache rows, bf16 bits
        assert np.array_equal(krow, O.pack_bf16(kb))
        assert np.array_equal(vrow, O.pack_bf16(vb))


@pytest.mark.parametrize("S", [1, 127])
def test_prefill_odd_row_count(tg, backend, O, cases, S):
    """One sequence of odd length (the other cases run two sequences): the
    rotated k rows and the v rows in the cache are bit-exact."""
    kv, out = run_prefill(tg, backend, cases, S, B=1, seed=17)
    qb, kb, vb = cases.prefill_inputs(17, S, seq=0)
    assert float(np.abs(out[0] - O.prefill_causal(qb, kb, vb)).max()) <= TOL
    krow, vrow = kv.read_rows(0, 0, 0, S)
    assert np.array_equal(krow, O.pack_bf16(kb))
    assert np.array_equal(vrow, O.pack_bf16(vb))


def test_prefill_unaligned_device_inputs(tg, backend, cases):
    """q / k / v device buffers 4 bytes off a 16-byte boundary take the
    RoPE kernel's per-pair path; aligned ones its 16-byte row path.  Both
    must give the same cache rows and the same output, bit for bit."""
    import torch
    S, B = 129, 2
    raw = [cases.prefill_raw(23, S, seq=i) for i in range(B)]
    host = [np.ascontiguousarray(np.stack([r[j] for r in raw])) for j in range(3)]
    results = []
    for shift in (0, 1):
        dev = []
        for a in host:
            flat = torch.zeros(a.size + 4, dtype=torch.float32, device="cuda")
            view = flat[shift:shift + a.size].view(a.shape)
            view.copy_(torch.from_numpy(a))
            dev.append(view)
        assert all((t.data_ptr() % 16 == 0) == (shift == 0) for t in dev)
        kv = tg.KVCache(backend, 1, B, S, dtype=tg.DTYPE_BF16)
        out = torch.zeros(B, S, cases.QD, device="cuda")
        kv.prefill(0, B, S, dev[0], dev[1], dev[2], out)
        backend.synchronize()
        rows = [kv.read_rows(0, i, 0, S) for i in range(B)]
        results.append((out.cpu().numpy(), rows))
        kv.destroy()
    assert np.array_equal(results[0][0], results[1][0])
    for (k0, v0), (k1, v1) in zip(results[0][1], results[1][1]):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1)


def test_prefill_golden_from_reference(tg, backend, golden, cases):
    S = int(golden["prefill_S"])
    kv, out = run_prefill(tg, backend, cases, S, B=1, seed=int(golden["seed"]))
    assert float(np.abs(out[0] - golden["prefill_out"]).max()) <= TOL


def test_prefill_then_decode_continues(tg, backend, O, cases):
    """The cache the prefill fills is the one decode continues from."""
    S = 200
    kv, _ = run_prefill(tg, backend, cases, S, B=1, seed=9, max_ctx=512)
    qb, kb, vb = cases.prefill_inputs(9, S)
    q = O.normal(1234, cases.QD)
    k = O.normal(1235, cases.KD)
    v = O.round_bf16(O.normal(1236, cases.KD))
    Q, K = q[None].copy(), k[None].copy()
    out = np.zeros((1, cases.QD), np.float32)
    kv.decode_layer(0, Q, K, v[None].copy(), np.array([S], np.int32), out)
    qr = O.rope_heads(q, 14, 64, S)
    kr = O.round_bf16(O.rope_heads(k, 2, 64, S))
    kc = np.concatenate([kb, kr[None]])
    vc = np.concatenate([vb, v[None]])
    ref = O.attention(qr, kc, vc, S)
    assert float(np.abs(out[0] - ref).max()) <= TOL


def test_prefill_config5_length_sampled_rows(tg, backend, O, cases):
    """BASELINE config 5 sequence length (2048) on 2 sequences; rows at tile
    edges and spread over the prompt are checked against the oracle."""
    S, B = 2048, 2
    kv, out = run_prefill(tg, backend, cases, S, B=B, seed=55)
    rows = [0, 1, 127, 128, 129, 1000, 1535, 2046, 2047]
    for i in range(B):
        qb, kb, vb = cases.prefill_inputs(55, S, seq=i)
        for t in rows:
            ref = O.attention(qb[t], kb, vb, t)
            err = float(np.abs(out[i, t] - ref).max())
            assert err <= TOL, (i, t, err)


def test_prefill_rejects_unsupported(tg, backend):
    kv = tg.KVCache(backend, 1, 1, 64, dtype=tg.DTYPE_F32)
    z = np.zeros((1, 8, 896), np.float32)
    zk = np.zeros((1, 8, 128), np.float32)
    with pytest.raises(tg.TGError) as e:
        kv.prefill(0, 1, 8, z, zk, zk, z.copy())
    assert e.value.status == tg.TG_ERR_UNSUPPORTED
    kvb = tg.KVCache(backend, 1, 1, 64, dtype=tg.DTYPE_BF16)
    big = np.zeros((1, 65, 896), np.float32)
    bk = np.zeros((1, 65, 128), np.float32)
    with pytest.raises(tg.TGError) as e:
        kvb.prefill(0, 1, 65, big, bk, bk, big.copy())
    assert e.value.status == tg.TG_ERR_INVALID_ARG
