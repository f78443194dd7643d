"""Parity of the CUDA decode path with the CPU oracle, through the C ABI.

Bars (from the task contract):
  * RoPE and cache-write: bit-exact with the reference's CPU code;
  * attention over an fp32 cache: max-abs <= 1e-4;
  * attention over a bf16 cache: the oracle runs on the same bf16-rounded
    values widened to fp32; max-abs <= 2e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F32_TOL = 1e-4
BF16_TOL = 2e-3


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def maxabs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def run_batch(tg, backend, cases, positions, bf16, seed=11, max_ctx=None,
              layer=0, n_layers=1, stream0=False):
    """Fill a cache with each sequence's rows 0..pos-1, run one decode step
    through tg_decode_layer and return (gpu outputs, oracle results, kv).
    Sequence i draws its inputs from stream i (stream 0 for all when
    stream0, as the golden fixtures do)."""
    B = len(positions)
    max_ctx = max_ctx or (max(positions) + 1)
    kv = tg.KVCache(backend, n_layers, B, max_ctx,
                    dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
    Q = np.zeros((B, cases.QD), np.float32)
    K = np.zeros((B, cases.KD), np.float32)
    V = np.zeros((B, cases.KD), np.float32)
    refs = []
    for i, pos in enumerate(positions):
        sq = 0 if stream0 else i
        q, k_new, v_new, kc, vc = cases.decode_inputs(seed, pos, bf16, seq=sq, layer=layer)
        if pos > 0:
            kv.write_rows(layer, i, 0, kc[:pos], vc[:pos])
        Q[i], K[i], V[i] = q, k_new, v_new
        refs.append(cases.oracle_decode(seed, pos, bf16, seq=sq, layer=layer))
    out = np.zeros((B, cases.QD), np.float32)
    kv.decode_layer(layer, Q, K, V, np.array(positions, np.int32), out)
    return Q, K, out, refs, kv


# ----------------------------------------------------------------- RoPE

def test_rope_op_bit_exact_against_reference(backend, golden, O, cases):
    seed = int(golden["seed"])
    q0 = O.normal(O.derive_seed(seed, 0, 0, 11), cases.QD)
    k0 = O.normal(O.derive_seed(seed, 0, 0, 12), cases.KD)
    for i, pos in enumerate(golden["rope_pos"]):
        q, k = q0.copy(), k0.copy()
        backend.rope_op(q, 14, 64, int(pos), 1000000.0)
        backend.rope_op(k, 2, 64, int(pos), 1000000.0)
        assert np.array_equal(bits(q), bits(golden["rope_q"][i])), pos
        assert np.array_equal(bits(k), bits(golden["rope_k"][i])), pos


def test_rope_op_on_device_tensor(backend, O):
    import torch
    x = O.normal(3, 896)
    t = torch.from_numpy(x.copy()).cuda()
    backend.rope_op(t, 14, 64, 777, 1000000.0)
    backend.synchronize()
    assert np.array_equal(bits(t.cpu().numpy()), bits(O.rope_heads(x, 14, 64, 777)))


def test_rope_other_base_and_head_dim(backend, O):
    x = O.normal(4, 8 * 128)
    y = x.copy()
    backend.rope_op(y, 8, 128, 4242, 10000.0)
    assert np.array_equal(bits(y), bits(O.rope_heads(x, 8, 128, 4242, 10000.0)))


# ------------------------------------------------------ attention_op (compat)

@pytest.mark.parametrize("pos", [0, 1, 7, 15, 16, 17, 31, 32, 33, 63, 64, 65,
                                 127, 255, 256, 1000])
def test_attention_op_fp32(backend, cases, pos):
    q, _, _, kc, vc, ctx = cases.oracle_decode(21, pos)
    out = np.zeros(cases.QD, np.float32)
    backend.attention_op(q, kc, vc, out, 14, 2, 64, pos)
    assert maxabs(out, ctx) <= F32_TOL


def test_attention_op_golden(backend, golden, cases):
    seed = int(golden["seed"])
    for i, pos in enumerate(golden["dec_f32_pos"]):
        q, _, _, kc, vc, _ = cases.oracle_decode(seed, int(pos))
        out = np.zeros(cases.QD, np.float32)
        backend.attention_op(q, kc, vc, out, 14, 2, 64, int(pos))
        assert maxabs(out, golden["dec_f32_out"][i]) <= F32_TOL


def test_attention_op_other_shapes(backend, O):
    """kernel_attn handles any GQA shape; so does the CUDA-core kernel."""
    for n_head, n_kv, hd, pos in ((8, 8, 32, 50), (16, 1, 128, 70), (12, 4, 64, 300)):
        q = O.normal(1, n_head * hd)
        kc = O.normal(2, (pos + 1) * n_kv * hd)
        vc = O.normal(3, (pos + 1) * n_kv * hd)
        out = np.zeros(n_head * hd, np.float32)
        backend.attention_op(q, kc, vc, out, n_head, n_kv, hd, pos)
        ref = O.attention(q, kc, vc, pos, n_head, n_kv, hd)
        assert maxabs(out, ref) <= F32_TOL


def test_compat_fused_forward_loop(backend, O, cases):
    """The reference's fused forward loop (tmac_gguf.cpp:1490-1496) driven
    through the compat ops on host arrays, token by token, 3 layers: rope_op
    q and k, elem_op(2) the K/V rows into g_k_cache/g_v_cache, attention_op
    over the layer's cache, one batch per token as metal_batch_begin/end."""
    L, MAXS, n_tok = 3, 256, 40
    g_k_cache = np.zeros((L, MAXS, 128), np.float32)
    g_v_cache = np.zeros((L, MAXS, 128), np.float32)
    ref_k = np.zeros_like(g_k_cache)
    ref_v = np.zeros_like(g_v_cache)
    q_vec = np.zeros(896, np.float32)
    k_new = np.zeros(128, np.float32)
    v_new = np.zeros(128, np.float32)
    context = np.zeros(896, np.float32)
    worst = 0.0
    for pos in range(n_tok):
        backend.metal_batch_begin()
        expected = []
        for layer in range(L):
            q_vec[:] = O.normal(O.derive_seed(5, layer, pos, 1), 896)
            k_new[:] = O.normal(O.derive_seed(5, layer, pos, 2), 128)
            v_new[:] = O.normal(O.derive_seed(5, layer, pos, 3), 128)
            qr, kr = q_vec.copy(), k_new.copy()
            expected.append(O.decode_step(qr, kr, v_new.copy(), ref_k[layer],
                                          ref_v[layer], pos))
            backend.rope_op(q_vec, 14, 64, pos, 1000000.0)
            backend.rope_op(k_new, 2, 64, pos, 1000000.0)
            backend.elem_op(2, g_k_cache[layer, pos], k_new, 128)
            backend.elem_op(2, g_v_cache[layer, pos], v_new, 128)
            backend.attention_op(q_vec, g_k_cache[layer], g_v_cache[layer],
                                 context, 14, 2, 64, pos)
            # host arrays are reused next layer: close the batch per layer
            backend.metal_batch_end()
            worst = max(worst, maxabs(context, expected[-1]))
            assert np.array_equal(bits(g_k_cache[layer, pos]), bits(ref_k[layer, pos]))
            assert np.array_equal(bits(q_vec), bits(qr))
            backend.metal_batch_begin()
        backend.metal_batch_end()
    assert worst <= F32_TOL


def test_device_owned_cache_region(backend, O, cases):
    """g_k_cache registered device-owned: only GPU ops write it, no copies."""
    pos_max = 20
    kc = np.zeros((64, 128), np.float32)
    vc = np.zeros((64, 128), np.float32)
    backend.register_host(kc, 1)
    backend.register_host(vc, 1)
    ref_k = np.zeros_like(kc)
    ref_v = np.zeros_like(vc)
    q = np.zeros(896, np.float32)
    k = np.zeros(128, np.float32)
    v = np.zeros(128, np.float32)
    out = np.zeros(896, np.float32)
    for pos in range(pos_max):
        q[:] = O.normal(pos * 3 + 1, 896)
        k[:] = O.normal(pos * 3 + 2, 128)
        v[:] = O.normal(pos * 3 + 3, 128)
        exp = O.decode_step(q.copy(), k.copy(), v.copy(), ref_k, ref_v, pos)
        backend.metal_batch_begin()
        backend.rope_op(q, 14, 64, pos, 1000000.0)
        backend.rope_op(k, 2, 64, pos, 1000000.0)
        backend.elem_op(2, kc[pos], k, 128)
        backend.elem_op(2, vc[pos], v, 128)
        backend.attention_op(q, kc, vc, out, 14, 2, 64, pos)
        backend.metal_batch_end()
        assert maxabs(out, exp) <= F32_TOL
    # the host copy was never written back; an explicit sync brings it
    assert not kc.any()
    backend.region_sync(kc)
    assert np.array_equal(bits(kc[:pos_max]), bits(ref_k[:pos_max]))
    backend.unregister_host(kc)
    backend.unregister_host(vc)


# ------------------------------------------------------ batched decode

EDGE_POS = [0, 1, 15, 16, 17, 31, 32, 33, 63, 64, 65, 127, 128, 200, 255]


def test_decode_layer_fp32_ragged(tg, backend, cases):
    Q, K, out, refs, kv = run_batch(tg, backend, cases, EDGE_POS, bf16=False)
    assert not kv.uses_tensor_cores()
    for i, pos in enumerate(EDGE_POS):
        qr, kr, vr, kc, vc, ctx = refs[i]
        assert np.array_equal(bits(Q[i]), bits(qr)), pos        # RoPE, bit-exact
        assert np.array_equal(bits(K[i]), bits(kr)), pos
        krow, vrow = kv.read_rows(0, i, pos, 1)                   # cache-write
        assert np.array_equal(bits(krow[0]), bits(kc[pos])), pos
        assert np.array_equal(bits(vrow[0]), bits(vc[pos])), pos
        assert maxabs(out[i], ctx) <= F32_TOL, pos


def test_decode_layer_bf16_ragged(tg, backend, O, cases):
    Q, K, out, refs, kv = run_batch(tg, backend, cases, EDGE_POS, bf16=True)
    assert kv.uses_tensor_cores()
    for i, pos in enumerate(EDGE_POS):
        qr, kr, vr, kc, vc, ctx = refs[i]
        assert np.array_equal(bits(Q[i]), bits(qr)), pos
        krow, vrow = kv.read_rows(0, i, pos, 1)
        assert np.array_equal(krow[0], O.pack_bf16(kc[pos])), pos  # RNE bits
        assert np.array_equal(vrow[0], O.pack_bf16(vc[pos])), pos
        assert maxabs(out[i], ctx) <= BF16_TOL, pos


def test_decode_golden_through_gpu(tg, backend, golden, cases):
    seed = int(golden["seed"])
    for tag, bf16, tol in (("f32", False, F32_TOL), ("bf16", True, BF16_TOL)):
        positions = [int(p) for p in golden[f"dec_{tag}_pos"]]
        Q, K, out, _, _ = run_batch(tg, backend, cases, positions, bf16, seed=seed,
                                    stream0=True)
        for i in range(len(positions)):
            assert np.array_equal(bits(Q[i]), bits(golden[f"dec_{tag}_q"][i]))
            assert np.array_equal(bits(K[i]), bits(golden[f"dec_{tag}_k"][i]))
            assert maxabs(out[i], golden[f"dec_{tag}_out"][i]) <= tol


def test_bf16_tile_edges_and_long(tg, backend, cases):
    positions = [4095, 4096, 4097, 1, 8191, 300]
    _, _, out, refs, _ = run_batch(tg, backend, cases, positions, bf16=True, seed=3)
    for i, pos in enumerate(positions):
        assert maxabs(out[i], refs[i][5]) <= BF16_TOL, pos


def test_config2_shape_batch64_fp32_two_layers(tg, backend, O, cases):
    """BASELINE config 2 shape: 64 sequences, context ~ U[1,256], fp32."""
    rng = np.random.default_rng(2026)
    positions = [int(x) for x in rng.integers(0, 256, size=64)]
    for layer in (0, 1):
        _, _, out, refs, _ = run_batch(tg, backend, cases, positions, bf16=False,
                                       seed=40, max_ctx=256, layer=layer, n_layers=2)
        for i in range(64):
            assert maxabs(out[i], refs[i][5]) <= F32_TOL


def test_config3_shape_subset_bf16(tg, backend, cases):
    """BASELINE config 3 shape (context 4096, bf16) on 12 sequences."""
    positions = [4095] * 12
    _, _, out, refs, _ = run_batch(tg, backend, cases, positions, bf16=True, seed=9)
    for i in range(12):
        assert maxabs(out[i], refs[i][5]) <= BF16_TOL


def test_device_arrays_and_batched_attention(tg, backend, cases):
    """Inputs resident on the device (torch tensors) through the same ABI."""
    import torch
    positions = [5, 100, 64]
    _, _, out_host, refs, kv = run_batch(tg, backend, cases, positions, bf16=True, seed=77)
    qd = torch.from_numpy(np.stack([r[0] for r in refs])).cuda()
    pd = torch.tensor(positions, dtype=torch.int32, device="cuda")
    od = torch.zeros_like(qd)
    kv.attention(0, qd, pd, od)
    backend.synchronize()
    np.testing.assert_allclose(od.cpu().numpy(), out_host, atol=1e-6, rtol=0)


def _fill_same(kv_list, cases, positions, bf16, seed, layers):
    """Write the same rows 0..pos-1 of every layer into each cache; return
    the per-layer raw inputs (Q, K, V) and the oracle results."""
    B = len(positions)
    inputs, refs = [], []
    for layer in range(layers):
        Q = np.zeros((B, cases.QD), np.float32)
        K = np.zeros((B, cases.KD), np.float32)
        V = np.zeros((B, cases.KD), np.float32)
        lrefs = []
        for i, pos in enumerate(positions):
            q, k_new, v_new, kc, vc = cases.decode_inputs(seed, pos, bf16, seq=i, layer=layer)
            for kv in kv_list:
                if pos > 0:
                    kv.write_rows(layer, i, 0, kc[:pos], vc[:pos])
            Q[i], K[i], V[i] = q, k_new, v_new
            lrefs.append(cases.oracle_decode(seed, pos, bf16, seq=i, layer=layer))
        inputs.append((Q, K, V))
        refs.append(lrefs)
    return inputs, refs


@pytest.mark.parametrize("splitkv", [False, True])
def test_pinned_host_buffers_match_pageable(tg, backend, O, cases, splitkv):
    """Host buffers in page-locked memory take the direct path (inputs packed
    into one copy per call, outputs written by the kernels through the
    buffers' device addresses); results are bit-identical to pageable numpy
    buffers and within the bar of the oracle.  Long positions split
    sequences across CTAs, so the merge kernel's writes are covered too."""
    import torch
    positions = [0, 33, 4095, 9000]
    layers = 2
    max_ctx = max(positions) + 1
    kv_a = tg.KVCache(backend, layers, len(positions), max_ctx, dtype=tg.DTYPE_BF16)
    kv_b = tg.KVCache(backend, layers, len(positions), max_ctx, dtype=tg.DTYPE_BF16)
    inputs, refs = _fill_same([kv_a, kv_b], cases, positions, True, 31, layers)
    pos_np = np.array(positions, np.int32)
    pos_pin = torch.from_numpy(pos_np.copy()).pin_memory()
    res_a, res_b = [], []
    backend.metal_batch_begin()
    for layer in range(layers):
        Q, K, V = (x.copy() for x in inputs[layer])
        out = np.zeros_like(Q)
        (kv_a.decode_layer_splitkv if splitkv else kv_a.decode_layer)(layer, Q, K, V, pos_np, out)
        res_a.append((Q, K, out))
        Qp, Kp, Vp = (torch.from_numpy(x.copy()).pin_memory() for x in inputs[layer])
        outp = torch.zeros(Qp.shape, dtype=torch.float32).pin_memory()
        (kv_b.decode_layer_splitkv if splitkv else kv_b.decode_layer)(layer, Qp, Kp, Vp,
                                                                     pos_pin, outp)
        res_b.append((Qp, Kp, outp))
    backend.metal_batch_end()
    for layer in range(layers):
        Q, K, out = res_a[layer]
        Qp, Kp, outp = (t.numpy() for t in res_b[layer])
        assert np.array_equal(bits(Qp), bits(Q)), layer       # rotated q written back
        assert np.array_equal(bits(Kp), bits(K)), layer       # rotated k written back
        assert np.array_equal(bits(outp), bits(out)), layer   # same kernels, same bits
        for i, pos in enumerate(positions):
            qr, kr, vr, kc, vc, ctx = refs[layer][i]
            assert np.array_equal(bits(Qp[i]), bits(qr)), (layer, pos)
            ka, va = kv_a.read_rows(layer, i, pos, 1)
            kb, vb = kv_b.read_rows(layer, i, pos, 1)
            assert np.array_equal(kb, ka) and np.array_equal(vb, va)
            assert np.array_equal(kb[0], O.pack_bf16(kc[pos])), (layer, pos)
            assert maxabs(outp[i], ctx) <= BF16_TOL, (layer, pos)
    # outside a batch the call returns with the host outputs valid
    Q, K, V = (torch.from_numpy(x.copy()).pin_memory() for x in inputs[0])
    outp = torch.zeros(Q.shape, dtype=torch.float32).pin_memory()
    kv_c = tg.KVCache(backend, 1, len(positions), max_ctx, dtype=tg.DTYPE_BF16)
    _fill_same([kv_c], cases, positions, True, 31, 1)
    kv_c.decode_layer(0, Q, K, V, pos_pin, outp)
    assert np.array_equal(bits(outp.numpy()), bits(res_a[0][2]))


def test_pinned_host_buffers_short_cache(tg, backend, O, cases):
    """The reference's own case -- an fp32 cache of at most 1024 positions
    on the short-cache kernel -- with page-locked buffers inside a batch:
    inputs move by the staging kernel, the rotated q / k and the output are
    written through the buffers' device addresses (no device->host copies
    between the kernels); bit-identical to pageable buffers, RoPE and the
    cache row bit-exact, attention within the fp32 bar."""
    import torch
    positions = [0, 33, 255, 1000]
    layers = 3
    max_ctx = 1024
    kv_a = tg.KVCache(backend, layers, len(positions), max_ctx, dtype=tg.DTYPE_F32)
    kv_b = tg.KVCache(backend, layers, len(positions), max_ctx, dtype=tg.DTYPE_F32)
    inputs, refs = _fill_same([kv_a, kv_b], cases, positions, False, 57, layers)
    pos_np = np.array(positions, np.int32)
    pos_pin = torch.from_numpy(pos_np.copy()).pin_memory()
    res_a, res_b = [], []
    backend.metal_batch_begin()
    for layer in range(layers):
        Q, K, V = (x.copy() for x in inputs[layer])
        out = np.zeros_like(Q)
        kv_a.decode_layer(layer, Q, K, V, pos_np, out)
        res_a.append((Q, K, out))
        Qp, Kp, Vp = (torch.from_numpy(x.copy()).pin_memory() for x in inputs[layer])
        outp = torch.zeros(Qp.shape, dtype=torch.float32).pin_memory()
        kv_b.decode_layer(layer, Qp, Kp, Vp, pos_pin, outp)
        res_b.append((Qp, Kp, outp))
    backend.metal_batch_end()
    for layer in range(layers):
        Q, K, out = res_a[layer]
        Qp, Kp, outp = (t.numpy() for t in res_b[layer])
        assert np.array_equal(bits(Qp), bits(Q)), layer
        assert np.array_equal(bits(Kp), bits(K)), layer
        assert np.array_equal(bits(outp), bits(out)), layer
        for i, pos in enumerate(positions):
            qr, kr, vr, kc, vc, ctx = refs[layer][i]
            assert np.array_equal(bits(Qp[i]), bits(qr)), (layer, pos)
            assert np.array_equal(bits(Kp[i]), bits(kr)), (layer, pos)
            kb, vb = kv_b.read_rows(layer, i, pos, 1)
            assert np.array_equal(bits(kb[0]), bits(kc[pos])), (layer, pos)
            assert maxabs(outp[i], ctx) <= F32_TOL, (layer, pos)


@pytest.mark.parametrize("splitkv", [False, True])
def test_staged_positions_change_between_batches(tg, backend, O, cases, splitkv):
    """The bf16 decode kernel builds its tile schedule from the positions
    before its grid-dependency wait, while the staging kernel in front of it
    may still be copying them.  Batches that reuse the same staging slots
    with different positions (and so different schedules) must each decode
    with their own: a schedule built from the previous batch's positions
    gives wrong outputs or a bad-position error."""
    import torch
    P = ([9000, 40, 5000, 7], [3, 8100, 64, 6000])
    layers = 4
    max_ctx = max(max(p) for p in P) + 1
    kvs, data = [], []
    for j, positions in enumerate(P):
        kv = tg.KVCache(backend, layers, len(positions), max_ctx, dtype=tg.DTYPE_BF16)
        inputs, refs = _fill_same([kv], cases, positions, True, 71 + j, layers)
        kvs.append(kv)
        data.append((torch.from_numpy(np.array(positions, np.int32)).pin_memory(),
                     inputs, refs))
    for rnd, j in enumerate([0, 1, 0, 1]):
        kv, (pos_pin, inputs, refs) = kvs[j], data[j]
        # Every buffer of the batch stays allocated until tg_batch_end, where
        # the rotated q / k and the outputs reach the host.
        res = []
        backend.metal_batch_begin()
        for layer in range(layers):
            Qp, Kp, Vp = (torch.from_numpy(x.copy()).pin_memory() for x in inputs[layer])
            outp = torch.zeros(Qp.shape, dtype=torch.float32).pin_memory()
            (kv.decode_layer_splitkv if splitkv else kv.decode_layer)(layer, Qp, Kp, Vp,
                                                                     pos_pin, outp)
            res.append((Qp, Kp, Vp, outp))
        backend.metal_batch_end()
        for layer in range(layers):
            Qp, Kp, _, outp = (t.numpy() for t in res[layer])
            for i, pos in enumerate(P[j]):
                qr, kr, vr, kc, vc, ctx = refs[layer][i]
                assert np.array_equal(bits(Qp[i]), bits(qr)), (rnd, layer, pos)
                assert np.array_equal(bits(Kp[i]), bits(kr)), (rnd, layer, pos)
                assert maxabs(outp[i], ctx) <= BF16_TOL, (rnd, layer, pos)


# ------------------------------------------------------ split-KV on one GPU

def test_splitkv_world1_equals_batched(tg, backend, cases):
    positions = [50, 700]
    Q, _, out, refs, kv = run_batch(tg, backend, cases, positions, bf16=True, seed=12)
    out2 = np.zeros_like(out)
    kv.attention_splitkv(0, Q, np.array(positions, np.int32), out2)
    np.testing.assert_allclose(out2, out, atol=1e-6, rtol=0)


@pytest.mark.parametrize("bf16,n_shards", [(True, 2), (True, 4), (False, 3)])
def test_shard_records_merge(tg, backend, cases, bf16, n_shards):
    """A context split over shard caches (as GPUs would hold it), each
    shard's softmax records computed separately and merged."""
    positions = [5000, 1234, 0]
    B = len(positions)
    gctx = max(positions) + 1
    refs = [cases.oracle_decode(31, p, bf16, seq=i) for i, p in enumerate(positions)]
    Q = np.stack([r[0] for r in refs])
    rf = 14 * 66
    recs = np.zeros((n_shards, B, rf), np.float32)
    for r in range(n_shards):
        start, length = tg.shard_range(gctx, n_shards, r)
        sh = tg.KVCache(backend, 1, B, max(length, 1), shard_start=start,
                        global_ctx=gctx,
                        dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
        for i, p in enumerate(positions):
            kc, vc = refs[i][3], refs[i][4]
            lo, hi = start, min(start + length, p + 1)
            if hi > lo:
                sh.write_rows(0, i, 0, kc[lo:hi], vc[lo:hi])
        sh.attention_records(0, Q, np.array(positions, np.int32), recs[r])
        sh.destroy()
    out = np.zeros((B, cases.QD), np.float32)
    backend.merge_records(recs, out, n_shards, B)
    tol = BF16_TOL if bf16 else F32_TOL
    for i in range(B):
        assert maxabs(out[i], refs[i][5]) <= tol


# ------------------------------------------------------ full-size properties

def test_long_context_131072_sampled_and_properties(tg, backend, O, cases):
    """BASELINE config 4 size (context 131072, bf16): one sequence checked
    against the oracle in full; constant V and V-linearity on the same keys."""
    N = 131072
    pos = N - 1
    q, k_new, v_new, kc, vc = cases.decode_inputs(404, pos, bf16=True)
    kv = tg.KVCache(backend, 1, 1, N, dtype=tg.DTYPE_BF16)
    kv.write_rows(0, 0, 0, kc[:pos], vc[:pos])
    Q, K = q[None].copy(), k_new[None].copy()
    out = np.zeros((1, cases.QD), np.float32)
    kv.decode_layer(0, Q, K, v_new[None].copy(), np.array([pos], np.int32), out)
    ref = cases.oracle_decode(404, pos, bf16=True)
    assert maxabs(out[0], ref[5]) <= BF16_TOL
    # V == c for every row: softmax weights sum to 1, so out == c
    c = O.round_bf16(O.normal(5, 128))
    kv.write_rows(0, 0, 0, None, np.broadcast_to(c, (N, 128)).copy())
    kv.attention(0, Q, np.array([pos], np.int32), out)
    expect = np.concatenate([np.tile(c[:64], 7), np.tile(c[64:], 7)])
    assert maxabs(out[0], expect) <= 1e-5
    # linearity: out(V1 + V2) == out(V1) + out(V2).  V1, V2 and V1 + V2 are
    # multiples of 1/8 in [-8, 8], so all three are exact in bf16.
    v1 = np.clip(np.round(vc * 8) / 8, -4, 4).astype(np.float32)
    v2 = np.clip(np.round(O.normal(6, N * 128).reshape(N, 128) * 8) / 8,
                 -4, 4).astype(np.float32)
    outs = []
    for vv in (v1, v2, v1 + v2):
        kv.write_rows(0, 0, 0, None, np.ascontiguousarray(vv))
        kv.attention(0, Q, np.array([pos], np.int32), out)
        outs.append(out[0].copy())
    assert maxabs(outs[2], outs[0] + outs[1]) <= 1e-4


# ------------------------------------------------------ CUDA graphs

def test_graph_capture_replays_decode_step(tg, backend, cases):
    """Two layers of a decode step captured once and replayed give the same
    results as direct calls; host pointers are refused while capturing."""
    import torch
    positions = [40, 700, 3]
    B = len(positions)
    kv = tg.KVCache(backend, 2, B, 1024, dtype=tg.DTYPE_BF16)
    kv.fill_normal(99)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    q0 = torch.randn(2, B, 896, device="cuda", generator=g)
    k0 = torch.randn(2, B, 128, device="cuda", generator=g)
    v0 = torch.randn(2, B, 128, device="cuda", generator=g)
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")

    def run(q, k, out):
        for l in range(2):
            kv.decode_layer(l, q[l], k[l], v0[l], pos, out[l])

    qa, ka, oa = q0.clone(), k0.clone(), torch.zeros(2, B, 896, device="cuda")
    run(qa, ka, oa)                      # direct (also sizes the scratch)
    backend.synchronize()
    qb, kb, ob = q0.clone(), k0.clone(), torch.zeros(2, B, 896, device="cuda")
    n0 = backend.launch_count()
    backend.graph_begin()
    run(qb, kb, ob)
    with pytest.raises(tg.TGError) as e:  # host memory inside a capture
        kv.attention(0, np.zeros((B, 896), np.float32), np.array(positions, np.int32),
                     np.zeros((B, 896), np.float32))
    assert e.value.status == tg.TG_ERR_STATE
    graph = backend.graph_end()
    assert backend.launch_count() == n0  # recorded, not run
    graph.launch()
    backend.synchronize()
    assert backend.launch_count() > n0
    assert torch.equal(qa, qb) and torch.equal(ka, kb)
    assert torch.equal(oa, ob)
    graph.destroy()
    # kernel timing events captured into a graph are re-recorded per replay
    backend.profile_enable(True)
    backend.graph_begin()
    run(qb, kb, ob)
    gp = backend.graph_end()
    backend.profile_enable(False)
    for _ in range(2):
        gp.launch()
        ms, n = backend.profile_read()
        assert n == 2 and ms > 0
    gp.destroy()
    kv.destroy()


# ------------------------------------------------------ errors and hygiene

def test_errors_are_reported(tg, backend, cases):
    kv = tg.KVCache(backend, 1, 2, 64, dtype=tg.DTYPE_BF16)
    q = np.zeros((2, 896), np.float32)
    out = np.zeros_like(q)
    with pytest.raises(tg.TGError) as e:
        kv.attention(0, q, np.array([3, 64], np.int32), out)   # 64 >= max_ctx
    assert e.value.status == tg.TG_ERR_INVALID_ARG
    import torch
    bad = torch.tensor([3, 500], dtype=torch.int32, device="cuda")
    with pytest.raises(tg.TGError) as e:
        kv.attention(0, q, bad, out)                            # device-side check
    assert e.value.status == tg.TG_ERR_DEVICE
    kv.attention(0, q, np.array([3, 5], np.int32), out)         # context recovers
    # a device view that is only 4-byte aligned is refused before any launch
    qmis = torch.zeros(2 * 896 + 1, device="cuda")[1:].view(2, 896)
    with pytest.raises(tg.TGError) as e:
        kv.attention(0, qmis, np.array([3, 5], np.int32), out)
    assert e.value.status == tg.TG_ERR_INVALID_ARG
    with pytest.raises(tg.TGError) as e:
        backend.elem_op(1, np.zeros(4, np.float32), np.zeros(4, np.float32), 4)
    assert e.value.status == tg.TG_ERR_UNSUPPORTED
    with pytest.raises(tg.TGError) as e:
        backend.metal_batch_end()
    assert e.value.status == tg.TG_ERR_STATE
    with pytest.raises(tg.TGError):
        kv.decode_layer(1, q, np.zeros((2, 128), np.float32),
                        np.zeros((2, 128), np.float32), np.array([0, 0], np.int32), out)


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_short_cache_kernel_other_group(tg, backend, O, bf16):
    """Caches of at most 1024 positions take the one-CTA-per-(sequence, KV
    head) kernel; 12 query heads over 3 KV heads keep a bf16 cache off the
    tensor-core kernel too.  Ragged positions up to the capacity."""
    n_head, n_kv, hd, cap = 12, 3, 64, 1024
    positions = [0, 1, 31, 32, 255, 1023, 700]
    B = len(positions)
    kv = tg.KVCache(backend, 1, B, cap, n_head=n_head, n_kv_head=n_kv, head_dim=hd,
                    dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
    gen = O.normal_bf16 if bf16 else O.normal
    Q = np.stack([O.normal(50 + i, n_head * hd) for i in range(B)])
    out = np.zeros_like(Q)
    ks, vs = [], []
    for i, pos in enumerate(positions):
        kc = gen(60 + i, (pos + 1) * n_kv * hd).reshape(pos + 1, -1)
        vc = gen(70 + i, (pos + 1) * n_kv * hd).reshape(pos + 1, -1)
        kv.write_rows(0, i, 0, kc, vc)
        ks.append(kc)
        vs.append(vc)
    kv.attention(0, Q, np.array(positions, np.int32), out)
    tol = BF16_TOL if bf16 else F32_TOL
    for i, pos in enumerate(positions):
        ref = O.attention(Q[i], ks[i], vs[i], pos, n_head, n_kv, hd)
        assert maxabs(out[i], ref) <= tol, (i, pos)
    kv.destroy()


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_short_cache_decode_step_other_group(tg, backend, O, bf16):
    """The one-launch decode step of short caches (RoPE, new-row write and
    attention in the short-cache kernel) with 12 query / 3 KV heads:
    rotated q and k bit-exact, cache rows as stored, output within the bar."""
    n_head, n_kv, hd, cap = 12, 3, 64, 300
    positions = [0, 5, 299, 130]
    B = len(positions)
    kv = tg.KVCache(backend, 1, B, cap, n_head=n_head, n_kv_head=n_kv, head_dim=hd,
                    dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
    gen = O.normal_bf16 if bf16 else O.normal
    Q = np.stack([O.normal(80 + i, n_head * hd) for i in range(B)])
    K = np.stack([O.normal(90 + i, n_kv * hd) for i in range(B)])
    V = np.stack([gen(100 + i, n_kv * hd) for i in range(B)])
    caches = []
    for i, pos in enumerate(positions):
        kc = np.zeros((pos + 1, n_kv * hd), np.float32)
        vc = np.zeros_like(kc)
        if pos > 0:
            kc[:pos] = gen(110 + i, pos * n_kv * hd).reshape(pos, -1)
            vc[:pos] = gen(120 + i, pos * n_kv * hd).reshape(pos, -1)
            kv.write_rows(0, i, 0, kc[:pos], vc[:pos])
        caches.append((kc, vc))
    Qg, Kg = Q.copy(), K.copy()
    out = np.zeros_like(Q)
    kv.decode_layer(0, Qg, Kg, V, np.array(positions, np.int32), out)
    tol = BF16_TOL if bf16 else F32_TOL
    for i, pos in enumerate(positions):
        q = O.rope_heads(Q[i], n_head, hd, pos)
        k = O.rope_heads(K[i], n_kv, hd, pos)
        assert np.array_equal(bits(Qg[i]), bits(q)) and np.array_equal(bits(Kg[i]), bits(k))
        kc, vc = caches[i]
        kc[pos] = O.round_bf16(k) if bf16 else k
        vc[pos] = V[i]
        kr, vr = kv.read_rows(0, i, pos, 1)
        if bf16:
            assert np.array_equal(kr[0], O.pack_bf16(kc[pos]))
            assert np.array_equal(vr[0], O.pack_bf16(vc[pos]))
        else:
            assert np.array_equal(bits(kr[0]), bits(kc[pos]))
            assert np.array_equal(bits(vr[0]), bits(vc[pos]))
        ref = O.attention(q, kc, vc, pos, n_head, n_kv, hd)
        assert maxabs(out[i], ref) <= tol, (i, pos)
    kv.destroy()


def test_short_cache_kernel_reports_bad_positions(tg, backend, cases):
    import torch
    kv = tg.KVCache(backend, 1, 2, 64, dtype=tg.DTYPE_F32)
    q = np.zeros((2, 896), np.float32)
    out = np.zeros_like(q)
    bad = torch.tensor([3, 500], dtype=torch.int32, device="cuda")
    with pytest.raises(tg.TGError) as e:
        kv.attention(0, q, bad, out)                            # device-side check
    assert e.value.status == tg.TG_ERR_DEVICE
    kv.attention(0, q, np.array([3, 5], np.int32), out)         # context recovers
    kv.destroy()


def test_outputs_leave_neighbours_untouched(tg, backend, cases):
    import torch
    positions = [10, 3000]
    Q, _, out, refs, kv = run_batch(tg, backend, cases, positions, bf16=True, seed=8)
    buf = torch.full((4 * 896,), float("nan"), device="cuda")
    view = buf[896:3 * 896]
    kv.attention(0, torch.from_numpy(Q).cuda(), np.array(positions, np.int32), view)
    backend.synchronize()
    h = buf.cpu().numpy()
    assert np.isnan(h[:896]).all() and np.isnan(h[3 * 896:]).all()
    np.testing.assert_allclose(h[896:3 * 896].reshape(2, 896), out, atol=1e-6, rtol=0)
