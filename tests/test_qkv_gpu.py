"""Parity of the CUDA Q/K/V projection (tg_qkv.cu) with the CPU oracle,
through the C ABI: fused_qkv_op / matmul_q (the reference's operator
surface, metal_backend.hpp:320-338 and :456-489), the fused layer step
tg_qkv_rope_cache_write / tg_decode_layer_x (tmac_gguf.cpp:1046-1128), the
attn_output matvec with its residual add (tg_attn_output, :1129-1140) and
the whole attention block (tg_attention_block, :1045-1140).

Bars, written per check:
  * weight decoding is exact: the kernel's products use the dequantised
    values the reference computes (an fp16 scale times a small integer);
  * a projected value may differ from the oracle's j-ordered binary32 sum
    only by summation order: |gpu - oracle| <= 2 * cols * 2^-24 * sum_j |w_j x_j|
    (twice the textbook bound on the rounding error of an n-term sum), plus
    one rounding of the bias add;
  * RoPE rotates the projected pair with the reference's arithmetic, so a
    rotated value is bounded by the two inputs' bounds plus 4 ulp;
  * a bf16 cache row additionally rounds once to bf16;
  * attention on the kernel's own q and cache rows: max-abs <= 1e-4 (fp32
    cache) or 2e-3 (bf16 cache), as for the attention-only path.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

U = 2.0 ** -24
F32_TOL = 1e-4
BF16_TOL = 2e-3


def dequant_np(O, wtype, w, rows, cols):
    """Vectorised Q5_0 / Q8_0 decoding (for the error bound only; checked
    against the oracle's element decoding below)."""
    bs = O.BLOCK_BYTES[wtype]
    blk = np.ascontiguousarray(w, np.uint8).reshape(rows, cols // 32, bs)
    d = blk[..., 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    d[d == 0] = 0.0
    if wtype == O.TYPE_Q8_0:
        q = blk[..., 2:34].copy().view(np.int8).astype(np.float32)
    else:
        qh = blk[..., 2:6].copy().view(np.uint32)[..., 0]
        qs = blk[..., 6:22]
        lo = np.concatenate([qs & 15, qs >> 4], axis=-1).astype(np.int32)
        hi = ((qh[..., None] >> np.arange(32, dtype=np.uint32)) & 1).astype(np.int32)
        q = ((hi << 4) | lo).astype(np.float32) - 16
    return (d[..., None] * q).reshape(rows, cols)


def sum_bound(Wf, x):
    """Per-row bound on |gpu - oracle| from summation order alone."""
    n = Wf.shape[1]
    return 2.0 * n * U * (np.abs(Wf.astype(np.float64)) @ np.abs(x.astype(np.float64))) + 1e-30


def ulp(a):
    a = np.abs(np.asarray(a, np.float32))
    return np.spacing(a).astype(np.float64)


def check_within(gpu, ref, bound, what):
    err = np.abs(np.asarray(gpu, np.float64) - np.asarray(ref, np.float64))
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, (f"{what}: {bad.size} values out of bound, first {bad[:5]}: "
                           f"err {err[bad[:5]]} bound {np.asarray(bound)[bad[:5]]}")


def as_f32(a):
    """Cache rows read back: fp32 as is, bf16 bit patterns widened."""
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def rot_bound(b_pre, y):
    """Bound of rotated values from the bounds of the pair before rotation."""
    pair = b_pre.reshape(-1, 2).sum(axis=1).repeat(2)
    return pair + 4.0 * ulp(y)


def test_dequant_np_matches_oracle(O, cases):
    for wt in (O.TYPE_Q5_0, O.TYPE_Q8_0):
        w = O.qblocks(wt, 5 + wt, 4, 96, cases.D_SCALE[wt])
        a = dequant_np(O, wt, w, 4, 96)
        b = O.dequant_rows(wt, w, 4, 96)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ------------------------------------------------ reference operator surface

@pytest.mark.parametrize("v_q8", [False, True])
def test_fused_qkv_op_matches_oracle(backend, O, cases, v_q8):
    vt = O.TYPE_Q8_0 if v_q8 else O.TYPE_Q5_0
    wq, wk, wv, *_ = cases.qkv_weights(71, vt, bias=False)
    x = cases.qkv_x(72)[0].copy()
    yq = np.zeros(cases.QD, np.float32)
    yk = np.zeros(cases.KD, np.float32)
    yv = np.zeros(cases.KD, np.float32)
    backend.fused_qkv_op(wq, wk, wv, x, yq, yk, yv, cases.QD, cases.KD, cases.KD, 896, v_q8)
    for y, w, t, rows in ((yq, wq, O.TYPE_Q5_0, cases.QD), (yk, wk, O.TYPE_Q5_0, cases.KD),
                          (yv, wv, vt, cases.KD)):
        ref = O.matmul_q(t, w, x, rows, 896)
        check_within(y, ref, sum_bound(dequant_np(O, t, w, rows, 896), x), f"type {t}")


@pytest.mark.parametrize("wtype,rows,cols", [
    (6, 896, 896),    # attn_q / attn_output shape
    (8, 896, 896),
    (6, 64, 4864),    # an FFN down projection's 4864 inputs
    (6, 5, 32),       # one block per row, rows not a multiple of 8 (2-byte staging)
    (8, 13, 96),      # cols not a multiple of 128 (scalar dot path)
])
def test_matmul_q_matches_oracle(backend, O, wtype, rows, cols):
    w = O.qblocks(wtype, 90 + rows, rows, cols, 0.004 if wtype == 6 else 0.0005)
    x = O.normal(91, cols)
    y = np.zeros(rows, np.float32)
    backend.matmul_q(wtype, rows, cols, w, x, y)
    ref = O.matmul_q(wtype, w, x, rows, cols)
    check_within(y, ref, sum_bound(dequant_np(O, wtype, w, rows, cols), x), "matmul_q")


def test_matmul_q_unaligned_device_input(backend, O):
    """x on the device at an address that is 4- but not 16-byte aligned:
    the kernel takes its scalar-load path."""
    import torch
    rows, cols = 24, 896
    w = O.qblocks(6, 93, rows, cols, 0.004)
    x = O.normal(94, cols)
    buf = torch.zeros(cols + 1, dtype=torch.float32, device="cuda")
    buf[1:] = torch.from_numpy(x).cuda()
    xd = buf[1:]
    assert xd.data_ptr() % 16 != 0
    wd = torch.from_numpy(w).cuda()
    yd = torch.zeros(rows, dtype=torch.float32, device="cuda")
    backend.matmul_q(6, rows, cols, wd, xd, yd)
    backend.synchronize()
    ref = O.matmul_q(6, w, x, rows, cols)
    check_within(yd.cpu().numpy(), ref, sum_bound(dequant_np(O, 6, w, rows, cols), x), "matmul_q")


def test_matmul_q_rejects_bad_shapes(backend, tg, O):
    w = O.qblocks(6, 1, 4, 64)
    x = O.normal(2, 64)
    y = np.zeros(4, np.float32)
    with pytest.raises(tg.TGError) as e:
        backend.matmul_q(6, 4, 48, w, x, y)     # cols not a multiple of 32
    assert e.value.status == tg.TG_ERR_INVALID_ARG
    with pytest.raises(tg.TGError) as e:
        backend.matmul_q(12, 4, 64, w, x, y)    # Q4_K: not this path
    assert e.value.status == tg.TG_ERR_UNSUPPORTED


def test_fused_qkv_op_in_batch_with_registered_weights(backend, tg, O, cases):
    """The reference's pattern: weights registered once (uploaded once),
    the op encoded inside metal_batch_begin / metal_batch_end with its bias
    adds (elem_op 0) following on the same host arrays."""
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(81, O.TYPE_Q8_0, bias=True)
    for w in (wq, wk, wv):
        backend.register_host(w, tg.REGION_DEVICE_OWNED)
    try:
        for step in range(2):
            x = cases.qkv_x(82 + step)[0].copy()
            yq = np.zeros(cases.QD, np.float32)
            yk = np.zeros(cases.KD, np.float32)
            yv = np.zeros(cases.KD, np.float32)
            backend.metal_batch_begin()
            backend.fused_qkv_op(wq, wk, wv, x, yq, yk, yv, cases.QD, cases.KD, cases.KD,
                                 896, True)
            backend.elem_op(0, yq, bq, cases.QD)
            backend.elem_op(0, yk, bk, cases.KD)
            backend.elem_op(0, yv, bv, cases.KD)
            backend.metal_batch_end()
            for y, w, t, b, rows in ((yq, wq, 6, bq, cases.QD), (yk, wk, 6, bk, cases.KD),
                                     (yv, wv, 8, bv, cases.KD)):
                ref = O.matmul_q(t, w, x, rows, 896) + b
                bound = sum_bound(dequant_np(O, t, w, rows, 896), x) + ulp(ref)
                check_within(y, ref, bound, f"step {step} type {t}")
    finally:
        for w in (wq, wk, wv):
            backend.unregister_host(w)


# ------------------------------------------------ fused layer step

def _layer_case(tg, backend, O, cases, positions, bf16, vt, bias, seed):
    """A cache with rows 0..pos-1 of every sequence filled, the layer's
    weights and inputs, and the oracle's q / k / v per sequence."""
    B = len(positions)
    max_ctx = max(positions) + 1
    kv = tg.KVCache(backend, 1, B, max_ctx, dtype=tg.DTYPE_BF16 if bf16 else tg.DTYPE_F32)
    gen = O.normal_bf16 if bf16 else O.normal
    for i, pos in enumerate(positions):
        if pos > 0:
            kc = gen(O.derive_seed(seed, 0, i, cases.T_KC), pos * cases.KD).reshape(pos, -1)
            vc = gen(O.derive_seed(seed, 0, i, cases.T_VC), pos * cases.KD).reshape(pos, -1)
            kv.write_rows(0, i, 0, kc, vc)
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(seed, vt, bias)
    W = tg.QKVWeights(wq, wk, wv, 896, v_type=vt, b_q=bq, b_k=bk, b_v=bv)
    X = cases.qkv_x(seed + 1, B).copy()
    refs = [O.qkv_step(wq, wk, wv, bq, bk, bv, X[i], pos, v_type=vt)
            for i, pos in enumerate(positions)]
    bounds = []
    for i in range(B):
        bqk = [sum_bound(dequant_np(O, O.TYPE_Q5_0, w, r, 896), X[i])
               for w, r in ((wq, cases.QD), (wk, cases.KD))]
        bv_ = sum_bound(dequant_np(O, vt, wv, cases.KD, 896), X[i])
        q, k, v = refs[i]
        bounds.append((rot_bound(bqk[0] + ulp(q), q), rot_bound(bqk[1] + ulp(k), k),
                       bv_ + ulp(v)))
    return kv, W, X, refs, bounds


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("vt,bias", [(6, True), (8, True), (6, False)])
def test_qkv_rope_cache_write_matches_oracle(tg, backend, O, cases, bf16, vt, bias):
    positions = [0, 5, 63, 17, 200, 1]
    kv, W, X, refs, bounds = _layer_case(tg, backend, O, cases, positions, bf16, vt, bias, 301)
    q_out = np.zeros((len(positions), cases.QD), np.float32)
    kv.qkv_rope_cache_write(0, W, X, positions, q_out)
    for i, pos in enumerate(positions):
        q, k, v = refs[i]
        bq, bk, bv = bounds[i]
        check_within(q_out[i], q, bq, f"q seq {i}")
        kr, vr = kv.read_rows(0, i, pos, 1)
        kr = as_f32(kr).reshape(-1)
        vr = as_f32(vr).reshape(-1)
        if bf16:
            # bf16 rows: one more rounding (at most half a bf16 ulp, 2^-9 |x|).
            check_within(kr, k, bk + np.abs(k) * 2.0 ** -8, f"k row seq {i}")
            check_within(vr, v, bv + np.abs(v) * 2.0 ** -8, f"v row seq {i}")
        else:
            check_within(kr, k, bk, f"k row seq {i}")
            check_within(vr, v, bv, f"v row seq {i}")


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("B", [37, 130])
def test_qkv_batched_path_matches_oracle(tg, backend, O, cases, bf16, B):
    """Batches of 9 or more sequences take the batched kernel (16 rows x 64
    sequences per CTA); 37 leaves a partial group, 130 spans three."""
    rng = np.random.default_rng(B)
    positions = [int(v) for v in rng.integers(0, 300, size=B)]
    kv, W, X, refs, bounds = _layer_case(tg, backend, O, cases, positions, bf16, 8, True,
                                         700 + B)
    q_out = np.zeros((B, cases.QD), np.float32)
    kv.qkv_rope_cache_write(0, W, X, positions, q_out)
    for i, pos in enumerate(positions):
        q, k, v = refs[i]
        bq, bk, bv = bounds[i]
        check_within(q_out[i], q, bq, f"q seq {i}")
        kr, vr = kv.read_rows(0, i, pos, 1)
        kr = as_f32(kr).reshape(-1)
        vr = as_f32(vr).reshape(-1)
        slack_k = np.abs(k) * 2.0 ** -8 if bf16 else 0.0
        slack_v = np.abs(v) * 2.0 ** -8 if bf16 else 0.0
        check_within(kr, k, bk + slack_k, f"k row seq {i}")
        check_within(vr, v, bv + slack_v, f"v row seq {i}")
    kv.destroy()


@pytest.mark.parametrize("split", [1, 2, 3, 4, 7, 8])
def test_qkv_batched_every_cluster_width(tg, backend, O, cases, split):
    """The tensor-core projection at each cluster width (the CTAs of a
    cluster split the columns and sum their partials in rank order): RoPE
    pairs, bias and bf16 cache rows of 70 sequences (a partial second
    group; rank k finishes sequences 64k/S.. of each group)."""
    B = 70
    rng = np.random.default_rng(900 + split)
    positions = [int(v) for v in rng.integers(0, 300, size=B)]
    kv, W, X, refs, bounds = _layer_case(tg, backend, O, cases, positions, True, 8, True,
                                         910 + split)
    q_out = np.zeros((B, cases.QD), np.float32)
    tg.set_projection_split(split)
    try:
        kv.qkv_rope_cache_write(0, W, X, positions, q_out)
        backend.synchronize()
    finally:
        tg.set_projection_split(0)
    for i, pos in enumerate(positions):
        q, k, v = refs[i]
        bq, bk, bv = bounds[i]
        check_within(q_out[i], q, bq, f"q seq {i}")
        kr, vr = kv.read_rows(0, i, pos, 1)
        check_within(as_f32(kr).reshape(-1), k, bk + np.abs(k) * 2.0 ** -8, f"k row seq {i}")
        check_within(as_f32(vr).reshape(-1), v, bv + np.abs(v) * 2.0 ** -8, f"v row seq {i}")
    kv.destroy()


@pytest.mark.parametrize("split", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("B,ot,rows,cols", [(70, 8, 200, 896), (20, 6, 256, 224),
                                            (12, 8, 130, 32)])
def test_attn_output_every_cluster_width(tg, backend, O, cases, split, B, ot, rows, cols):
    """attn_output on the tensor cores at each cluster width: 7 chunks over
    4 or 8 ranks leave ranks of 1 and 2 chunks, a single chunk clamps the
    width to 1, widths 3, 5, 6 and 7 split the 64 sequence columns of a
    group unevenly; the residual add happens once per value."""
    wo = O.qblocks(ot, 811 + B + split, rows, cols, cases.D_SCALE[ot])
    ctx = O.normal(812 + split, B * cols).reshape(B, cols)
    h0 = O.normal(813 + split, B * rows).reshape(B, rows)
    hid = h0.copy()
    tg.set_projection_split(split)
    try:
        backend.attn_output(ot, wo, rows, cols, ctx, hid, n_seqs=B)
    finally:
        tg.set_projection_split(0)
    Wf = dequant_np(O, ot, wo, rows, cols)
    for s in range(B):
        ref = h0[s] + O.matmul_q(ot, wo, ctx[s], rows, cols)
        check_within(hid[s], ref, sum_bound(Wf, ctx[s]) + ulp(ref), f"seq {s}")


def test_fixed_cluster_width_on_the_first_launch():
    """A fixed width on a process's first tensor-core launch (nothing before
    it has opted the kernel in to its shared-memory request)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = (
        "import sys, numpy as np\n"
        f"sys.path[:0] = [{root!r}, {os.path.join(root, 'tests')!r}, {os.path.join(root, 'oracle')!r}]\n"
        "from conftest import load_package\n"
        "import oracle as O\n"
        "tg = load_package()\n"
        "tg.set_projection_split(4)\n"
        "be = tg.CudaBackend(0)\n"
        "rows, cols, B = 128, 256, 16\n"
        "w = O.qblocks(8, 5, rows, cols, 0.01)\n"
        "x = O.normal(6, B * cols).reshape(B, cols)\n"
        "h = np.zeros((B, rows), np.float32)\n"
        "be.attn_output(8, w, rows, cols, x, h, n_seqs=B)\n"
        "ref = np.stack([O.matmul_q(8, w, x[s], rows, cols) for s in range(B)])\n"
        "assert np.allclose(h, ref, rtol=1e-5, atol=1e-5), float(np.max(np.abs(h - ref)))\n"
        "print('ok')\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_projection_split_rejects_other_widths(tg):
    for bad in (9, -1, 16):
        with pytest.raises(tg.TGError):
            tg.set_projection_split(bad)
    tg.set_projection_split(0)


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_decode_layer_x_matches_oracle(tg, backend, O, cases, bf16):
    """x -> attention output in one call; attention checked on the kernel's
    own q and cache rows with the attention bars."""
    positions = [3, 64, 130, 0, 255, 31, 32, 33]
    seed = 401
    kv, W, X, refs, bounds = _layer_case(tg, backend, O, cases, positions, bf16, 6, True, seed)
    out = np.zeros((len(positions), cases.QD), np.float32)
    kv.decode_layer_x(0, W, X, positions, out)
    # The projected q (same kernel, same inputs) from a second call on a
    # fresh copy of the cache state.
    kv2, W2, X2, _, _ = _layer_case(tg, backend, O, cases, positions, bf16, 6, True, seed)
    q_out = np.zeros_like(out)
    kv2.qkv_rope_cache_write(0, W2, X2, positions, q_out)
    tol = BF16_TOL if bf16 else F32_TOL
    for i, pos in enumerate(positions):
        check_within(q_out[i], refs[i][0], bounds[i][0], f"q seq {i}")
        kc, vc = kv.read_rows(0, i, 0, pos + 1)
        kc = as_f32(kc).reshape(pos + 1, -1)
        vc = as_f32(vc).reshape(pos + 1, -1)
        ref = O.attention(q_out[i], kc, vc, pos)
        err = float(np.max(np.abs(out[i].astype(np.float64) - ref)))
        assert err <= tol, (i, pos, err)
    kv.destroy()
    kv2.destroy()


@pytest.mark.parametrize("B,ot,rows,cols", [(1, 6, 896, 896), (1, 8, 896, 896),
                                            (20, 6, 896, 896), (70, 8, 200, 896),
                                            (20, 6, 96, 1056), (20, 6, 96, 1088)])
def test_attn_output_matches_oracle(tg, backend, O, cases, B, ot, rows, cols):
    """hidden += W_o context (tmac_gguf.cpp:1129-1140): the product within
    the summation-order bound, then one rounding of the add.  B >= 9 takes
    the tensor-core kernel (3xTF32; 200 rows leave a partial 128-row tile,
    70 sequences a partial group; 1056 columns are its limit), or past it
    (1088) the CUDA-core batched kernel."""
    wo = O.qblocks(ot, 801 + B, rows, cols, cases.D_SCALE[ot])
    ctx = O.normal(802, B * cols).reshape(B, cols)
    h0 = O.normal(803, B * rows).reshape(B, rows)
    hid = h0.copy()
    backend.attn_output(ot, wo, rows, cols, ctx, hid, n_seqs=B)
    Wf = dequant_np(O, ot, wo, rows, cols)
    for s in range(B):
        ref = h0[s] + O.matmul_q(ot, wo, ctx[s], rows, cols)
        check_within(hid[s], ref, sum_bound(Wf, ctx[s]) + ulp(ref), f"seq {s}")


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
@pytest.mark.parametrize("B", [5, 12])
def test_attention_block_matches_oracle(tg, backend, O, cases, bf16, B):
    """x -> projection -> attention -> hidden += W_o context in one call.
    The attention part is checked through decode_layer_x on a copy of the
    cache state (test_decode_layer_x_matches_oracle bounds it against the
    oracle); hidden must equal h0 + W_o . context of that context within
    the summation-order bound."""
    rng = np.random.default_rng(B)
    positions = [int(v) for v in rng.integers(0, 200, size=B)]
    seed = 900 + B
    kv, W, X, refs, bounds = _layer_case(tg, backend, O, cases, positions, bf16, 8, True, seed)
    kv2, W2, X2, _, _ = _layer_case(tg, backend, O, cases, positions, bf16, 8, True, seed)
    wo = cases.attn_output_weight(seed, 6)
    h0 = cases.residual_in(seed, B)
    hid = h0.copy()
    kv.attention_block(0, W, wo, X, positions, hid, o_type=6)
    ctx = np.zeros((B, cases.QD), np.float32)
    kv2.decode_layer_x(0, W2, X2, positions, ctx)
    Wf = dequant_np(O, 6, wo, cases.QD, cases.QD)
    for s in range(B):
        ref = O.attn_output(6, wo, ctx[s], h0[s])
        check_within(hid[s], ref, sum_bound(Wf, ctx[s]) + ulp(ref), f"seq {s}")
        # and the caches hold the same new rows
        a = kv.read_rows(0, s, positions[s], 1)
        b = kv2.read_rows(0, s, positions[s], 1)
        assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    kv.destroy()
    kv2.destroy()


def test_qkv_on_a_shard_that_does_not_hold_the_position(tg, backend, O, cases):
    """Split-KV shards: the row is written only by the shard holding pos;
    q is produced on every shard."""
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(501, 6, True)
    W = tg.QKVWeights(wq, wk, wv, 896, b_q=bq, b_k=bk, b_v=bv)
    x = cases.qkv_x(502, 1).copy()
    kv = tg.KVCache(backend, 1, 1, 64, dtype=tg.DTYPE_F32, shard_start=64, global_ctx=128)
    q_out = np.zeros((1, cases.QD), np.float32)
    kv.qkv_rope_cache_write(0, W, x, [10], q_out)
    k, v = kv.read_rows(0, 0, 0, 64)
    assert not np.any(np.asarray(k)) and not np.any(np.asarray(v))
    q, _, _ = O.qkv_step(wq, wk, wv, bq, bk, bv, x[0], 10)
    bound = rot_bound(sum_bound(dequant_np(O, 6, wq, cases.QD, 896), x[0]) + ulp(q), q)
    check_within(q_out[0], q, bound, "q")
    kv.qkv_rope_cache_write(0, W, x, [70], q_out)
    k, v = kv.read_rows(0, 0, 6, 1)
    assert np.any(np.asarray(k)) and np.any(np.asarray(v))
    kv.destroy()


def test_decode_layer_x_device_tensors_and_graph(tg, backend, O, cases):
    """Weights, x, positions and output as device tensors; the step captured
    into a CUDA graph and replayed gives the direct call's result."""
    import torch
    positions = [40, 7, 99]
    B = len(positions)
    kv = tg.KVCache(backend, 1, B, 128, dtype=tg.DTYPE_BF16)
    kv.fill_normal(603)
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(601, 8, True)
    dev = [torch.from_numpy(a).cuda() for a in (wq, wk, wv, bq, bk, bv)]
    W = tg.QKVWeights(*dev[:3], 896, v_type=8, b_q=dev[3], b_k=dev[4], b_v=dev[5])
    x_d = torch.from_numpy(cases.qkv_x(602, B).copy()).cuda()
    pos_d = torch.tensor(positions, dtype=torch.int32, device="cuda")
    out_a = torch.zeros((B, cases.QD), dtype=torch.float32, device="cuda")
    kv.decode_layer_x(0, W, x_d, pos_d, out_a)       # direct (sizes the scratch)
    backend.synchronize()
    out_b = torch.zeros_like(out_a)
    backend.graph_begin()
    kv.decode_layer_x(0, W, x_d, pos_d, out_b)
    g = backend.graph_end()
    assert not torch.any(out_b)                      # recorded, not run
    g.launch()
    backend.synchronize()
    assert torch.equal(out_a, out_b)
    g.destroy()
    kv.destroy()
