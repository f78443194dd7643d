"""Pins the oracle's quantized Q/K/V projection (oracle/tg_oracle.c:
tgo_f16_to_f32, tgo_dequant, tgo_matmul_q, tgo_qkv_step) before it is
trusted as the checker of the CUDA projection kernel: bit-for-bit against
golden_qkv.npz, which the reference's own layer step (tmac_gguf.cpp:1045-1128
with its weight decoding :220-415 and matmul :476-514) produced, and against
the reference build directly where oracle/_ref/libref.so is present."""
from __future__ import annotations

import hashlib

import numpy as np
import pytest


def _sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _case_inputs(O, cases, seed, vt, bias, pos):
    wq, wk, wv, bq, bk, bv = cases.qkv_weights(seed, vt, bias)
    x = cases.qkv_x(seed)[0]
    kc = np.zeros((pos + 1, cases.KD), np.float32)
    vc = np.zeros((pos + 1, cases.KD), np.float32)
    if pos > 0:
        kc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_KC), pos * cases.KD).reshape(pos, -1)
        vc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_VC), pos * cases.KD).reshape(pos, -1)
    return wq, wk, wv, bq, bk, bv, x, kc, vc


def test_qkv_inputs_are_stable(golden_qkv, O, cases):
    seed = int(golden_qkv["seed"])
    for i, (vt, bias, pos) in enumerate(golden_qkv["cases"]):
        wq, wk, wv, bq, bk, bv, x, kc, vc = _case_inputs(O, cases, seed + i, int(vt),
                                                         bool(bias), int(pos))
        sha = _sha(wq, wk, wv, *(b for b in (bq, bk, bv) if b is not None), x, kc, vc)
        assert sha == str(golden_qkv["qkv_in_sha"][i])


def test_qkv_step_matches_reference_golden(golden_qkv, O, cases):
    """Projections, bias adds, RoPE, cache-write and attention of the oracle
    equal the reference's outputs bit for bit."""
    seed = int(golden_qkv["seed"])
    for i, (vt, bias, pos) in enumerate(golden_qkv["cases"]):
        vt, pos = int(vt), int(pos)
        wq, wk, wv, bq, bk, bv, x, kc, vc = _case_inputs(O, cases, seed + i, vt, bool(bias), pos)
        q, k, v = O.qkv_step(wq, wk, wv, bq, bk, bv, x, pos, v_type=vt, k_cache=kc, v_cache=vc)
        ctx = O.attention(q, kc, vc, pos)
        assert np.array_equal(bits(q), bits(golden_qkv["qkv_q"][i])), i
        assert np.array_equal(bits(k), bits(golden_qkv["qkv_k"][i])), i
        assert np.array_equal(bits(v), bits(golden_qkv["qkv_v"][i])), i
        assert np.array_equal(bits(ctx), bits(golden_qkv["qkv_ctx"][i])), i
        assert np.array_equal(bits(kc[pos]), bits(k)) and np.array_equal(bits(vc[pos]), bits(v))


def test_attention_block_matches_reference_golden(golden_qkv, O, cases):
    """Projection step + attention + attn_output matmul + residual add of the
    oracle equal the reference's tmac_gguf.cpp:1045-1140 bit for bit."""
    seed0 = int(golden_qkv["seed"])
    for i, (vt, ot, bias, pos) in enumerate(golden_qkv["blk_cases"]):
        vt, ot, pos = int(vt), int(ot), int(pos)
        seed = seed0 + 100 + i
        wq, wk, wv, bq, bk, bv = cases.qkv_weights(seed, vt, bool(bias))
        wo = cases.attn_output_weight(seed, ot)
        x = cases.qkv_x(seed)[0]
        h0 = cases.residual_in(seed)[0]
        kc = np.zeros((pos + 1, cases.KD), np.float32)
        vc = np.zeros((pos + 1, cases.KD), np.float32)
        if pos > 0:
            kc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_KC), pos * cases.KD).reshape(pos, -1)
            vc[:pos] = O.normal(O.derive_seed(seed, 0, 0, cases.T_VC), pos * cases.KD).reshape(pos, -1)
        sha = _sha(wq, wk, wv, *(b for b in (bq, bk, bv) if b is not None), wo, x, h0, kc, vc)
        assert sha == str(golden_qkv["blk_in_sha"][i])
        q, k, v = O.qkv_step(wq, wk, wv, bq, bk, bv, x, pos, v_type=vt, k_cache=kc, v_cache=vc)
        ctx = O.attention(q, kc, vc, pos)
        hid = O.attn_output(ot, wo, ctx, h0)
        assert np.array_equal(bits(hid), bits(golden_qkv["blk_hidden"][i])), i


def test_f16_widening_known_answers(O):
    L = O.lib()
    known = {0x0000: 0.0, 0x8000: 0.0, 0x3c00: 1.0, 0xc000: -2.0, 0x0001: 2.0 ** -24,
             0x03ff: 1023 * 2.0 ** -24, 0x0400: 2.0 ** -14, 0x7bff: 65504.0,
             0x7c00: np.inf, 0xfc00: -np.inf, 0x3555: 0.333251953125}
    for h, want in known.items():
        assert L.tgo_f16_to_f32(h) == want, hex(h)
    assert np.isnan(L.tgo_f16_to_f32(0x7e00))
    # The reference maps -0 to +0 (tmac_gguf.cpp:225).
    assert np.copysign(1.0, L.tgo_f16_to_f32(0x8000)) == 1.0


def test_q5_0_layout_known_answer(O):
    """One hand-built Q5_0 block: d = 0.5, element j < 16 in the low nibble
    of byte j, element j >= 16 in the high nibble of byte j-16, high bit j
    of the 32-bit word; value d*(q - 16)."""
    blk = np.zeros(22, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    blk[2:6] = np.frombuffer(np.uint32(0x80000001).tobytes(), np.uint8)
    blk[6] = 0xF3          # element 0 low nibble 3, element 16 high nibble 15
    blk[6 + 15] = 0x0A     # element 15 low nibble 10, element 31 high nibble 0
    L = O.lib()
    vals = [L.tgo_dequant(O.TYPE_Q5_0, blk, j) for j in range(32)]
    assert vals[0] == 0.5 * ((1 << 4 | 3) - 16)     # high bit 0 set
    assert vals[16] == 0.5 * (15 - 16)
    assert vals[15] == 0.5 * (10 - 16)
    assert vals[31] == 0.5 * ((1 << 4 | 0) - 16)    # high bit 31 set
    assert vals[1] == 0.5 * -16


def test_q8_0_layout_known_answer(O):
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(-0.25).tobytes(), np.uint8)
    blk[2:34] = np.arange(32, dtype=np.int8).astype(np.uint8) - np.uint8(16)
    L = O.lib()
    assert [L.tgo_dequant(O.TYPE_Q8_0, blk, j) for j in range(32)] == \
        [-0.25 * (j - 16) for j in range(32)]


def test_planted_bias_error_is_caught(golden_qkv, O, cases):
    """The golden check can fail: one bias element off by one ulp changes
    the oracle's q and the comparison sees it."""
    seed = int(golden_qkv["seed"])
    vt, bias, pos = (int(v) for v in golden_qkv["cases"][0])
    wq, wk, wv, bq, bk, bv, x, kc, vc = _case_inputs(O, cases, seed, vt, bool(bias), pos)
    bq = bq.copy()
    bq[100] = np.nextafter(bq[100], np.float32(np.inf))
    q, _, _ = O.qkv_step(wq, wk, wv, bq, bk, bv, x, pos, v_type=vt, k_cache=kc, v_cache=vc)
    assert not np.array_equal(bits(q), bits(golden_qkv["qkv_q"][0]))


@pytest.mark.skipif("not __import__('oracle').ref_available()")
@pytest.mark.parametrize("wtype,rows,cols", [(6, 64, 896), (8, 64, 896), (6, 3, 4864),
                                             (8, 5, 32), (0, 7, 96)])
def test_matmul_equals_reference_build(O, wtype, rows, cols):
    if wtype == O.TYPE_F32:
        w = O.normal(31, rows * cols).view(np.uint8).reshape(rows, -1)
    else:
        w = O.qblocks(wtype, 31 + wtype, rows, cols, 0.004)
    x = O.normal(32, cols)
    a = O.matmul_q(wtype, w, x, rows, cols)
    b = O.ref_matmul(wtype, w, x, rows, cols)
    assert np.array_equal(bits(a), bits(b))


@pytest.mark.skipif("not __import__('oracle').ref_available()")
def test_f16_widening_equals_reference_build_exhaustively(O):
    L, R = O.lib(), O.ref()
    for h in range(65536):
        a, b = L.tgo_f16_to_f32(h), R.tgref_f16_to_f32(h)
        assert (a == b and np.copysign(1, a) == np.copysign(1, b)) or (a != a and b != b), hex(h)
