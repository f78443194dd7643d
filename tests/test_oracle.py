"""Pins the CPU oracle (oracle/tg_oracle.c) before it is trusted as the
checker: bit-for-bit against the golden fixtures that the reference's own
code produced (tests/golden/make_golden.py), and, where the reference build
oracle/_ref/libref.so is present, against the reference directly."""
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


def test_input_stream_is_stable(golden, O, cases):
    """The seeded generator still produces the inputs the fixtures used."""
    seed = int(golden["seed"])
    q0 = O.normal(O.derive_seed(seed, 0, 0, 11), cases.QD)
    k0 = O.normal(O.derive_seed(seed, 0, 0, 12), cases.KD)
    assert _sha(q0, k0) == str(golden["rope_in_sha"])
    for tag, bf16 in (("f32", False), ("bf16", True)):
        for pos, sha in zip(golden[f"dec_{tag}_pos"], golden[f"dec_{tag}_in_sha"]):
            assert _sha(*cases.decode_inputs(seed, int(pos), bf16)) == str(sha)
    q, k, v = cases.prefill_inputs(seed, int(golden["prefill_S"]))
    assert _sha(q, k, v) == str(golden["prefill_in_sha"])


def test_normal_stream_statistics(O):
    x = O.normal(123, 200000)
    assert abs(float(x.mean())) < 0.01
    assert abs(float(x.std()) - 1.0) < 0.01
    assert np.array_equal(O.normal(123, 1000), x[:1000])


def test_rope_matches_reference_golden(golden, O, cases):
    seed = int(golden["seed"])
    q0 = O.normal(O.derive_seed(seed, 0, 0, 11), cases.QD)
    k0 = O.normal(O.derive_seed(seed, 0, 0, 12), cases.KD)
    for i, pos in enumerate(golden["rope_pos"]):
        q = O.rope_heads(q0, O.N_HEAD, O.HEAD_DIM, int(pos))
        k = O.rope_heads(k0, O.N_KV_HEAD, O.HEAD_DIM, int(pos))
        assert np.array_equal(bits(q), bits(golden["rope_q"][i])), pos
        assert np.array_equal(bits(k), bits(golden["rope_k"][i])), pos


def test_rope_cos_sin_table_matches_rotation(O):
    """The (cos, sin) pairs the device table holds rotate exactly like
    apply_rope when each product and sum is rounded once."""
    x = O.normal(77, 64)
    for pos in (0, 3, 255, 4095, 131071):
        cs = O.rope_cos_sin(64, pos)
        c, s = cs[0::2], cs[1::2]
        x0, x1 = x[0::2], x[1::2]
        y = np.empty_like(x)
        y[0::2] = (x0 * c).astype(np.float32) - (x1 * s).astype(np.float32)
        y[1::2] = (x0 * s).astype(np.float32) + (x1 * c).astype(np.float32)
        assert np.array_equal(bits(y), bits(O.rope_heads(x, 1, 64, pos)))


@pytest.mark.parametrize("tag,bf16", [("f32", False), ("bf16", True)])
def test_decode_matches_reference_golden(golden, O, cases, tag, bf16):
    seed = int(golden["seed"])
    for i, pos in enumerate(golden[f"dec_{tag}_pos"]):
        q, k, _, _, _, ctx = cases.oracle_decode(seed, int(pos), bf16)
        assert np.array_equal(bits(q), bits(golden[f"dec_{tag}_q"][i]))
        assert np.array_equal(bits(k), bits(golden[f"dec_{tag}_k"][i]))
        assert np.array_equal(bits(ctx), bits(golden[f"dec_{tag}_out"][i])), pos


def test_prefill_matches_reference_golden(golden, O, cases):
    seed = int(golden["seed"])
    S = int(golden["prefill_S"])
    q, k, v = cases.prefill_inputs(seed, S)
    out = O.prefill_causal(q, k, v)
    assert np.array_equal(bits(out), bits(golden["prefill_out"]))


@pytest.mark.skipif("not __import__('oracle').ref_available()")
@pytest.mark.parametrize("pos", [0, 2, 31, 32, 33, 511, 2047])
def test_oracle_equals_reference_build(O, cases, pos):
    """Direct check against the reference's own compiled lines."""
    q, k_new, v_new, kc, vc = cases.decode_inputs(99, pos)
    q1, k1, kc1, vc1 = q.copy(), k_new.copy(), kc.copy(), vc.copy()
    a = O.decode_step(q1, k1, v_new, kc1, vc1, pos)
    q2, k2, kc2, vc2 = q.copy(), k_new.copy(), kc.copy(), vc.copy()
    b = O.ref_decode_step(q2, k2, v_new, kc2, vc2, pos)
    assert np.array_equal(bits(a), bits(b))
    assert np.array_equal(bits(kc1), bits(kc2))
    assert np.array_equal(bits(vc1), bits(vc2))


@pytest.mark.skipif("not __import__('oracle').ref_available()")
def test_multithreaded_units_equal_serial(O, cases):
    units = [cases.oracle_decode(5, p, seq=i) for i, p in enumerate([3, 40, 130, 1])]
    q = np.stack([u[0] for u in units])
    kl = [u[3] for u in units]
    vl = [u[4] for u in units]
    pos = [3, 40, 130, 1]
    a = O.attention_units_mt(q, kl, vl, pos, n_threads=3)
    b = O.ref_attention_units_mt(q, kl, vl, pos, n_threads=2)
    for i, u in enumerate(units):
        assert np.array_equal(bits(a[i]), bits(u[5]))
        assert np.array_equal(bits(b[i]), bits(u[5]))


def test_bf16_rounding_is_rne(O):
    vals = np.array([1.0, 1.00390625, 1.005859375, 1.001953125, -2.5e-3,
                     3.0e38, 1e-40, np.inf, -np.inf], dtype=np.float32)
    r = O.round_bf16(vals)
    # 1 + 2^-8 is halfway between 1 and 1 + 2^-7: ties to even -> 1.0
    assert r[1] == np.float32(1.0)
    assert r[2] == np.float32(1.0078125)
    assert r[3] == np.float32(1.0)
    assert np.isinf(r[7]) and np.isinf(r[8])
    assert np.array_equal(O.pack_bf16(r).astype(np.uint32) << 16, bits(r))


def test_split_merge_restatement(O, cases):
    """Partial (m, l, o) states merged on the host give the oracle result:
    the algebra every split-KV kernel and the cross-GPU merge rely on."""
    pos = 300
    q, _, _, kc, vc, ctx = cases.oracle_decode(8, pos)
    import ctypes as C
    scores = np.empty(pos + 1, dtype=np.float32)
    for qh in (0, 6, 7, 13):
        cuts = [0, 17, 64, 65, 250, pos + 1]
        ms, ls, os_ = [], [], []
        for a, b in zip(cuts[:-1], cuts[1:]):
            m, l = C.c_float(), C.c_float()
            o = np.empty(64, dtype=np.float32)
            O.lib().tgo_partial_head(q, kc.reshape(-1), vc.reshape(-1), qh, 14, 2,
                                     64, a, b, C.byref(m), C.byref(l), o, scores)
            ms.append(m.value)
            ls.append(l.value)
            os_.append(o)
        out = np.empty(64, dtype=np.float32)
        O.lib().tgo_merge_partials(len(ms), np.array(ms, np.float32),
                                   np.array(ls, np.float32),
                                   np.ascontiguousarray(np.stack(os_)), 64, out)
        np.testing.assert_allclose(out, ctx[qh * 64:(qh + 1) * 64], atol=2e-6)
