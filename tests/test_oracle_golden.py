"""The CPU oracle pinned against the reference's golden vectors (no GPU).

quant_reference_hotpath.bin is the F32/Q8_0/Q4_K extract of the reference's
tests/fixtures/quant_reference.bin (checked there by test_quant_reference_decode,
tests/unit/tests.cpp:1244, at rel 1e-6); golden_vectors.npz holds outputs of the
reference's own code compiled from source (tests/golden/make_golden.py).
"""
from __future__ import annotations

import struct

import numpy as np
import pytest

from conftest import GOLDEN
from oracle.oracle import TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, Reference, reference_available


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def read_fmqr(path):
    data = path.read_bytes()
    assert data[:5] == b"FMQR1"
    (n,) = struct.unpack_from("<I", data, 8)
    pos, recs = 12, []
    while pos < len(data):
        t, bb, nf = struct.unpack_from("<III", data, pos)
        pos += 12
        raw = np.frombuffer(data, dtype=np.uint8, count=bb, offset=pos)
        pos += bb
        exp = np.frombuffer(data, dtype=np.float32, count=nf, offset=pos)
        pos += 4 * nf
        recs.append((t, bb, nf, raw, exp))
    assert len(recs) == n
    return recs


def test_quant_reference_records(oracle):
    recs = read_fmqr(GOLDEN / "quant_reference_hotpath.bin")
    assert sorted(r[0] for r in recs) == [TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K]
    geo = {TYPE_F32: (1, 4), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}
    for t, bb, nf, raw, exp in recs:
        assert geo[t] == (nf, bb)
        got = oracle.dequant(t, raw, nf)
        # the reference's own acceptance bound for this fixture
        np.testing.assert_allclose(got, exp, rtol=1e-6, atol=0)
        # and in fact bit-exact for these four decoders
        assert np.array_equal(bits(got), bits(exp)), f"type {t}"


@pytest.mark.parametrize("name,t,bs", [("q8_0", TYPE_Q8_0, 32), ("q4_k", TYPE_Q4_K, 256), ("q6_k", TYPE_Q6_K, 256)])
def test_dequant_golden(oracle, golden, name, t, bs):
    src = golden[f"dequant_{name}_src"]
    exp = golden[f"dequant_{name}_out"]
    got = oracle.dequant(t, src, exp.size)
    assert np.array_equal(bits(got), bits(exp))


@pytest.mark.parametrize("name,t", [("q8_0", TYPE_Q8_0), ("q4_k", TYPE_Q4_K), ("q6_k", TYPE_Q6_K)])
def test_gemv_fused_scalar_golden(oracle, golden, name, t):
    o, i, T = golden["gemv_shape"]
    y = oracle.gemv_fused_scalar(t, golden[f"gemv_{name}_w"], golden[f"gemv_{name}_x"], o, i)
    assert np.array_equal(bits(y), bits(golden[f"gemv_{name}_y_scalar"]))
    # the reference's AVX2 order agrees with the order-neutral double reference
    y64 = oracle.gemv_f64(t, golden[f"gemv_{name}_w"], golden[f"gemv_{name}_x"], o, i)
    err = np.max(np.abs(golden[f"gemv_{name}_y_auto"] - y64)) / np.max(np.abs(y64))
    assert err < 1e-6


def test_f32_orders_golden(oracle, golden):
    w, x = golden["f32_w"], golden["f32_x"]
    o, i = w.shape
    assert np.array_equal(bits(oracle.gemv_f32(w, x, o, i, "scalar")), bits(golden["f32_y_scalar"]))
    assert np.array_equal(bits(oracle.gemv_f32(w, x, o, i, "avx2")), bits(golden["f32_y_auto"]))


@pytest.mark.parametrize("E,k", [(4, 2), (8, 2), (64, 6), (128, 8)])
def test_route_golden(oracle, golden, E, k):
    pre = f"route_E{E}_k{k}_"
    rc, ids, w, probs = oracle.route(golden[pre + "logits"], k)
    assert rc == 0
    assert np.array_equal(ids, golden[pre + "ids"])
    assert np.array_equal(bits(w), bits(golden[pre + "weights"]))
    assert np.array_equal(bits(probs), bits(golden[pre + "probs"]))
    # all-equal logits select the lowest ids, in order
    assert list(ids[0]) == list(range(k))


def test_swiglu_golden(oracle, golden):
    got = oracle.swiglu(golden["swiglu_gate"], golden["swiglu_up"])
    assert np.array_equal(bits(got), bits(golden["swiglu_out"]))


def test_route_errors(oracle):
    lg = np.zeros((2, 4), dtype=np.float32)
    lg[1, 2] = np.nan
    assert oracle.route(lg, 2)[0] == 28  # INTERNAL_ERROR (non-finite value in softmax)
    lg[1, 2] = np.inf
    assert oracle.route(lg, 2)[0] == 28
    assert oracle.route(np.zeros((1, 4), np.float32), 5)[0] == 26  # INVALID_ARGUMENT (k > E)


def test_group_by_expert(oracle):
    ids = np.array([[2, 0], [0, 1], [2, 1], [3, 0]], dtype=np.uint32)
    counts, offsets, pairs, slot_of = oracle.group(ids, 5)
    assert list(counts) == [3, 2, 2, 1, 0]
    assert list(offsets) == [0, 3, 5, 7, 8, 8]
    # expert 0: pairs (t0,r1)=1, (t1,r0)=2, (t3,r1)=7 ; expert 1: 3, 5 ; expert 2: 0, 4 ; expert 3: 6
    assert list(pairs) == [1, 2, 7, 3, 5, 0, 4, 6]
    assert all(pairs[slot_of[p]] == p for p in range(8))


def test_encoders_roundtrip(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 0.02, size=4096).astype(np.float32)
    for t, tol in ((TYPE_Q8_0, 0.02 * 4 / 127), (TYPE_Q4_K, 0.02 * 8 / 15)):
        enc = oracle.quantize(t, x)
        dec = oracle.dequant(t, enc, x.size)
        assert np.max(np.abs(dec - x)) < tol


@pytest.mark.skipif(not reference_available(), reason="compiled reference shim not built here")
def test_oracle_matches_live_reference(oracle):
    ref = Reference()
    rng = np.random.default_rng(11)
    for t in (TYPE_Q8_0, TYPE_Q4_K):
        w = oracle.quantize(t, rng.normal(0, 0.02, size=64 * 1024).astype(np.float32))
        x = rng.normal(0, 1, size=1024).astype(np.float32)
        bs = 32 if t == TYPE_Q8_0 else 256
        assert np.array_equal(bits(oracle.dequant(t, w, 64 * 1024)), bits(ref.dequant(t, w, 64 * 1024)))
        ys = ref.gemv_quant(t, w, x, 64, 1024, scalar=True)
        assert np.array_equal(bits(oracle.gemv_fused_scalar(t, w, x, 64, 1024)[0]), bits(ys))
        assert bs
    lg = rng.normal(size=(256, 64)).astype(np.float32)
    a, b = oracle.route(lg, 6), ref.route(lg, 6)
    assert a[0] == b[0] == 0 and np.array_equal(a[1], b[1]) and np.array_equal(bits(a[2]), bits(b[2]))


def test_route_ex_default_is_the_native_router(oracle):
    # the variant router with its defaults reduces to the pinned native router
    rng = np.random.default_rng(41)
    lg = rng.normal(0, 2, size=(300, 64)).astype(np.float32)
    rc0, ids0, w0, p0 = oracle.route(lg, 6)
    rc1, ids1, w1, p1 = oracle.route_ex(lg, 6)
    assert rc0 == rc1 == 0
    assert np.array_equal(ids0, ids1)
    assert np.array_equal(w0.view(np.uint32), w1.view(np.uint32))
    assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32))


def _route_ex_numpy(lg, k, gating, lbias, sbias, groups, used, eps_add, eps=6.103515625e-5, scale=1.0):
    """An independent restatement of src/engine.cpp:1603-1702 in numpy."""
    T, E = lg.shape
    ids = np.zeros((T, k), np.uint32)
    ws = np.zeros((T, k), np.float32)
    for t in range(T):
        s = lg[t].astype(np.float32)
        if lbias is not None:
            s = (s + lbias).astype(np.float32)
        if gating == 1:
            p = (1.0 / (1.0 + np.exp(-s.astype(np.float64)))).astype(np.float32)
        elif gating == 2:
            p = np.sqrt(np.log1p(np.exp(s.astype(np.float64)))).astype(np.float32)
        elif gating == 3:
            p = s.copy()
        else:
            ex = np.exp(s.astype(np.float64) - np.float64(s.max()))
            p = (ex / ex.sum()).astype(np.float32)
        sel = p.copy() if sbias is None else (p + sbias).astype(np.float32)
        if groups > 1:
            per = E // groups
            gs = [np.float32(np.float32(0) + np.sort(sel[g * per:(g + 1) * per])[::-1][0]) +
                  np.float32(np.sort(sel[g * per:(g + 1) * per])[::-1][1]) for g in range(groups)]
            order = sorted(range(groups), key=lambda g: (-gs[g], g))
            for g in order[used:]:
                sel[g * per:(g + 1) * per] = -np.inf
        pick = sorted(range(E), key=lambda e: (-sel[e], e))[:k]
        w = p[pick].astype(np.float32)
        total = np.float32(0)
        for v in w:
            total = np.float32(total + v)
        if gating == 3:
            ex = np.exp(w.astype(np.float64) - np.float64(w.max()))
            w = (ex / ex.sum()).astype(np.float32)
        den = np.float64(total) + eps if eps_add else max(np.float64(total), eps)
        w = (w.astype(np.float64) / den).astype(np.float32)
        w = (w.astype(np.float64) * scale).astype(np.float32)
        ids[t], ws[t] = pick, w
    return ids, ws


@pytest.mark.parametrize("gating,groups,used,biased,eps_add", [(1, 8, 4, True, False), (2, 1, 1, False, True),
                                                              (3, 1, 1, True, False), (0, 4, 2, True, False)])
def test_route_ex_matches_numpy_restatement(oracle, gating, groups, used, biased, eps_add):
    rng = np.random.default_rng(gating * 10 + groups)
    T, E, k = 64, 64, 6
    lg = rng.normal(0, 1.5, size=(T, E)).astype(np.float32)
    lb = rng.normal(0, 0.3, size=E).astype(np.float32) if biased else None
    sb = rng.normal(0, 0.1, size=E).astype(np.float32) if biased else None
    rc, ids, w, _ = oracle.route_ex(lg, k, gating=gating, logit_bias=lb, selection_bias=sb, groups=groups,
                                    groups_used=used, epsilon_additive=eps_add)
    assert rc == 0
    ids_n, w_n = _route_ex_numpy(lg, k, gating, lb, sb, groups, used, eps_add)
    assert np.array_equal(ids, ids_n)
    assert np.allclose(w, w_n, rtol=2e-7, atol=0)
