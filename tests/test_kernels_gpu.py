"""Parity of the sm_100a kernels with the CPU oracle, through the C ABI.

Bars (stated per dtype):
  * dequantisation, router ids / weights / probabilities, grouping: bit-exact;
  * F32 matvec in FM_ORDER_SCALAR / FM_ORDER_AVX2: bit-exact;
  * quantised GEMV and the MoE block (f32 accumulation on tensor cores, fp16
    operands that represent the codes and the activations exactly):
    max |y - y_ref| <= 1e-3 * max |y_ref| against the double-accumulated
    reference; the measured error is ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.oracle import TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, bf16_round

pytestmark = pytest.mark.gpu
TOL = 1e-3


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


# ---------------------------------------------------------------- K1 dequant

@pytest.mark.parametrize("name,t", [("q8_0", TYPE_Q8_0), ("q4_k", TYPE_Q4_K), ("q6_k", TYPE_Q6_K)])
def test_dequant_golden_bitexact(cuda, golden, name, t):
    src, exp = golden[f"dequant_{name}_src"], golden[f"dequant_{name}_out"]
    got = cuda.dequantize_tensor_region(t, dev(src), exp.size).cpu().numpy()
    assert np.array_equal(bits(got), bits(exp))


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K])
def test_dequant_full_matrix_bitexact(cuda, oracle, t):
    # a Mixtral-shaped gate matrix [14336 x 4096], synthesised on the device
    rows, cols = 14336, 4096
    w = cuda.synth_weights(t, rows, cols, seed=7)
    got = cuda.dequantize_tensor_region(t, w, rows * cols).cpu().numpy()
    ref = oracle.dequant(t, w.cpu().numpy(), rows * cols)
    assert np.array_equal(bits(got), bits(ref))


def test_dequant_f32_and_errors(cuda):
    x = torch.randn(1000, device="cuda")
    assert torch.equal(cuda.dequantize_tensor_region(TYPE_F32, x, 1000), x)
    with pytest.raises(Exception) as ei:
        cuda.dequantize_tensor_region(TYPE_Q4_K, x, 255)
    assert "SHAPE_MISMATCH" in str(ei.value)


# ---------------------------------------------------------------- K2 GEMV

@pytest.mark.parametrize("name,t", [("q8_0", TYPE_Q8_0), ("q4_k", TYPE_Q4_K), ("q6_k", TYPE_Q6_K)])
def test_gemv_golden(cuda, golden, name, t):
    o, i, T = (int(v) for v in golden["gemv_shape"])
    x = golden[f"gemv_{name}_x"]
    y = cuda.gemv_quant(t, dev(golden[f"gemv_{name}_w"]), dev(x, torch.bfloat16), o, i).cpu().numpy()
    assert rel_err(y, golden[f"gemv_{name}_y_auto"]) < TOL


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K])
@pytest.mark.parametrize("tokens", [1, 2, 3, 8, 9, 17])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_gemv_vs_oracle(cuda, oracle, t, tokens, xdt):
    rng = np.random.default_rng(100 + tokens + t)
    out_dim, in_dim = 200, 1024  # 200 rows: partial 16/32-row tiles
    w = oracle.quantize(t, rng.normal(0, 0.02, size=out_dim * in_dim).astype(np.float32))
    x = rng.normal(0, 1, size=(tokens, in_dim)).astype(np.float32)
    if xdt == "bf16":
        x = bf16_round(x)
        xt = dev(x, torch.bfloat16)
    else:
        xt = dev(x)
    y = cuda.gemv_quant(t, dev(w), xt, out_dim, in_dim).cpu().numpy()
    ref = oracle.gemv_f64(t, w, x, out_dim, in_dim)
    err = rel_err(y, ref)
    assert err < TOL, err
    assert err < 1e-4  # what the design delivers; the stated bar is TOL


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K])
def test_gemv_mixtral_shapes(cuda, oracle, t):
    # gate [14336 x 4096] and down [4096 x 14336] at T = 1 and T = 8 (bf16 x)
    for out_dim, in_dim in ((14336, 4096), (4096, 14336)):
        w = cuda.synth_weights(t, out_dim, in_dim, seed=out_dim)
        wn = w.cpu().numpy()
        for tokens in (1, 8):
            x = bf16_round(np.random.default_rng(tokens).normal(0, 1, size=(tokens, in_dim)).astype(np.float32))
            y = cuda.gemv_quant(t, w, dev(x, torch.bfloat16), out_dim, in_dim).cpu().numpy()
            rows = np.arange(0, out_dim, 37)
            ref = oracle.gemv_f64(t, np.ascontiguousarray(
                wn.reshape(out_dim, -1)[rows]).ravel(), x, rows.size, in_dim)
            assert rel_err(y[:, rows], ref) < TOL


def test_gemv_linearity(cuda):
    # size-independent property at the full Q4_K shape: W(a + b) = Wa + Wb
    w = cuda.synth_weights(TYPE_Q4_K, 14336, 4096, seed=1)
    a = torch.randn(4, 4096, device="cuda")
    b = torch.randn(4, 4096, device="cuda")
    ya = cuda.gemv_quant(TYPE_Q4_K, w, a, 14336, 4096)
    yb = cuda.gemv_quant(TYPE_Q4_K, w, b, 14336, 4096)
    yab = cuda.gemv_quant(TYPE_Q4_K, w, a + b, 14336, 4096)
    scale = (ya.abs().max() + yb.abs().max()).item()
    assert ((yab - ya - yb).abs().max().item()) / scale < 1e-5


def test_gemv_f32_weights(cuda):
    w = torch.randn(300, 640, device="cuda")
    x = torch.randn(5, 640, device="cuda")
    y = cuda.gemv_quant(TYPE_F32, w.reshape(-1).view(torch.uint8), x, 300, 640)
    ref = (x.double() @ w.double().T)
    assert ((y.double() - ref).abs().max() / ref.abs().max()).item() < 1e-5


def test_matvec_f32_orders_bitexact(cuda, golden, oracle):
    from freemoe_b200 import ORDER_AVX2, ORDER_SCALAR

    w, x = golden["f32_w"], golden["f32_x"]
    o, i = w.shape
    ys = cuda.matvec_f32(dev(w), dev(x), o, i, ORDER_SCALAR).cpu().numpy()
    ya = cuda.matvec_f32(dev(w), dev(x), o, i, ORDER_AVX2).cpu().numpy()
    assert np.array_equal(bits(ys), bits(golden["f32_y_scalar"]))
    assert np.array_equal(bits(ya), bits(golden["f32_y_auto"]))
    rng = np.random.default_rng(5)
    for o, i in ((64, 64), (128, 64), (258, 64), (33, 200), (17, 24), (5, 7)):
        w = rng.normal(size=(o, i)).astype(np.float32)
        x = rng.normal(size=i).astype(np.float32)
        ys = cuda.matvec_f32(dev(w), dev(x), o, i, ORDER_SCALAR).cpu().numpy()
        ya = cuda.matvec_f32(dev(w), dev(x), o, i, ORDER_AVX2).cpu().numpy()
        assert np.array_equal(bits(ys), bits(oracle.gemv_f32(w, x, o, i, "scalar")))
        assert np.array_equal(bits(ya), bits(oracle.gemv_f32(w, x, o, i, "avx2")))


# ---------------------------------------------------------------- K4 router

@pytest.mark.parametrize("E,k", [(4, 2), (8, 2), (64, 6), (128, 8)])
def test_route_golden_bitexact(cuda, golden, E, k):
    pre = f"route_E{E}_k{k}_"
    ids, w, probs = cuda.route(dev(golden[pre + "logits"]), k, want_probs=True)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), golden[pre + "ids"])
    assert np.array_equal(bits(w.cpu().numpy()), bits(golden[pre + "weights"]))
    assert np.array_equal(bits(probs.cpu().numpy()), bits(golden[pre + "probs"]))


@pytest.mark.parametrize("E,k,T", [(4, 2, 1), (8, 2, 64), (64, 6, 4096), (128, 8, 8192), (1024, 32, 33), (3, 3, 5), (1, 1, 2)])
def test_route_vs_oracle(cuda, oracle, E, k, T):
    rng = np.random.default_rng(E * 31 + k)
    lg = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    lg[:: max(1, T // 7)] = np.round(lg[:: max(1, T // 7)], 1)  # ties
    rc, ids_o, w_o, p_o = oracle.route(lg, k)
    assert rc == 0
    ids, w, probs = cuda.route(dev(lg), k, want_probs=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w_o))
    assert np.array_equal(bits(probs.cpu().numpy()), bits(p_o))


def test_route_non_finite_sets_device_status(cuda):
    lg = torch.zeros(3, 8, device="cuda")
    lg[1, 4] = float("nan")
    cuda.route(lg, 2)
    assert cuda.device_status(clear=True) == 28  # INTERNAL_ERROR
    assert cuda.device_status() == 0
    with pytest.raises(Exception) as ei:
        cuda.route(torch.zeros(1, 4, device="cuda"), 5)
    assert "INVALID_ARGUMENT" in str(ei.value)
    ids, w = cuda.route(torch.zeros(0, 8, device="cuda"), 2)  # empty batch
    assert ids.numel() == 0


@pytest.mark.parametrize("E,k,T", [(4, 2, 1), (8, 2, 64), (64, 6, 4096), (128, 8, 8192), (1024, 4, 100)])
def test_group_vs_oracle(cuda, oracle, E, k, T):
    rng = np.random.default_rng(T)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    c_o, o_o, p_o, s_o = oracle.group(ids, E)
    counts, offsets, pairs, slot_of = cuda.group_by_expert(dev(ids.astype(np.int32)), E)
    assert np.array_equal(counts.cpu().numpy().astype(np.uint32), c_o)
    assert np.array_equal(offsets.cpu().numpy().astype(np.uint32), o_o)
    assert np.array_equal(pairs.cpu().numpy().astype(np.uint32), p_o)
    assert np.array_equal(slot_of.cpu().numpy().astype(np.uint32), s_o)


@pytest.mark.parametrize("gating,groups,used,biased,eps_add,E,k",
                         [(1, 8, 4, True, False, 256, 8), (1, 1, 1, True, False, 64, 6), (2, 1, 1, False, True, 128, 8),
                          (3, 1, 1, True, False, 32, 4), (0, 4, 2, True, False, 64, 6), (0, 1, 1, True, True, 1024, 8),
                          (1, 32, 3, False, False, 1024, 32)])
def test_route_ex_vs_oracle(cuda, oracle, gating, groups, used, biased, eps_add, E, k):
    # router variants of src/engine.cpp:1603-1702: ids, weights and probabilities bit-exact
    rng = np.random.default_rng(E + 7 * gating + groups)
    T = 2000
    lg = rng.normal(0, 1.5, size=(T, E)).astype(np.float32)
    lb = rng.normal(0, 0.3, size=E).astype(np.float32) if biased else None
    sb = rng.normal(0, 0.1, size=E).astype(np.float32) if biased else None
    rc, ids_o, w_o, p_o = oracle.route_ex(lg, k, gating=gating, logit_bias=lb, selection_bias=sb, groups=groups,
                                          groups_used=used, epsilon_additive=eps_add)
    assert rc == 0
    lbd = dev(lb) if biased else None
    sbd = dev(sb) if biased else None
    cfg = cuda.router_config(gating=gating, logit_bias=lbd, selection_bias=sbd, groups=groups, groups_used=used,
                             epsilon_additive=eps_add)
    ids, w, p = cuda.route_ex(dev(lg), k, cfg, want_probs=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w_o))
    assert np.array_equal(bits(p.cpu().numpy()), bits(p_o))


def test_route_ex_nan_selection_flags(cuda):
    lg = torch.randn(4, 16, device="cuda")
    sb = torch.zeros(16, device="cuda")
    sb[3] = float("nan")
    cfg = cuda.router_config(gating=1, selection_bias=sb)
    cuda.route_ex(lg, 2, cfg)
    assert cuda.device_status(clear=True) == 28  # INTERNAL_ERROR (Engine::topk's check)


@pytest.mark.parametrize("E,k,T", [(8, 2, 1), (64, 6, 4096), (128, 8, 8192), (1024, 8, 3000), (7, 3, 1000)])
def test_group_batched_vs_oracle(cuda, oracle, E, k, T):
    # the many-warp grouping used by prefill: bit-identical to the oracle
    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    c_o, o_o, p_o, s_o = oracle.group(ids, E)
    counts, offsets, pairs, slot_of = cuda.group_by_expert_batched(dev(ids.astype(np.int32)), E)
    assert np.array_equal(counts.cpu().numpy().astype(np.uint32), c_o)
    assert np.array_equal(offsets.cpu().numpy().astype(np.uint32), o_o)
    assert np.array_equal(pairs.cpu().numpy().astype(np.uint32), p_o)
    assert np.array_equal(slot_of.cpu().numpy().astype(np.uint32), s_o)


@pytest.mark.parametrize("out_dim,in_dim,t", [(1280, 1280, TYPE_Q8_0), (1280, 1280, TYPE_Q4_K),
                                               (1792, 1280, TYPE_Q4_K), (1280, 1792, TYPE_Q4_K),
                                               (32000, 1280, TYPE_Q4_K)])
def test_gemv_reference_bench_shapes(cuda, oracle, out_dim, in_dim, t):
    # the quantised GEMV shapes of the reference's kernel benchmark (src/main.cpp:631-637)
    w = cuda.synth_weights(t, out_dim, in_dim, seed=out_dim + in_dim)
    x = torch.randn(1, in_dim, device="cuda")
    y = cuda.gemv_quant(t, w, x, out_dim, in_dim).cpu().numpy().ravel()
    rows = np.arange(0, out_dim, max(1, out_dim // 512))
    rb = w.numel() // out_dim
    wr = w.cpu().numpy().reshape(out_dim, rb)[rows].ravel()
    ref = oracle.gemv_f64(t, wr, x.cpu().numpy().ravel(), len(rows), in_dim)[0]
    assert rel_err(y[rows], ref) < TOL


# ---------------------------------------------------------------- MoE block

def make_experts(oracle, rng, E, d, ffn, t):
    slots = []
    for _ in range(E):
        parts = [oracle.quantize(t, rng.normal(0, 0.02, size=n).astype(np.float32))
                 for n in (ffn * d, ffn * d, d * ffn)]
        slots.append(np.concatenate(parts))
    return slots


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K])
@pytest.mark.parametrize("T", [1, 4, 9, 33, 70])
@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_moe_block_vs_oracle(cuda, oracle, t, T, xdt):
    rng = np.random.default_rng(T * 7 + t)
    E, k, d, ffn = 8, 2, 512, 768
    slots = make_experts(oracle, rng, E, d, ffn, t)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    if xdt == "bf16":
        x = bf16_round(x)
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    xt = dev(x, torch.bfloat16) if xdt == "bf16" else dev(x)
    y, ids, w = cuda.moe_block(xt, dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=t, return_routing=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w_o))
    assert rel_err(y.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K])
def test_moe_block_non_finite_logit_token(cuda, oracle, t):
    """A token whose router logits hold a NaN gets no experts: INTERNAL_ERROR in
    the status word, its ids absent, its output row exactly zero (the combine
    of no terms), and every other token as the oracle computes it alone.  With
    bf16 activations and Q4_K this runs the fused router + grouping + image
    launch of the tcgen05 stage."""
    rng = np.random.default_rng(900 + t)
    E, k, d, ffn, T = 8, 2, 512, 768, 6
    slots = make_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    logits[2, 5] = np.nan
    y, ids, _ = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=t, return_routing=True)
    assert cuda.device_status(clear=True) == 28  # INTERNAL_ERROR
    y = y.cpu().numpy()
    assert np.all(ids.cpu().numpy().astype(np.uint32)[2] == 0xFFFFFFFF)
    assert np.all(bits(y[2]) == 0)
    valid = [0, 1, 3, 4, 5]
    rc, ids_o, w_o, _ = oracle.route(logits[valid], k)
    y_o = oracle.moe_block(x[valid], ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y[valid], y_o) < TOL


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K])
def test_moe_block_skewed_routing(cuda, oracle, t):
    # one expert takes every token (5 token tiles of the same rows), two take
    # none, the rest share the second choices
    rng = np.random.default_rng(500 + t)
    E, k, d, ffn, T = 8, 2, 512, 768, 40
    slots = make_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    logits[:, 2] += 8.0
    logits[:, [5, 6]] -= 8.0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    assert (ids_o[:, 0] == 2).all()
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    y, ids, w = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=t, return_routing=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("T", [64, 100])
def test_moe_block_tile_pairs(cuda, oracle, T):
    """At 16 or more routed pairs per expert the tcgen05 GEMVs convert each weight
    block once for two 8-token tiles: one expert with many tiles (an odd count
    among them), experts with a single tile (a pair without its second tile),
    an expert with none; checked norm-wise and element-wise."""
    rng = np.random.default_rng(1500 + T)
    E, k, d, ffn = 8, 2, 512, 768
    slots = make_experts(oracle, rng, E, d, ffn, TYPE_Q4_K)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    logits[:, 2] += 3.0
    logits[:, 5] -= 9.0
    logits[:, 6] -= 1.5
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    counts = np.bincount(ids_o.ravel(), minlength=E)
    assert counts[5] == 0 and ((counts + 7) // 8 % 2 == 1).any()
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, TYPE_Q4_K)
    y, ids, w = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=TYPE_Q4_K, return_routing=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    got = y.cpu().numpy()
    assert rel_err(got, y_o) < TOL
    big = np.abs(y_o) > 1e-2 * np.abs(y_o).max()
    assert float((np.abs(got - y_o)[big] / np.abs(y_o[big])).max()) < TOL
    y2 = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                        gate_type=TYPE_Q4_K)
    assert torch.equal(y2.cpu(), y.cpu())  # the stream-K counters were left at zero


@pytest.mark.parametrize("T", [3, 20])
def test_moe_block_wide_model_short_ffn(cuda, oracle, T):
    # 16 experts, d 2048, ffn 256: the down projection is a single 256-value K
    # step (the second warp of each tile has no items), 15 experts active at T=20
    rng = np.random.default_rng(700 + T)
    E, k, d, ffn = 16, 2, 2048, 256
    slots = make_experts(oracle, rng, E, d, ffn, TYPE_Q4_K)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, TYPE_Q4_K)
    y, ids, w = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=TYPE_Q4_K, return_routing=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("T", [1, 5, 40])
def test_moe_block_mixed_record(cuda, oracle, T):
    # mixed-type expert records: Q4_K gate/up with a Q6_K down projection
    rng = np.random.default_rng(900 + T)
    E, k, d, ffn = 8, 2, 512, 768
    slots = []
    for _ in range(E):
        parts = [oracle.quantize(TYPE_Q4_K, rng.normal(0, 0.02, size=ffn * d).astype(np.float32)),
                 oracle.quantize(TYPE_Q4_K, rng.normal(0, 0.02, size=ffn * d).astype(np.float32)),
                 oracle.quantize(TYPE_Q6_K, rng.normal(0, 0.02, size=d * ffn).astype(np.float32))]
        slots.append(np.concatenate(parts))
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, TYPE_Q4_K, TYPE_Q4_K, TYPE_Q6_K)
    dslots = [dev(s) for s in slots]
    y = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), dslots, top_k=k, ffn=ffn, gate_type=TYPE_Q4_K,
                       down_type=TYPE_Q6_K)
    assert cuda.device_status() == 0
    assert rel_err(y.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K])
@pytest.mark.parametrize("T,xdt", [(1, "bf16"), (9, "f32"), (37, "bf16"), (70, "f32")])
def test_moe_block_ragged_tiles_d1024(cuda, oracle, t, T, xdt):
    # the streamed GEMV on rows of four K steps: ragged token tiles, several
    # token tiles of one expert (expert 1 takes most tokens), an expert with
    # none; also checked element-wise where |y_ref| is not tiny
    rng = np.random.default_rng(1300 + T + t)
    E, k, d, ffn = 6, 2, 1024, 1024
    slots = make_experts(oracle, rng, E, d, ffn, t)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    if xdt == "bf16":
        x = bf16_round(x)
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    logits[:, 1] += 2.0
    logits[:, 4] -= 9.0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    xt = dev(x, torch.bfloat16) if xdt == "bf16" else dev(x)
    y, ids, w = cuda.moe_block(xt, dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                               gate_type=t, return_routing=True)
    assert cuda.device_status() == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    got = y.cpu().numpy()
    assert rel_err(got, y_o) < TOL
    big = np.abs(y_o) > 1e-2 * np.abs(y_o).max()
    assert float((np.abs(got - y_o)[big] / np.abs(y_o[big])).max()) < TOL


def test_moe_block_streamed_missing_expert_flags(cuda, oracle):
    rng = np.random.default_rng(3)
    E, k, d, ffn = 4, 2, 1024, 1024
    slots = make_experts(oracle, rng, E, d, ffn, TYPE_Q4_K)
    x = torch.randn(6, d, device="cuda")
    logits = torch.zeros(6, E, device="cuda")
    logits[:, 3] = 5.0  # every token routes to expert 3
    dslots = [dev(s) for s in slots]
    dslots[3] = None
    cuda.moe_block(x, logits, dslots, top_k=k, ffn=ffn, gate_type=TYPE_Q4_K)
    torch.cuda.synchronize()
    assert cuda.device_status(clear=True) == 18  # EXPERT_EXECUTION_MISMATCH


def test_moe_block_missing_expert_flags(cuda, oracle):
    rng = np.random.default_rng(1)
    E, k, d, ffn = 4, 2, 256, 256
    slots = make_experts(oracle, rng, E, d, ffn, TYPE_Q4_K)
    x = torch.randn(6, d, device="cuda")
    logits = torch.zeros(6, E, device="cuda")
    logits[:, 3] = 5.0  # every token routes to expert 3
    dslots = [dev(s) for s in slots]
    dslots[3] = None
    cuda.moe_block(x, logits, dslots, top_k=k, ffn=ffn, gate_type=TYPE_Q4_K)
    assert cuda.device_status(clear=True) == 18  # EXPERT_EXECUTION_MISMATCH


def test_misaligned_quantised_matrices_are_refused(cuda, oracle):
    """A Q4_K matrix whose first byte is not 16-byte aligned (the loads the
    kernels issue) is refused on the host with INVALID_ARGUMENT, not read."""
    import ctypes as C

    from freemoe_b200 import hotpath
    from freemoe_b200._lib import FmError, load

    rng = np.random.default_rng(2)
    E, k, d, ffn = 2, 1, 256, 256
    slots = make_experts(oracle, rng, E, d, ffn, TYPE_Q4_K)
    pad = [np.concatenate([s, np.zeros(16, np.uint8)]) for s in slots]
    dslots = [dev(s) for s in pad]
    table = hotpath.slot_table(dslots, torch.device("cuda"))
    x = torch.randn(3, d, device="cuda")
    logits = torch.randn(3, E, device="cuda")
    y = torch.empty(3, d, device="cuda")
    gb = ffn * (d // 256) * 144
    ws = torch.empty(hotpath.moe_workspace_bytes(3, E, k, d, ffn), dtype=torch.uint8, device="cuda")
    lib = load()
    for up, down in ((gb + 8, 2 * gb), (gb, 2 * gb + 2)):
        a = hotpath.moe_args(x, logits, table, experts=E, top_k=k, d_model=d, ffn=ffn, gate_type=TYPE_Q4_K,
                             up_type=TYPE_Q4_K, down_type=TYPE_Q4_K, up_offset=up, down_offset=down, y=y)
        rc = lib.fmcuda_moe_block(C.byref(a), C.c_void_p(ws.data_ptr()), ws.numel(), None)
        assert rc == 26, rc  # INVALID_ARGUMENT
    w = dev(np.concatenate([np.zeros(4, np.uint8), slots[0][:gb]]))
    with pytest.raises(FmError) as e:
        cuda.gemv_quant(TYPE_Q4_K, w[4:], x, out_dim=ffn, in_dim=d)
    assert e.value.code == 26
    torch.cuda.synchronize()
    assert cuda.device_status(clear=True) == 0
