"""Parity of the tcgen05 grouped-GEMM prefill (fmcuda_moe_prefill) with the oracle.

The prefill path computes the reference's per-token expert loop
(src/engine.cpp:1711-1811) for a whole batch with fp16 tensor-core operands
(weights dequantised from their Q8_0 / Q4_K bytes to within one fp16 rounding,
activations in fp16) and f32 accumulation.  Bars:
  * router ids and weights: bit-exact (the same router kernel as decode);
  * y: max |y - y_ref| <= 2e-3 * max |y_ref| against the double-accumulated
    oracle (fp16 operands; the measured error is ~1e-4).
Shapes cover ragged groups (empty experts, experts with several 128-token
tiles, partial last tiles), a K that ends in half a 256-value chunk (Q8_0,
8-byte-aligned rows), the shared expert with and without its gate scalar, and
the DeepSeek- and Qwen3-shaped layers (oracle on sampled tokens).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.oracle import TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, bf16_round

pytestmark = pytest.mark.gpu
TOL = 2e-3


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def zipf_logits(rng, T, E, s=1.1):
    """Gumbel-top-k on log p_e (Zipf(s), ranks permuted): skewed, ragged groups."""
    p = 1.0 / np.arange(1, E + 1) ** s
    logp = np.log(p / p.sum())[rng.permutation(E)]
    return (logp[None, :] + rng.gumbel(size=(T, E))).astype(np.float32)


def host_experts(oracle, rng, E, d, ffn, t):
    slots = []
    for _ in range(E):
        parts = [oracle.quantize(t, rng.normal(0, 0.02, size=n).astype(np.float32))
                 for n in (ffn * d, ffn * d, d * ffn)]
        slots.append(np.concatenate(parts))
    return slots


def device_experts(cuda, E, d, ffn, t, seed):
    return [torch.cat([cuda.synth_weights(t, ffn, d, seed * 1000 + 3 * e),
                       cuda.synth_weights(t, ffn, d, seed * 1000 + 3 * e + 1),
                       cuda.synth_weights(t, d, ffn, seed * 1000 + 3 * e + 2)]) for e in range(E)]


def run_and_check(cuda, oracle, x, logits, slots_host, slots_dev, k, d, ffn, t, sample=None, shared=None,
                  shared_host=None, gate_scalar=None):
    y, ids, w = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), slots_dev, top_k=k, ffn=ffn, gate_type=t, shared=shared,
                                 return_routing=True)
    torch.cuda.synchronize()
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    assert rc == 0
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w_o))
    sel = np.arange(x.shape[0]) if sample is None else sample
    y_o = oracle.moe_block(x[sel], ids_o[sel], w_o[sel], slots_host, d, ffn, t)
    if shared_host is not None:
        sh_slot, sh_ffn, sh_t = shared_host
        ones = np.ones((len(sel), 1), dtype=np.float32)
        if gate_scalar is not None:
            ones = gate_scalar[sel].reshape(-1, 1).astype(np.float32)
        y_o = y_o + oracle.moe_block(x[sel], np.zeros((len(sel), 1), np.uint32), ones, [sh_slot], d, sh_ffn, sh_t)
    err = rel_err(y.cpu().numpy()[sel], y_o)
    assert err < TOL, err
    return err


@pytest.mark.parametrize("t", [TYPE_Q8_0, TYPE_Q4_K])
@pytest.mark.parametrize("T", [1, 37, 300])
def test_prefill_small_vs_oracle(cuda, oracle, t, T):
    rng = np.random.default_rng(100 + T + t)
    E, k, d, ffn = 8, 2, 256, 256
    slots = host_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    y, ids, w = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                                 gate_type=t, return_routing=True)
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    assert np.array_equal(bits(w.cpu().numpy()), bits(w_o))
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("T", [37, 300])
def test_prefill_q6_k_vs_oracle(cuda, oracle, T):
    """Q6_K throughout: 210-byte blocks, rows of 210 (gate/up) and 420 (down)
    bytes, so no block start is 4-byte aligned in general."""
    rng = np.random.default_rng(500 + T)
    E, k, d, ffn, t = 8, 2, 256, 512, TYPE_Q6_K
    slots = host_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    y = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn, gate_type=t)
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


def test_prefill_mixed_record(cuda, oracle):
    """Q4_K gate/up with a Q6_K down projection (the usual Q4_K_M mix), down rows
    of 1260 bytes; prefill and decode paths both against the oracle."""
    rng = np.random.default_rng(77)
    E, k, d, ffn, T = 8, 2, 512, 1536, 300
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
    y = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), dslots, top_k=k, ffn=ffn, gate_type=TYPE_Q4_K,
                         down_type=TYPE_Q6_K)
    assert cuda.device_status() == 0
    assert rel_err(y.cpu().numpy(), y_o) < TOL
    y_dec = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), dslots, top_k=k, ffn=ffn, gate_type=TYPE_Q4_K,
                           down_type=TYPE_Q6_K)
    assert rel_err(y_dec.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("t,big,xs", [(TYPE_Q8_0, 1.0, 1.0), (TYPE_Q4_K, 2000.0, 1e-3)])
def test_prefill_large_block_scales(cuda, oracle, t, big, xs):
    """Experts whose block scales are too large for the converters' subnormal
    fast path (Q8_0 d >= 2^-8, Q4_K d >= 4) take the generic path; both kinds
    of block sit in one launch and must agree with the oracle.  x is scaled so
    that the activations stay inside fp16 range."""
    rng = np.random.default_rng(31 + t)
    E, k, d, ffn, T = 4, 2, 256, 256, 64
    slots = []
    for e in range(E):
        std = big if e % 2 else 0.02
        slots.append(np.concatenate([oracle.quantize(t, rng.normal(0, std, size=n).astype(np.float32))
                                     for n in (ffn * d, ffn * d, d * ffn)]))
    x = bf16_round(rng.normal(0, xs, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    y, ids, w = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                                 gate_type=t, return_routing=True)
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    big_rows = np.isin(ids_o, [1, 3]).any(axis=1)
    assert big_rows.any() and (~big_rows).any()
    assert rel_err(y.cpu().numpy(), y_o) < TOL
    # the decode path reads the same records
    y_dec = cuda.moe_block(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                           gate_type=t)
    assert rel_err(y_dec.cpu().numpy(), y_o) < TOL


@pytest.mark.parametrize("xdt", ["bf16", "f32"])
def test_prefill_ragged_groups_half_chunk(cuda, oracle, xdt):
    # Zipf routing: empty experts, experts with 3+ token tiles; down K = 384
    # ends in half a 256-value chunk and its Q8_0 rows are 8-byte aligned.
    rng = np.random.default_rng(7)
    E, k, d, ffn, T, t = 16, 4, 256, 384, 700, TYPE_Q8_0
    slots = host_experts(oracle, rng, E, d, ffn, t)
    x = rng.normal(0, 1, size=(T, d)).astype(np.float32)
    if xdt == "bf16":
        x = bf16_round(x)
    logits = zipf_logits(rng, T, E)
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    counts = np.bincount(ids_o.ravel(), minlength=E)
    assert counts.max() > 256 and (counts % 128 != 0).any()
    xt = dev(x, torch.bfloat16) if xdt == "bf16" else dev(x)
    y = cuda.moe_prefill(xt, dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn, gate_type=t)
    assert cuda.device_status() == 0
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


def test_prefill_empty_experts(cuda, oracle):
    rng = np.random.default_rng(3)
    E, k, d, ffn, T, t = 8, 2, 256, 256, 50, TYPE_Q4_K
    slots = host_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = np.full((T, E), -5.0, dtype=np.float32)
    logits[:, 2] = 3.0
    logits[:, 5] = 2.0 + rng.normal(0, 0.1, size=T).astype(np.float32)
    dslots = [dev(s) for s in slots]
    dslots[0] = None  # never routed: a missing slot is fine when no token needs it
    y = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), dslots, top_k=k, ffn=ffn, gate_type=t)
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


def test_prefill_agrees_with_decode_path(cuda, oracle):
    rng = np.random.default_rng(11)
    E, k, d, ffn, T, t = 8, 2, 512, 768, 64, TYPE_Q4_K
    slots = [dev(s) for s in host_experts(oracle, rng, E, d, ffn, t)]
    x = dev(bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32)), torch.bfloat16)
    logits = dev(rng.normal(0, 1, size=(T, E)).astype(np.float32))
    y_p = cuda.moe_prefill(x, logits, slots, top_k=k, ffn=ffn, gate_type=t).cpu().numpy()
    y_d = cuda.moe_block(x, logits, slots, top_k=k, ffn=ffn, gate_type=t).cpu().numpy()
    assert cuda.device_status() == 0
    assert rel_err(y_p, y_d) < TOL


@pytest.mark.parametrize("gated", [False, True])
def test_prefill_shared_expert(cuda, oracle, gated):
    rng = np.random.default_rng(21 + gated)
    E, k, d, ffn, T, t, sh_ffn = 8, 2, 256, 256, 200, TYPE_Q8_0, 512
    slots = host_experts(oracle, rng, E, d, ffn, t)
    sh_slot = host_experts(oracle, rng, 1, d, sh_ffn, t)[0]
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    gs = (1.0 / (1.0 + np.exp(-rng.normal(0, 1, size=T)))).astype(np.float32) if gated else None
    gs_dev = dev(gs) if gated else None
    sh_dev = dev(sh_slot)
    shared = cuda.shared_expert_args(sh_dev, d_model=d, ffn=sh_ffn, gate_type=t, gate_scalar=gs_dev)
    y = cuda.moe_prefill(dev(x, torch.bfloat16), dev(logits), [dev(s) for s in slots], top_k=k, ffn=ffn,
                         gate_type=t, shared=shared)
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route(logits, k)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    g = gs.reshape(-1, 1) if gated else np.ones((T, 1), np.float32)
    y_o = y_o + oracle.moe_block(x, np.zeros((T, 1), np.uint32), g, [sh_slot], d, sh_ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL


def test_prefill_missing_expert_flags(cuda, oracle):
    rng = np.random.default_rng(5)
    E, k, d, ffn, t = 4, 2, 256, 256, TYPE_Q4_K
    slots = [dev(s) for s in host_experts(oracle, rng, E, d, ffn, t)]
    x = torch.randn(40, d, device="cuda")
    logits = torch.zeros(40, E, device="cuda")
    logits[:, 3] = 5.0
    slots[3] = None
    cuda.moe_prefill(x, logits, slots, top_k=k, ffn=ffn, gate_type=t)
    torch.cuda.synchronize()
    assert cuda.device_status(clear=True) == 18  # EXPERT_EXECUTION_MISMATCH


def test_prefill_rejects_unsupported(cuda):
    x = torch.randn(4, 256, device="cuda")
    logits = torch.randn(4, 4, device="cuda")
    slots = [torch.zeros(1 << 20, dtype=torch.uint8, device="cuda") for _ in range(4)]
    with pytest.raises(Exception, match="SHAPE_MISMATCH|multiple of"):
        cuda.moe_prefill(x, logits, slots, top_k=2, ffn=192, gate_type=TYPE_Q8_0)
    with pytest.raises(Exception, match="UNSUPPORTED|Q8_0 or Q4_K"):
        cuda.moe_prefill(x, logits, slots, top_k=2, ffn=256, gate_type=TYPE_F32)


def test_prefill_deepseek_shape(cuda, oracle):
    # d 2048, 64 routed experts ffn 1408 top-6 + 2 shared experts (one FFN of
    # width 2816), Q8_0; Zipf-skewed routing; oracle on sampled tokens.
    rng = np.random.default_rng(2024)
    E, k, d, ffn, T, t, sh_ffn = 64, 6, 2048, 1408, 1024, TYPE_Q8_0, 2816
    slots_dev = device_experts(cuda, E, d, ffn, t, seed=1)
    sh_dev = device_experts(cuda, 1, d, sh_ffn, t, seed=2)[0]
    slots_host = [s.cpu().numpy() for s in slots_dev]
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = zipf_logits(rng, T, E)
    shared = cuda.shared_expert_args(sh_dev, d_model=d, ffn=sh_ffn, gate_type=t)
    sample = np.sort(rng.choice(T, size=12, replace=False))
    err = run_and_check(cuda, oracle, x, logits, slots_host, slots_dev, k, d, ffn, t, sample=sample,
                        shared=shared, shared_host=(sh_dev.cpu().numpy(), sh_ffn, t))
    assert err < TOL


def test_prefill_qwen3_shape(cuda, oracle):
    # d 4096, 128 experts ffn 1536 top-8, Q4_K, uniform-random router logits.
    rng = np.random.default_rng(3030)
    E, k, d, ffn, T, t = 128, 8, 4096, 1536, 512, TYPE_Q4_K
    slots_dev = device_experts(cuda, E, d, ffn, t, seed=3)
    slots_host = [s.cpu().numpy() for s in slots_dev]
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.uniform(-1, 1, size=(T, E)).astype(np.float32)
    sample = np.sort(rng.choice(T, size=6, replace=False))
    run_and_check(cuda, oracle, x, logits, slots_host, slots_dev, k, d, ffn, t, sample=sample)


def test_prefill_router_variant(cuda, oracle):
    # DeepSeek-V3-style routing through the prefill block: sigmoid gating, a
    # selection bias and group-limited routing (8 groups, 4 kept)
    rng = np.random.default_rng(77)
    E, k, d, ffn, T, t = 64, 6, 256, 256, 300, TYPE_Q8_0
    slots = host_experts(oracle, rng, E, d, ffn, t)
    x = bf16_round(rng.normal(0, 1, size=(T, d)).astype(np.float32))
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    sb = rng.normal(0, 0.2, size=E).astype(np.float32)
    sbd = dev(sb)
    cfg = cuda.router_config(gating=1, selection_bias=sbd, groups=8, groups_used=4, scale=2.5)
    dslots = [dev(s) for s in slots]  # the slot table holds raw pointers: keep the tensors alive
    table = cuda.slot_table(dslots, "cuda")
    xt, lt = dev(x, torch.bfloat16), dev(logits)
    gb = cuda.row_bytes(t, d) * ffn
    y = torch.empty(T, d, dtype=torch.float32, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    a = cuda.moe_args(xt, lt, table, experts=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                      up_offset=gb, down_offset=2 * gb, y=y, ids_out=ids, router=cfg)
    need = cuda.moe_prefill_workspace_bytes(T, E, k, d, ffn)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    import ctypes as C
    from freemoe_b200._lib import check, load
    check(load().fmcuda_moe_prefill(C.byref(a), None, C.c_void_p(ws.data_ptr()), need, None))
    torch.cuda.synchronize()
    assert cuda.device_status() == 0
    rc, ids_o, w_o, _ = oracle.route_ex(logits, k, gating=1, selection_bias=sb, groups=8, groups_used=4, scale=2.5)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ids_o)
    y_o = oracle.moe_block(x, ids_o, w_o, slots, d, ffn, t)
    assert rel_err(y.cpu().numpy(), y_o) < TOL
