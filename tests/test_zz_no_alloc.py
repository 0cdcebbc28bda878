"""fmcuda_moe_block_noalloc: the MoE block for callers that cannot allocate.

Some hosts cannot call cudaMalloc once decoding runs -- all of their HBM is
already committed to expert slots, or the device allocator belongs to the host
framework -- so the library offers a variant of the MoE block whose scratch is
a fixed array inside the library image.  These tests call it through the C ABI
and compare it with fmcuda_moe_block (which uses a caller workspace) on two
calls in a row with different inputs, so a result that depended on what the
previous call left in the shared scratch would show.  Collected last on
purpose (file name), and independent of the other tests' state.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from freemoe_b200._lib import MOE_NOALLOC_SCRATCH_BYTES, MoeArgs
from oracle.oracle import TYPE_Q4_K, TYPE_Q8_0, bf16_round

TOL = 1e-3  # the MoE-block bar of the other GPU tests


def make_block(oracle, seed, t, E=8, k=2, d=512, ffn=768, T=5):
    rng = np.random.default_rng(seed)
    slots = [torch.from_numpy(np.concatenate([oracle.quantize(t, rng.normal(0, 0.02, n).astype(np.float32))
                                              for n in (ffn * d, ffn * d, d * ffn)])).cuda() for _ in range(E)]
    x = torch.from_numpy(bf16_round(rng.normal(0, 1, (T, d)).astype(np.float32))).cuda().to(torch.bfloat16)
    logits = torch.from_numpy(rng.normal(0, 1, (T, E)).astype(np.float32)).cuda()
    return slots, x, logits, dict(E=E, k=k, d=d, ffn=ffn, T=T)


def args_for(cuda, slots, x, logits, cfg, t, y):
    gate_bytes = cuda.row_bytes(t, cfg["d"]) * cfg["ffn"]
    table = cuda.slot_table(slots, x.device)
    a = cuda.moe_args(x, logits, table, experts=cfg["E"], top_k=cfg["k"], d_model=cfg["d"], ffn=cfg["ffn"],
                      gate_type=t, up_type=t, down_type=t, up_offset=gate_bytes, down_offset=2 * gate_bytes, y=y)
    return a, table


@pytest.mark.gpu
@pytest.mark.parametrize("t", [TYPE_Q4_K, TYPE_Q8_0])
def test_noalloc_matches_workspace_entry_point(cuda, oracle, t):
    from freemoe_b200._lib import check, load

    lib = load()
    for call, seed in enumerate((101, 202)):  # two calls in a row, different inputs
        slots, x, logits, cfg = make_block(oracle, seed + t, t, T=5 + 4 * call)
        y_ref = torch.empty(cfg["T"], cfg["d"], device="cuda")
        y_new = torch.full((cfg["T"], cfg["d"]), float("nan"), device="cuda")
        a_ref, keep_ref = args_for(cuda, slots, x, logits, cfg, t, y_ref)
        need = cuda.moe_workspace_bytes(cfg["T"], cfg["E"], cfg["k"], cfg["d"], cfg["ffn"])
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        check(lib.fmcuda_moe_block(C.byref(a_ref), C.c_void_p(ws.data_ptr()), need, None))
        a_new, keep_new = args_for(cuda, slots, x, logits, cfg, t, y_new)
        check(lib.fmcuda_moe_block_noalloc(C.byref(a_new), None))
        torch.cuda.synchronize()
        assert cuda.device_status() == 0
        ref, got = y_ref.cpu().numpy(), y_new.cpu().numpy()
        assert np.isfinite(got).all()
        err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
        assert err <= TOL, f"call {call}: {err}"


@pytest.mark.gpu
def test_noalloc_refuses_blocks_larger_than_its_scratch(cuda):
    from freemoe_b200._lib import load

    lib = load()
    a = MoeArgs()
    a.tokens, a.experts, a.top_k, a.d_model, a.ffn = 64, 8, 8, 4096, 14336
    need = cuda.moe_workspace_bytes(64, 8, 8, 4096, 14336)
    assert need > MOE_NOALLOC_SCRATCH_BYTES
    assert lib.fmcuda_moe_block_noalloc(C.byref(a), None) == 26  # INVALID_ARGUMENT
    assert b"scratch" in lib.fmcuda_last_error()
