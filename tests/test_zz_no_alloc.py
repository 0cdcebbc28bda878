"""fmcuda_moe_block_noalloc: the MoE block for callers that cannot allocate.

Some hosts cannot call cudaMalloc once decoding runs -- all of their HBM is
already committed to expert slots, or the device allocator belongs to the host
framework -- so the library offers a variant of the MoE block whose scratch is
a fixed array inside the library image.  These tests call it through the C ABI
and compare it with fmcuda_moe_block (which uses a caller workspace) bit for
bit: both run the same kernels in the same order, so any difference would be
a fault of the shared scratch.  Calls come in a row with different inputs, so
a result that depended on what the previous call left in the scratch would
show; they cover the single-launch front end (T <= 64, plain router), the
separate router / grouping / x-plane kernels (T > 64, and a router variant),
and free device memory must not move once the scratch is mapped.  Collected
last on purpose (file name), and independent of the other tests' state.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from freemoe_b200._lib import MOE_NOALLOC_SCRATCH_BYTES, MoeArgs
from oracle.oracle import TYPE_Q4_K, TYPE_Q8_0, bf16_round

GATING_SIGMOID = 1  # FM_GATING_SIGMOID


def make_block(oracle, seed, t, E=8, k=2, d=512, ffn=768, T=5):
    rng = np.random.default_rng(seed)
    slots = [torch.from_numpy(np.concatenate([oracle.quantize(t, rng.normal(0, 0.02, n).astype(np.float32))
                                              for n in (ffn * d, ffn * d, d * ffn)])).cuda() for _ in range(E)]
    x = torch.from_numpy(bf16_round(rng.normal(0, 1, (T, d)).astype(np.float32))).cuda().to(torch.bfloat16)
    logits = torch.from_numpy(rng.normal(0, 1, (T, E)).astype(np.float32)).cuda()
    return slots, x, logits, dict(E=E, k=k, d=d, ffn=ffn, T=T)


def args_for(cuda, slots, x, logits, cfg, t, y, router=None):
    gate_bytes = cuda.row_bytes(t, cfg["d"]) * cfg["ffn"]
    table = cuda.slot_table(slots, x.device)
    a = cuda.moe_args(x, logits, table, experts=cfg["E"], top_k=cfg["k"], d_model=cfg["d"], ffn=cfg["ffn"],
                      gate_type=t, up_type=t, down_type=t, up_offset=gate_bytes, down_offset=2 * gate_bytes, y=y,
                      router=router)
    return a, table


def run_both(cuda, lib, slots, x, logits, cfg, t, router=None):
    """The block through fmcuda_moe_block and through fmcuda_moe_block_noalloc."""
    from freemoe_b200._lib import check

    y_ref = torch.empty(cfg["T"], cfg["d"], device="cuda")
    y_new = torch.full((cfg["T"], cfg["d"]), float("nan"), device="cuda")
    a_ref, keep_ref = args_for(cuda, slots, x, logits, cfg, t, y_ref, router)
    need = cuda.moe_workspace_bytes(cfg["T"], cfg["E"], cfg["k"], cfg["d"], cfg["ffn"])
    assert need <= MOE_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    check(lib.fmcuda_moe_block(C.byref(a_ref), C.c_void_p(ws.data_ptr()), need, None))
    a_new, keep_new = args_for(cuda, slots, x, logits, cfg, t, y_new, router)
    check(lib.fmcuda_moe_block_noalloc(C.byref(a_new), None))
    torch.cuda.synchronize()
    assert cuda.device_status() == 0
    return y_ref.cpu().numpy(), y_new.cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("t", [TYPE_Q4_K, TYPE_Q8_0])
def test_noalloc_matches_workspace_entry_point(cuda, oracle, t):
    from freemoe_b200._lib import load

    lib = load()
    # a tokens = 0 call looks the scratch up and does nothing else
    empty = MoeArgs()
    assert lib.fmcuda_moe_block_noalloc(C.byref(empty), None) == 0
    free_before = None
    # two calls in a row through the single-launch front end, then a call with
    # more tokens than it takes and a call with a router variant (both through
    # the separate router / grouping / x-plane kernels)
    router = cuda.router_config(gating=GATING_SIGMOID, groups=4, groups_used=2)
    for call, (seed, T, rt) in enumerate(((101, 5, None), (202, 9, None), (303, 70, None), (404, 12, router))):
        slots, x, logits, cfg = make_block(oracle, seed + t, t, T=T)
        torch.cuda.synchronize()
        if call == 1:
            free_before = torch.cuda.mem_get_info()[0]
        ref, got = run_both(cuda, lib, slots, x, logits, cfg, t, rt)
        if call == 1:
            # the scratch was mapped by the first call: this one moved no device memory
            assert torch.cuda.mem_get_info()[0] == free_before
        assert np.isfinite(got).all()
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), f"call {call} differs"


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
