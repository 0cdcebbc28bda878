"""Torch-tensor conveniences over the C ABI (device memory and streams only).

Each function is a thin call through ``libfreemoe_b200.so``; PyTorch provides
the device buffers and the current stream.  Names follow the reference's
routines for the path (cited per function).
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import (GEOMETRY, ORDER_ANY, TYPE_F32, X_BF16, X_F32, DeviceInfo, FmError, MoeArgs, RouterConfig, SharedExpert,
                   check, load)


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def row_bytes(type_id: int, in_dim: int) -> int:
    bs, bb = GEOMETRY[type_id]
    if in_dim % bs:
        raise FmError(8, "quantised row length is not a whole number of blocks")
    return in_dim // bs * bb


def init(device: int = 0) -> None:
    check(load().fmcuda_init(device))


def device_info(device: int = 0) -> dict:
    info = DeviceInfo()
    check(load().fmcuda_device_info_get(device, C.byref(info)))
    return {f: (getattr(info, f).decode() if f == "name" else getattr(info, f)) for f, _ in info._fields_}


def device_status(clear: bool = True) -> int:
    v = C.c_int32(0)
    check(load().fmcuda_device_status(1 if clear else 0, C.byref(v)))
    return v.value


def dequantize_tensor_region(type_id: int, src: torch.Tensor, n_elems: int, stream=None) -> torch.Tensor:
    """K1: src/quant.cpp:723-732 on the device (bit-exact)."""
    out = torch.empty(n_elems, dtype=torch.float32, device=src.device)
    check(load().fmcuda_dequant(type_id, _ptr(src), _ptr(out), n_elems, _stream(stream)))
    return out


def gemv_quant(type_id: int, w: torch.Tensor, x: torch.Tensor, out_dim: int, in_dim: int,
               stream=None) -> torch.Tensor:
    """K2: gemv_quant / gemm_quant (src/kernels.cpp:846-878, :316-345).

    ``x`` is [tokens, in_dim] (or [in_dim]) in float32 or bfloat16; returns
    float32 [tokens, out_dim]."""
    x2 = x.reshape(-1, in_dim).contiguous()
    dt = X_BF16 if x2.dtype == torch.bfloat16 else X_F32
    if x2.dtype not in (torch.bfloat16, torch.float32):
        raise FmError(26, "activations must be float32 or bfloat16")
    y = torch.empty(x2.shape[0], out_dim, dtype=torch.float32, device=x2.device)
    check(load().fmcuda_gemv(type_id, _ptr(w), _ptr(x2), dt, _ptr(y), x2.shape[0], out_dim, in_dim,
                             _stream(stream)))
    return y


def matvec_f32(w: torch.Tensor, x: torch.Tensor, out_dim: int, in_dim: int, order: int = ORDER_ANY,
               stream=None) -> torch.Tensor:
    """Backend::matvec (include/fm/backend.hpp:157) in a chosen summation order."""
    y = torch.empty(out_dim, dtype=torch.float32, device=x.device)
    check(load().fmcuda_matvec_f32(_ptr(w), _ptr(x), _ptr(y), out_dim, in_dim, order, _stream(stream)))
    return y


def route(logits: torch.Tensor, top_k: int, normalise: bool = True, epsilon: float = 6.103515625e-5,
          scale: float = 1.0, want_probs: bool = False, stream=None):
    """K4: Engine::softmax/topk + renormalisation (src/engine.cpp:378-411, :1680-1702)."""
    tokens, experts = logits.shape
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device=logits.device)
    w = torch.empty(tokens, top_k, dtype=torch.float32, device=logits.device)
    probs = torch.empty(tokens, experts, dtype=torch.float32, device=logits.device) if want_probs else None
    check(load().fmcuda_route(_ptr(logits), tokens, experts, top_k, 1 if normalise else 0, epsilon,
                              scale, _ptr(ids), _ptr(w), _ptr(probs), _stream(stream)))
    return (ids, w, probs) if want_probs else (ids, w)


def router_config(gating: int = 0, logit_bias: torch.Tensor | None = None,
                  selection_bias: torch.Tensor | None = None, groups: int = 1, groups_used: int = 1,
                  normalise: bool = True, epsilon_additive: bool = False, epsilon: float = 6.103515625e-5,
                  scale: float = 1.0) -> RouterConfig:
    """The C struct of a router variant (src/engine.cpp:1603-1702); the caller
    keeps the bias tensors alive."""
    c = RouterConfig()
    c.gating = gating
    c.logit_bias = logit_bias.data_ptr() if logit_bias is not None else None
    c.selection_bias = selection_bias.data_ptr() if selection_bias is not None else None
    c.groups, c.groups_used = groups, groups_used
    c.normalise = 1 if normalise else 0
    c.epsilon_additive = 1 if epsilon_additive else 0
    c.epsilon, c.scale = epsilon, scale
    return c


def route_ex(logits: torch.Tensor, top_k: int, config: RouterConfig, want_probs: bool = False, stream=None):
    """Router variants: ids [T, k] int32, weights [T, k] f32 (and probs [T, E])."""
    T, E = logits.shape
    ids = torch.empty(T, top_k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=logits.device)
    probs = torch.empty(T, E, dtype=torch.float32, device=logits.device) if want_probs else None
    check(load().fmcuda_route_ex(_ptr(logits.contiguous()), T, E, top_k, C.byref(config), _ptr(ids), _ptr(w),
                                 _ptr(probs) if probs is not None else None, _stream(stream)))
    return (ids, w, probs) if want_probs else (ids, w)


def group_by_expert(ids: torch.Tensor, experts: int, stream=None):
    """Grouping of (token, rank) pairs by expert: counts, offsets, pairs, slot_of."""
    tokens, top_k = ids.shape
    dev = ids.device
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    pairs = torch.empty(tokens * top_k, dtype=torch.int32, device=dev)
    slot_of = torch.empty(tokens * top_k, dtype=torch.int32, device=dev)
    check(load().fmcuda_group(_ptr(ids), tokens, top_k, experts, _ptr(counts), _ptr(offsets),
                              _ptr(pairs), _ptr(slot_of), _stream(stream)))
    return counts, offsets, pairs, slot_of


def group_by_expert_batched(ids: torch.Tensor, experts: int, stream=None):
    """The many-warp grouping for large batches (same outputs as group_by_expert)."""
    tokens, top_k = ids.shape
    dev = ids.device
    counts = torch.empty(experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(experts + 1, dtype=torch.int32, device=dev)
    pairs = torch.empty(tokens * top_k, dtype=torch.int32, device=dev)
    slot_of = torch.empty(tokens * top_k, dtype=torch.int32, device=dev)
    scratch = torch.empty(max(1, load().fmcuda_group_scratch_bytes(tokens * top_k, experts)), dtype=torch.uint8,
                          device=dev)
    check(load().fmcuda_group_batched(_ptr(ids), tokens, top_k, experts, _ptr(counts), _ptr(offsets),
                                      _ptr(pairs), _ptr(slot_of), _ptr(scratch), _stream(stream)))
    return counts, offsets, pairs, slot_of


def moe_workspace_bytes(tokens: int, experts: int, top_k: int, d_model: int, ffn: int) -> int:
    v = C.c_uint64(0)
    check(load().fmcuda_moe_workspace_bytes(tokens, experts, top_k, d_model, ffn, C.byref(v)))
    return v.value


def moe_args(x, logits, slot_table, *, experts, top_k, d_model, ffn, gate_type, up_type, down_type,
             up_offset, down_offset, y, ids_out=None, weights_out=None, normalise=True,
             epsilon=6.103515625e-5, scale=1.0, stage_events=None, router=None) -> MoeArgs:
    """Fills the C struct; ``stage_events`` is a ctypes array of 8 cudaEvent_t
    handles (or None).  The caller keeps every referenced tensor alive."""
    a = MoeArgs()
    a.x = x.data_ptr()
    a.x_dtype = X_BF16 if x.dtype == torch.bfloat16 else X_F32
    a.logits = logits.data_ptr()
    a.tokens = x.shape[0]
    a.experts = experts
    a.top_k = top_k
    a.d_model = d_model
    a.ffn = ffn
    a.expert_slots = slot_table.data_ptr()
    a.up_offset = up_offset
    a.down_offset = down_offset
    a.gate_type, a.up_type, a.down_type = gate_type, up_type, down_type
    a.normalise = 1 if normalise else 0
    a.epsilon = epsilon
    a.scale = scale
    a.y = y.data_ptr()
    a.ids_out = ids_out.data_ptr() if ids_out is not None else None
    a.weights_out = weights_out.data_ptr() if weights_out is not None else None
    a.stage_events = C.cast(stage_events, C.c_void_p) if stage_events is not None else None
    a.router = C.cast(C.pointer(router), C.c_void_p) if router is not None else None
    a._router_ref = router  # keep the struct alive with the args
    return a


def slot_table(slots, device) -> torch.Tensor:
    """Device array of expert payload base pointers (0 = not resident)."""
    ptrs = [0 if s is None else (s if isinstance(s, int) else s.data_ptr()) for s in slots]
    return torch.tensor(ptrs, dtype=torch.int64, device=device)


def moe_block(x: torch.Tensor, logits: torch.Tensor, slots, *, top_k: int, ffn: int, gate_type: int,
              up_type: int | None = None, down_type: int | None = None, workspace=None,
              return_routing: bool = False, stream=None):
    """One routed-expert MoE block (src/engine.cpp:1603-1772) on the device.

    ``slots`` is a list (per expert) of uint8 payload tensors laid out gate ||
    up || down (an ExpertRecord), or None for an expert that is not resident."""
    up_type = gate_type if up_type is None else up_type
    down_type = gate_type if down_type is None else down_type
    tokens, d_model = x.shape
    experts = logits.shape[1]
    gate_bytes = row_bytes(gate_type, d_model) * ffn
    up_bytes = row_bytes(up_type, d_model) * ffn
    table = slot_table(slots, x.device)
    need = moe_workspace_bytes(tokens, experts, top_k, d_model, ffn)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    y = torch.empty(tokens, d_model, dtype=torch.float32, device=x.device)
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device=x.device) if return_routing else None
    wts = torch.empty(tokens, top_k, dtype=torch.float32, device=x.device) if return_routing else None
    a = moe_args(x, logits, table, experts=experts, top_k=top_k, d_model=d_model, ffn=ffn,
                 gate_type=gate_type, up_type=up_type, down_type=down_type, up_offset=gate_bytes,
                 down_offset=gate_bytes + up_bytes, y=y, ids_out=ids, weights_out=wts)
    check(load().fmcuda_moe_block(C.byref(a), _ptr(workspace), workspace.numel(), _stream(stream)))
    if return_routing:
        return y, ids, wts
    return y


def moe_prefill_workspace_bytes(tokens: int, experts: int, top_k: int, d_model: int, ffn: int,
                                shared_ffn: int = 0) -> int:
    v = C.c_uint64(0)
    check(load().fmcuda_moe_prefill_workspace_bytes(tokens, experts, top_k, d_model, ffn, shared_ffn,
                                                     C.byref(v)))
    return v.value


def shared_expert_args(slot: torch.Tensor, *, d_model: int, ffn: int, gate_type: int, up_type=None,
                       down_type=None, gate_scalar: torch.Tensor | None = None) -> SharedExpert:
    """The C struct for a shared expert whose payload is gate || up || down."""
    up_type = gate_type if up_type is None else up_type
    down_type = gate_type if down_type is None else down_type
    gate_bytes = row_bytes(gate_type, d_model) * ffn
    up_bytes = row_bytes(up_type, d_model) * ffn
    s = SharedExpert()
    s.slot = slot.data_ptr()
    s.ffn = ffn
    s.up_offset = gate_bytes
    s.down_offset = gate_bytes + up_bytes
    s.gate_type, s.up_type, s.down_type = gate_type, up_type, down_type
    s.gate_scalar = gate_scalar.data_ptr() if gate_scalar is not None else None
    return s


def moe_prefill(x: torch.Tensor, logits: torch.Tensor, slots, *, top_k: int, ffn: int, gate_type: int,
                up_type: int | None = None, down_type: int | None = None, shared=None, workspace=None,
                return_routing: bool = False, stream=None):
    """The routed MoE block for a batch of tokens on the tcgen05 grouped GEMM
    (fmcuda_moe_prefill).  ``shared`` is an optional :func:`shared_expert_args`."""
    up_type = gate_type if up_type is None else up_type
    down_type = gate_type if down_type is None else down_type
    tokens, d_model = x.shape
    experts = logits.shape[1]
    gate_bytes = row_bytes(gate_type, d_model) * ffn
    up_bytes = row_bytes(up_type, d_model) * ffn
    table = slot_table(slots, x.device)
    need = moe_prefill_workspace_bytes(tokens, experts, top_k, d_model, ffn, shared.ffn if shared else 0)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    y = torch.empty(tokens, d_model, dtype=torch.float32, device=x.device)
    ids = torch.empty(tokens, top_k, dtype=torch.int32, device=x.device) if return_routing else None
    wts = torch.empty(tokens, top_k, dtype=torch.float32, device=x.device) if return_routing else None
    a = moe_args(x, logits, table, experts=experts, top_k=top_k, d_model=d_model, ffn=ffn,
                 gate_type=gate_type, up_type=up_type, down_type=down_type, up_offset=gate_bytes,
                 down_offset=gate_bytes + up_bytes, y=y, ids_out=ids, weights_out=wts)
    check(load().fmcuda_moe_prefill(C.byref(a), C.byref(shared) if shared is not None else None,
                                    _ptr(workspace), workspace.numel(), _stream(stream)))
    if return_routing:
        return y, ids, wts
    return y


def synth_weights(type_id: int, rows: int, cols: int, seed: int, std: float = 0.02,
                  device="cuda", stream=None) -> torch.Tensor:
    """Seeded Gaussian weights encoded on the device (Q8_0 / Q4_K / F32 bytes)."""
    nbytes = rows * row_bytes(type_id, cols)
    out = torch.empty(nbytes, dtype=torch.uint8, device=device)
    check(load().fmcuda_synth_weights(type_id, _ptr(out), rows, cols, seed, std, _stream(stream)))
    return out
