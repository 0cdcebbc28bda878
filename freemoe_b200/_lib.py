"""ctypes binding of ``libfreemoe_b200.so`` (the C ABI in include/freemoe_b200.h).

Loading fails loudly: there is no CPU fallback for the hot path.  If the
shared library is missing, build it with ``python freemoe_b200/build.py``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import os

# FREEMOE_B200_LIB selects another build of the same library (same ABI).
LIB_PATH = Path(os.environ.get("FREEMOE_B200_LIB") or Path(__file__).resolve().parent / "libfreemoe_b200.so")

# fm::ErrorCode ordinals (include/fm/common.hpp:27-57 of the reference)
ERROR_NAMES = {
    0: "OK", 1: "MALFORMED_GGUF", 2: "UNSUPPORTED_ARCHITECTURE", 3: "UNSUPPORTED_QUANTISATION",
    4: "INVALID_TOKENIZER", 5: "MISSING_REQUIRED_TENSOR", 6: "UNKNOWN_TENSOR",
    7: "DUPLICATE_TENSOR", 8: "SHAPE_MISMATCH", 9: "METADATA_MISMATCH", 10: "SOURCE_CHANGED",
    11: "IO_ERROR", 12: "SHORT_READ", 13: "DIRECT_IO_FALLBACK", 14: "ALLOCATION_FAILED",
    15: "BUDGET_TOO_SMALL", 16: "INVALID_EXPERT_ID", 17: "EXPERT_CHECKSUM_MISMATCH",
    18: "EXPERT_EXECUTION_MISMATCH", 19: "SLOTS_BUSY", 20: "STALE_COMPLETION",
    21: "TRANSFER_FAILED", 22: "FENCE_TIMEOUT", 23: "DEVICE_LOSS",
    24: "GPU_BACKEND_UNIMPLEMENTED", 25: "CPU_FALLBACK_DISABLED", 26: "INVALID_ARGUMENT",
    27: "NOT_IMPLEMENTED", 28: "INTERNAL_ERROR",
}

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 8, 12, 14
MOE_NOALLOC_SCRATCH_BYTES = 16 * 1024 * 1024  # FM_MOE_NOALLOC_SCRATCH_BYTES
X_F32, X_BF16 = 0, 1
ORDER_ANY, ORDER_SCALAR, ORDER_AVX2 = 0, 1, 2

# {block_size, block_bytes} (src/gguf.cpp:58-106 of the reference)
GEOMETRY = {TYPE_F32: (1, 4), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}


class FmError(RuntimeError):
    """A typed failure, the Python face of fm::Error (include/fm/common.hpp:62-71)."""

    def __init__(self, code: int, message: str):
        self.code = code
        self.name = ERROR_NAMES.get(code, f"E{code}")
        super().__init__(f"{self.name}: {message}")


class DeviceInfo(C.Structure):
    _fields_ = [
        ("name", C.c_char * 256),
        ("total_memory_bytes", C.c_uint64),
        ("free_memory_bytes", C.c_uint64),
        ("sm_count", C.c_int32),
        ("cc_major", C.c_int32),
        ("cc_minor", C.c_int32),
        ("driver_version", C.c_int32),
        ("runtime_version", C.c_int32),
        ("l2_bytes", C.c_int32),
    ]


class MoeArgs(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("x_dtype", C.c_int32),
        ("logits", C.c_void_p),
        ("tokens", C.c_uint32),
        ("experts", C.c_uint32),
        ("top_k", C.c_uint32),
        ("d_model", C.c_uint32),
        ("ffn", C.c_uint32),
        ("expert_slots", C.c_void_p),
        ("up_offset", C.c_uint64),
        ("down_offset", C.c_uint64),
        ("gate_type", C.c_uint32),
        ("up_type", C.c_uint32),
        ("down_type", C.c_uint32),
        ("normalise", C.c_int32),
        ("epsilon", C.c_double),
        ("scale", C.c_double),
        ("y", C.c_void_p),
        ("ids_out", C.c_void_p),
        ("weights_out", C.c_void_p),
        ("stage_events", C.c_void_p),
        ("router", C.c_void_p),
    ]


class EpLayerArgs(C.Structure):
    """fmcuda_ep_layer_args (include/freemoe_b200.h)."""
    _fields_ = [
        ("x", C.c_void_p),
        ("x_dtype", C.c_int32),
        ("logits", C.c_void_p),
        ("tokens", C.c_uint32),
        ("experts", C.c_uint32),
        ("top_k", C.c_uint32),
        ("d_model", C.c_uint32),
        ("ffn", C.c_uint32),
        ("local_slots", C.c_void_p),
        ("up_offset", C.c_uint64),
        ("down_offset", C.c_uint64),
        ("gate_type", C.c_uint32),
        ("up_type", C.c_uint32),
        ("down_type", C.c_uint32),
        ("normalise", C.c_int32),
        ("epsilon", C.c_double),
        ("scale", C.c_double),
        ("y", C.c_void_p),
    ]


EP_NCCL_ID_BYTES = 128

GATING_SOFTMAX, GATING_SIGMOID, GATING_SQRT_SOFTPLUS, GATING_SOFTMAX_WEIGHT = 0, 1, 2, 3


class RouterConfig(C.Structure):
    _fields_ = [
        ("gating", C.c_int32),
        ("logit_bias", C.c_void_p),
        ("selection_bias", C.c_void_p),
        ("groups", C.c_uint32),
        ("groups_used", C.c_uint32),
        ("normalise", C.c_int32),
        ("epsilon_additive", C.c_int32),
        ("epsilon", C.c_double),
        ("scale", C.c_double),
    ]


class SharedExpert(C.Structure):
    _fields_ = [
        ("slot", C.c_void_p),
        ("ffn", C.c_uint32),
        ("up_offset", C.c_uint64),
        ("down_offset", C.c_uint64),
        ("gate_type", C.c_uint32),
        ("up_type", C.c_uint32),
        ("down_type", C.c_uint32),
        ("gate_scalar", C.c_void_p),
    ]


class Extent(C.Structure):
    _fields_ = [("offset", C.c_uint64), ("size", C.c_uint64)]


class FileIdentity(C.Structure):
    _fields_ = [("size", C.c_uint64), ("dev", C.c_uint64), ("ino", C.c_uint64), ("mtime_ns", C.c_int64),
                ("ctime_ns", C.c_int64), ("content_probe", C.c_uint64)]


class RecordLoadStats(C.Structure):
    _fields_ = [("payload_bytes", C.c_uint64), ("physical_bytes", C.c_uint64), ("read_requests", C.c_uint64),
                ("coalesced_requests", C.c_uint64), ("direct_fallbacks", C.c_uint64), ("checksum", C.c_uint64),
                ("elapsed_ms", C.c_double)]


READER_BUFFERED, READER_DIRECT = 1, 3  # fm::ReaderMode ordinals

MOE_STAGES = ("router", "grouping", "x_planes", "gate_up", "act_planes", "down", "combine")
# the prefill path's stages under the same eight events (stage 5 is empty there)
PREFILL_STAGES = ("router", "grouping", "gather", "gate_up", "none", "down", "combine")


# (name, restype, argtypes): every symbol declared in include/freemoe_b200.h
_P, _U32, _U64, _I32, _D, _F = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32, C.c_double, C.c_float
SIGNATURES = [
    ("fmcuda_last_error", C.c_char_p, []),
    ("fmcuda_init", C.c_int, [_I32]),
    ("fmcuda_device_info_get", C.c_int, [_I32, C.POINTER(DeviceInfo)]),
    ("fmcuda_malloc", C.c_int, [_U64, C.POINTER(C.c_void_p)]),
    ("fmcuda_malloc_managed", C.c_int, [_U64, C.POINTER(C.c_void_p)]),
    ("fmcuda_free", C.c_int, [_P]),
    ("fmcuda_host_alloc", C.c_int, [_U64, C.POINTER(C.c_void_p)]),
    ("fmcuda_host_free", C.c_int, [_P]),
    ("fmcuda_stream_create", C.c_int, [C.POINTER(C.c_void_p)]),
    ("fmcuda_stream_destroy", C.c_int, [_P]),
    ("fmcuda_stream_sync", C.c_int, [_P]),
    ("fmcuda_event_create", C.c_int, [C.POINTER(C.c_void_p)]),
    ("fmcuda_event_destroy", C.c_int, [_P]),
    ("fmcuda_event_record", C.c_int, [_P, _P]),
    ("fmcuda_event_create_timing", C.c_int, [C.POINTER(C.c_void_p)]),
    ("fmcuda_event_elapsed_ms", C.c_int, [_P, _P, C.POINTER(C.c_float)]),
    ("fmcuda_upload_async", C.c_int, [_P, _P, _U64, _P, _P]),
    ("fmcuda_event_query", C.c_int, [_P, C.POINTER(C.c_int32)]),
    ("fmcuda_event_wait", C.c_int, [_P, _U32]),
    ("fmcuda_download", C.c_int, [_P, _P, _U64, _P]),
    ("fmcuda_memset_async", C.c_int, [_P, _I32, _U64, _P]),
    ("fmcuda_device_status", C.c_int, [_I32, C.POINTER(C.c_int32)]),
    ("fmcuda_row_bytes", C.c_uint64, [_U32, _U32]),
    ("fmcuda_dequant", C.c_int, [_U32, _P, _P, _U64, _P]),
    ("fmcuda_gemv", C.c_int, [_U32, _P, _P, _I32, _P, _U32, _U32, _U32, _P]),
    ("fmcuda_matvec_f32", C.c_int, [_P, _P, _P, _U32, _U32, _I32, _P]),
    ("fmcuda_route", C.c_int, [_P, _U32, _U32, _U32, _I32, _D, _D, _P, _P, _P, _P]),
    ("fmcuda_route_ex", C.c_int, [_P, _U32, _U32, _U32, C.POINTER(RouterConfig), _P, _P, _P, _P]),
    ("fmcuda_group", C.c_int, [_P, _U32, _U32, _U32, _P, _P, _P, _P, _P]),
    ("fmcuda_group_scratch_bytes", C.c_uint64, [_U32, _U32]),
    ("fmcuda_group_batched", C.c_int, [_P, _U32, _U32, _U32, _P, _P, _P, _P, _P, _P]),
    ("fmcuda_moe_workspace_bytes", C.c_int, [_U32, _U32, _U32, _U32, _U32, C.POINTER(C.c_uint64)]),
    ("fmcuda_moe_block", C.c_int, [C.POINTER(MoeArgs), _P, _U64, _P]),
    ("fmcuda_moe_block_noalloc", C.c_int, [C.POINTER(MoeArgs), _P]),
    ("fmcuda_moe_prefill_workspace_bytes", C.c_int, [_U32, _U32, _U32, _U32, _U32, _U32, C.POINTER(C.c_uint64)]),
    ("fmcuda_moe_prefill", C.c_int, [C.POINTER(MoeArgs), C.POINTER(SharedExpert), _P, _U64, _P]),
    ("fmcuda_ep_dispatch_scratch_bytes", C.c_uint64, [_U32, _U32, _U32]),
    ("fmcuda_ep_dispatch", C.c_int, [_P, _U32, _U32, _U32, _U32, _P, _I32, _U32, _P, _P, _P, _P, _P, _P, _P, _P]),
    ("fmcuda_moe_experts_workspace_bytes", C.c_uint64, [_U32, _U32, _U32, _U32]),
    ("fmcuda_moe_experts", C.c_int, [_P, _P, _U32, _U32, _P, _U64, _U64, _U32, _U32, _U32, _U32, _U32, _P, _P,
                                     _U64, _P]),
    ("fmcuda_moe_combine", C.c_int, [_P, _P, _P, _U32, _U32, _U32, _P, _P]),
    ("fmcuda_ep_dispatch_rows_scratch_bytes", C.c_uint64, [_U32, _U32]),
    ("fmcuda_ep_dispatch_rows", C.c_int, [_P, _P, _U32, _U32, _U32, _U32, _P, _I32, _U32, _P, _P, _P, _P, _P, _P,
                                          _P, _P, _P]),
    ("fmcuda_moe_experts_partial_workspace_bytes", C.c_uint64, [_U32, _U32, _U32, _U32, _U32]),
    ("fmcuda_moe_experts_partial", C.c_int, [_P, _P, _P, _U32, _U32, _U32, _P, _U64, _U64, _U32, _U32, _U32, _U32,
                                             _U32, _P, _P, _U64, _P]),
    ("fmcuda_ep_combine_rows", C.c_int, [_P, _P, _U32, _U32, _U32, _P, _P]),
    ("fmcuda_ep_nccl_unique_id", C.c_int, [_P]),
    ("fmcuda_ep_init", C.c_int, [_P, _U32, _U32, C.POINTER(C.c_void_p)]),
    ("fmcuda_ep_destroy", C.c_int, [_P]),
    ("fmcuda_ep_layer_workspace_bytes", C.c_int, [_U32, _U32, _U32, _U32, _U32, _U32, C.POINTER(C.c_uint64)]),
    ("fmcuda_ep_layer", C.c_int, [_P, C.POINTER(EpLayerArgs), _U32, _P, C.c_uint64, _P]),
    ("fmcuda_ep_mailbox_bytes", _U64, [_U32, _U32, _U32, _U32]),
    ("fmcuda_ep_mailbox_alloc", C.c_int, [_U64, C.POINTER(C.c_void_p), _P]),
    ("fmcuda_ep_mailbox_open", C.c_int, [_P, C.POINTER(C.c_void_p)]),
    ("fmcuda_ep_mailbox_close", C.c_int, [_P]),
    ("fmcuda_ep_mailbox_free", C.c_int, [_P]),
    ("fmcuda_ep_p2p_dispatch_scratch_bytes", _U64, [_U32, _U32]),
    ("fmcuda_ep_p2p_dispatch", C.c_int, [_P, _P, _U32, _U32, _U32, _U32, _U32, _P, C.c_int32, _U32, _P, _P, _U32,
                                         _U32, _P, _P, _U32, _P]),
    ("fmcuda_ep_p2p_experts_workspace_bytes", _U64, [_U32, _U32, _U32, _U32, _U32]),
    ("fmcuda_ep_p2p_experts", C.c_int, [_P, _P, _U32, _U32, _U32, _U32, _U32, _U32, _P, _U64, _U64, _U32, _U32, _U32,
                                        _U32, _U32, _P, _U64, _U32, _P]),
    ("fmcuda_ep_p2p_combine", C.c_int, [_P, _U32, _U32, _U32, _U32, _U32, _P, _U32, _U32, _P, _U32, _P]),
    ("fmcuda_fnv1a64_workspace_bytes", _U64, [_U64]),
    ("fmcuda_fnv1a64", C.c_int, [_P, _U64, _P, _P, _U64, _P]),
    ("fmcuda_file_identity_get", C.c_int, [C.c_char_p, C.POINTER(FileIdentity)]),
    ("fmcuda_coalesce_extents", C.c_int, [C.POINTER(Extent), _U32, _U64, _P, _P, _P, C.POINTER(C.c_uint32)]),
    ("fmcuda_record_loader_create", C.c_int, [C.c_char_p, C.c_int, _U64, _U64, _U32, _U32, C.c_int,
                                              C.POINTER(FileIdentity), C.POINTER(C.c_void_p)]),
    ("fmcuda_record_loader_destroy", C.c_int, [_P]),
    ("fmcuda_record_load_workspace_bytes", _U64, [_U64]),
    ("fmcuda_record_load", C.c_int, [_P, C.POINTER(Extent), _U32, _P, _U64, C.c_int, _U64, _P, _U64, _P, _U32,
                                     C.POINTER(RecordLoadStats)]),
    ("fmcuda_synth_weights", C.c_int, [_U32, _P, _U64, _U32, _U64, _F, _P]),
]

_lib = None


def load() -> C.CDLL:
    """Loads the shared library once; raises if it is missing (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FmError(24, f"{LIB_PATH} is missing: build it with `python freemoe_b200/build.py`")
    lib = C.CDLL(str(LIB_PATH))
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != 0:
        msg = load().fmcuda_last_error()
        raise FmError(rc, msg.decode() if msg else "")
