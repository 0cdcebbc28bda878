"""numpy bindings of the CPU oracle.

TEST INFRASTRUCTURE ONLY.  ``libfm_oracle.so`` is the C restatement
(fm_oracle.c) of the reference's hot-path arithmetic; ``_ref/libfmref.so`` is
the reference's own code compiled from source (ref_shim.cpp over
src/quant.cpp, src/kernels.cpp, src/engine.cpp, ...).  Only tests/, the smoke
check and the CPU legs of bench.py use this module, and only as the checker or
the timed CPU baseline, never as part of the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libfm_oracle.so"
REF_SO = HERE / "_ref" / "libfmref.so"
# The reference tree, only ever named by the environment (FM_REFERENCE); the
# test-side checkers that need it are built only when it is set.
REF_TREE = Path(os.environ["FM_REFERENCE"]) if os.environ.get("FM_REFERENCE") else None

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K = 0, 8, 12, 14
GEOMETRY = {TYPE_F32: (1, 4), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}
EPS = 6.103515625e-5

_P = C.c_void_p
_u32, _u64, _f, _d, _i = C.c_uint32, C.c_uint64, C.c_float, C.c_double, C.c_int


def build(ref: bool | None = None) -> None:
    """Builds the restatement, and the reference shim when its tree is present."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    if ref is None:
        ref = REF_TREE is not None and REF_TREE.exists()
    if ref:
        if REF_TREE is None or not REF_TREE.exists():
            raise FileNotFoundError("the reference checkers need the reference tree: set FM_REFERENCE")
        subprocess.run(["make", "-s", "-j8", "-C", str(HERE), "ref", "engine", f"REF={REF_TREE}"], check=True)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


class Oracle:
    """The C restatement (fm_oracle.c)."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            build(ref=False)
        lib = C.CDLL(str(path))
        sig = {
            "fmo_fp16_to_f32": (_f, [C.c_uint16]),
            "fmo_f32_to_fp16": (C.c_uint16, [_f]),
            "fmo_dequant_block": (_i, [_u32, _P, _P]),
            "fmo_dequant_region": (_i, [_u32, _P, _P, _u64]),
            "fmo_gemv_f32_scalar": (None, [_P, _P, _P, _u32, _u32]),
            "fmo_gemv_f32_avx2_order": (None, [_P, _P, _P, _u32, _u32]),
            "fmo_gemv_quant_f64": (_i, [_u32, _P, _P, _P, _u32, _u32, _u32]),
            "fmo_gemv_quant_fused_scalar": (_i, [_u32, _P, _P, _P, _u32, _u32, _u32]),
            "fmo_route": (_i, [_P, _u32, _u32, _u32, _i, _d, _d, _P, _P, _P]),
            "fmo_route_ex": (_i, [_P, _u32, _u32, _u32, _i, _P, _P, _u32, _u32, _i, _i, _d, _d, _P, _P, _P]),
            "fmo_group_by_expert": (_i, [_P, _u32, _u32, _u32, _P, _P, _P, _P]),
            "fmo_swiglu": (_f, [_f, _f]),
            "fmo_moe_block": (_i, [_P, _u32, _u32, _u32, _u32, _P, _P, _P, _u32, _u32, _u32, _P]),
            "fmo_quantize_q8_0": (None, [_P, _P, _u64]),
            "fmo_quantize_q4_k": (None, [_P, _P, _u64]),
            "fmo_quantize_q6_k": (None, [_P, _P, _u64]),
            "fmo_fnv1a64": (_u64, [_P, _u64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = lib

    # -- decoding
    def dequant(self, type_id: int, src: np.ndarray, n_elems: int) -> np.ndarray:
        out = np.empty(n_elems, dtype=np.float32)
        rc = self.lib.fmo_dequant_region(type_id, _ptr(np.ascontiguousarray(src)), _ptr(out), n_elems)
        if rc:
            raise RuntimeError(f"oracle dequant failed: {rc}")
        return out

    # -- products
    def gemv_f64(self, type_id: int, w: np.ndarray, x: np.ndarray, out_dim: int, in_dim: int) -> np.ndarray:
        x2 = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_dim)
        y = np.empty((x2.shape[0], out_dim), dtype=np.float64)
        rc = self.lib.fmo_gemv_quant_f64(type_id, _ptr(np.ascontiguousarray(w)), _ptr(x2), _ptr(y),
                                         x2.shape[0], out_dim, in_dim)
        if rc:
            raise RuntimeError(f"oracle gemv failed: {rc}")
        return y

    def gemv_fused_scalar(self, type_id, w, x, out_dim, in_dim) -> np.ndarray:
        x2 = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_dim)
        y = np.empty((x2.shape[0], out_dim), dtype=np.float32)
        rc = self.lib.fmo_gemv_quant_fused_scalar(type_id, _ptr(np.ascontiguousarray(w)), _ptr(x2), _ptr(y),
                                                  x2.shape[0], out_dim, in_dim)
        if rc:
            raise RuntimeError(f"oracle gemv failed: {rc}")
        return y

    def gemv_f32(self, w: np.ndarray, x: np.ndarray, out_dim: int, in_dim: int, order: str) -> np.ndarray:
        y = np.empty(out_dim, dtype=np.float32)
        fn = self.lib.fmo_gemv_f32_scalar if order == "scalar" else self.lib.fmo_gemv_f32_avx2_order
        fn(_ptr(np.ascontiguousarray(w, dtype=np.float32)), _ptr(np.ascontiguousarray(x, dtype=np.float32)),
           _ptr(y), out_dim, in_dim)
        return y

    # -- router
    def route(self, logits: np.ndarray, top_k: int, normalise=True, epsilon=EPS, scale=1.0):
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = lg.shape
        ids = np.empty((T, top_k), dtype=np.uint32)
        w = np.empty((T, top_k), dtype=np.float32)
        probs = np.empty((T, E), dtype=np.float32)
        rc = self.lib.fmo_route(_ptr(lg), T, E, top_k, 1 if normalise else 0, epsilon, scale,
                                _ptr(ids), _ptr(w), _ptr(probs))
        return rc, ids, w, probs

    def route_ex(self, logits, top_k, gating=0, logit_bias=None, selection_bias=None, groups=1, groups_used=1,
                 normalise=True, epsilon_additive=False, epsilon=EPS, scale=1.0):
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = lg.shape
        ids = np.empty((T, top_k), dtype=np.uint32)
        w = np.empty((T, top_k), dtype=np.float32)
        probs = np.empty((T, E), dtype=np.float32)
        lb = None if logit_bias is None else np.ascontiguousarray(logit_bias, dtype=np.float32)
        sb = None if selection_bias is None else np.ascontiguousarray(selection_bias, dtype=np.float32)
        rc = self.lib.fmo_route_ex(_ptr(lg), T, E, top_k, gating, _ptr(lb) if lb is not None else None,
                                   _ptr(sb) if sb is not None else None, groups, groups_used,
                                   1 if normalise else 0, 1 if epsilon_additive else 0, epsilon, scale,
                                   _ptr(ids), _ptr(w), _ptr(probs))
        return rc, ids, w, probs

    def group(self, ids: np.ndarray, experts: int):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        T, k = ids.shape
        counts = np.empty(experts, dtype=np.uint32)
        offsets = np.empty(experts + 1, dtype=np.uint32)
        pairs = np.empty(T * k, dtype=np.uint32)
        slot_of = np.empty(T * k, dtype=np.uint32)
        rc = self.lib.fmo_group_by_expert(_ptr(ids), T, k, experts, _ptr(counts), _ptr(offsets),
                                          _ptr(pairs), _ptr(slot_of))
        if rc:
            raise RuntimeError(f"oracle grouping failed: {rc}")
        return counts, offsets, pairs, slot_of

    def swiglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        return np.array([self.lib.fmo_swiglu(float(g), float(u)) for g, u in zip(gate.ravel(), up.ravel())],
                        dtype=np.float32).reshape(gate.shape)

    def moe_block(self, x, ids, weights, slots, d, ffn, gate_type, up_type=None, down_type=None):
        up_type = gate_type if up_type is None else up_type
        down_type = gate_type if down_type is None else down_type
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        k = ids.shape[1]
        bufs = [np.ascontiguousarray(s) for s in slots]
        base = (C.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
        y = np.empty((T, d), dtype=np.float32)
        rc = self.lib.fmo_moe_block(_ptr(x), T, d, ffn, k, _ptr(np.ascontiguousarray(ids, dtype=np.uint32)),
                                    _ptr(np.ascontiguousarray(weights, dtype=np.float32)), base,
                                    gate_type, up_type, down_type, _ptr(y))
        if rc:
            raise RuntimeError(f"oracle MoE block failed: {rc}")
        return y

    # -- encoders
    def quantize(self, type_id: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        if type_id == TYPE_F32:
            return x.view(np.uint8).copy()
        bs, bb = GEOMETRY[type_id]
        out = np.empty(x.size // bs * bb, dtype=np.uint8)
        fn = {TYPE_Q8_0: self.lib.fmo_quantize_q8_0, TYPE_Q4_K: self.lib.fmo_quantize_q4_k,
              TYPE_Q6_K: self.lib.fmo_quantize_q6_k}[type_id]
        fn(_ptr(x), _ptr(out), x.size)
        return out

    def fnv1a64(self, data: np.ndarray) -> int:
        d = np.ascontiguousarray(data).view(np.uint8)
        return int(self.lib.fmo_fnv1a64(_ptr(d), d.size))

    @staticmethod
    def coalesce_extents(extents, max_gap: int):
        """coalesce_extents (src/io.cpp:46-78): extents (offset, size) sorted by
        offset then size; one starting at most max_gap bytes past the current
        group's end joins it.  Returns [(offset, end, [extent indices])];
        raises ValueError for a zero-sized or overflowing extent."""
        order = sorted(range(len(extents)), key=lambda i: (extents[i][0], extents[i][1], i))
        groups = []
        for i in order:
            off, size = extents[i]
            if size == 0 or off > (1 << 64) - 1 - size:
                raise ValueError("invalid extent")
            end = off + size
            if groups and max_gap <= (1 << 64) - 1 - groups[-1][1] and off <= groups[-1][1] + max_gap:
                groups[-1][1] = max(groups[-1][1], end)
                groups[-1][2].append(i)
                continue
            groups.append([off, end, [i]])
        return [(g[0], g[1], g[2]) for g in groups]


class Reference:
    """The reference's own code, compiled from source (oracle/_ref/libfmref.so)."""

    def __init__(self, path: Path = REF_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} is missing (build with `make -C oracle ref`)")
        lib = C.CDLL(str(path))
        sig = {
            "fmr_last_error": (C.c_char_p, []),
            "fmr_dequant_block": (_i, [_u32, _P, _P]),
            "fmr_dequant_region": (_i, [_u32, _P, _P, _u64]),
            "fmr_resolved_isa": (C.c_char_p, []),
            "fmr_gemv_quant": (_i, [_u32, _P, _P, _P, _u32, _u32, _u32, _i]),
            "fmr_gemv_f32": (_i, [_P, _P, _P, _u32, _u32, _i]),
            "fmr_route": (_i, [_P, _u32, _u32, _u32, _P, _P, _P]),
            "fmr_swiglu": (_f, [_f, _f]),
            "fmr_fnv1a64": (_u64, [_P, _u64]),
            "fmr_coalesce_extents": (_i, [_P, _u32, _u64, _P, _P, _P, _P]),
            "fmr_file_identity": (_i, [C.c_char_p, _P]),
            "fmr_load_records_cpu": (C.c_int64, [C.c_char_p, _i, _u64, _P, _u32, _u32, _P, _P]),
            "fmr_moe_block": (_i, [_u32, _P, _u64, _u64, _P, _u32, _u32, _u32, _u32, _P, _P, _P, _u32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        self.lib = lib

    def isa(self) -> str:
        return self.lib.fmr_resolved_isa().decode()

    def coalesce_extents(self, extents, max_gap: int):
        """The reference's own coalesce_extents: [(offset, end, [extent indices])]."""
        n = len(extents)
        ext = np.array(extents, dtype=np.uint64).reshape(n, 2) if n else np.zeros((0, 2), np.uint64)
        go, ge = np.zeros(max(n, 1), np.uint64), np.zeros(max(n, 1), np.uint64)
        gof, ng = np.zeros(max(n, 1), np.uint32), np.zeros(1, np.uint32)
        rc = self.lib.fmr_coalesce_extents(_ptr(ext), n, max_gap, _ptr(go), _ptr(ge), _ptr(gof), _ptr(ng))
        if rc:
            raise ValueError(self.lib.fmr_last_error().decode())
        return [(int(go[j]), int(ge[j]), [i for i in range(n) if gof[i] == j]) for j in range(int(ng[0]))]

    def file_identity(self, path) -> tuple:
        """current_identity (src/common.cpp:79-119): (size, dev, ino, mtime_ns, ctime_ns, content_probe)."""
        out = np.zeros(6, np.uint64)
        rc = self.lib.fmr_file_identity(str(path).encode(), _ptr(out))
        if rc:
            raise RuntimeError(self.lib.fmr_last_error().decode())
        v = [int(x) for x in out]
        to_i64 = lambda u: u - (1 << 64) if u >= 1 << 63 else u
        return (v[0], v[1], v[2], to_i64(v[3]), to_i64(v[4]), v[5])

    def load_records_cpu(self, path, reader_mode: int, coalesce_gap: int, extents: np.ndarray,
                         checksums: np.ndarray, slot: np.ndarray) -> int:
        """load_slot's data path on the reference's CPU backend for records of
        extents [n_records, n_ext, 2] (see fmr_load_records_cpu)."""
        ext = np.ascontiguousarray(extents, dtype=np.uint64)
        ck = np.ascontiguousarray(checksums, dtype=np.uint64)
        rc = self.lib.fmr_load_records_cpu(str(path).encode(), reader_mode, coalesce_gap, _ptr(ext),
                                           ext.shape[1], ext.shape[0], _ptr(ck), _ptr(slot))
        if rc < 0:
            raise RuntimeError(self.lib.fmr_last_error().decode())
        return int(rc)

    def dequant(self, type_id, src, n_elems) -> np.ndarray:
        out = np.empty(n_elems, dtype=np.float32)
        rc = self.lib.fmr_dequant_region(type_id, _ptr(np.ascontiguousarray(src)), _ptr(out), n_elems)
        if rc:
            raise RuntimeError(self.lib.fmr_last_error().decode())
        return out

    def gemv_quant(self, type_id, w, x, out_dim, in_dim, threads=1, scalar=False) -> np.ndarray:
        y = np.empty(out_dim, dtype=np.float32)
        rc = self.lib.fmr_gemv_quant(type_id, _ptr(np.ascontiguousarray(w)),
                                     _ptr(np.ascontiguousarray(x, dtype=np.float32)), _ptr(y), out_dim,
                                     in_dim, threads, 1 if scalar else 0)
        if rc:
            raise RuntimeError(self.lib.fmr_last_error().decode())
        return y

    def gemv_f32(self, w, x, out_dim, in_dim, scalar=False) -> np.ndarray:
        y = np.empty(out_dim, dtype=np.float32)
        self.lib.fmr_gemv_f32(_ptr(np.ascontiguousarray(w, dtype=np.float32)),
                              _ptr(np.ascontiguousarray(x, dtype=np.float32)), _ptr(y), out_dim, in_dim,
                              1 if scalar else 0)
        return y

    def route(self, logits, top_k):
        lg = np.ascontiguousarray(logits, dtype=np.float32)
        T, E = lg.shape
        ids = np.empty((T, top_k), dtype=np.uint32)
        w = np.empty((T, top_k), dtype=np.float32)
        probs = np.empty((T, E), dtype=np.float32)
        rc = self.lib.fmr_route(_ptr(lg), T, E, top_k, _ptr(ids), _ptr(w), _ptr(probs))
        return rc, ids, w, probs

    def moe_block(self, type_id, slots, up_offset, down_offset, x, ids, weights, d, ffn, threads=1):
        """engine.cpp:1711-1772 over the reference's gemv_quant; ``slots`` are host uint8 arrays."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, k = ids.shape
        base = (C.c_void_p * len(slots))(*[s.ctypes.data for s in slots])
        y = np.empty((T, d), dtype=np.float32)
        rc = self.lib.fmr_moe_block(type_id, base, up_offset, down_offset, _ptr(x), T, d, ffn, k,
                                    _ptr(np.ascontiguousarray(ids, dtype=np.uint32)),
                                    _ptr(np.ascontiguousarray(weights, dtype=np.float32)), _ptr(y), threads)
        if rc:
            raise RuntimeError(self.lib.fmr_last_error().decode())
        return y

    def swiglu(self, gate, up) -> np.ndarray:
        return np.array([self.lib.fmr_swiglu(float(g), float(u)) for g, u in zip(gate.ravel(), up.ravel())],
                        dtype=np.float32).reshape(gate.shape)


def reference_available() -> bool:
    return REF_SO.exists()


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Rounds float32 values to bfloat16 (nearest even), returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)
