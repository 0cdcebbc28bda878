"""Cold -> warm expert loads: model file -> pinned ring -> HBM slot, checksummed on the device.

Host-side mirror of the reference's demand load for one expert record: the
names and arguments follow ``fm::ReadScheduler`` / ``fm::SchedulerConfig``
(include/fm/io.hpp:100-158) and ``ResidencyManager::load_slot``
(src/residency.cpp:624-724); errors are :class:`FmError` with the
reference's ``fm::ErrorCode`` (SOURCE_CHANGED, SHORT_READ, IO_ERROR,
EXPERT_CHECKSUM_MISMATCH, INVALID_ARGUMENT, FENCE_TIMEOUT ...).  Every call
goes through ``libfreemoe_b200.so``; nothing here reads or hashes payload
bytes in Python.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L


@dataclass
class LoadStats:
    payload_bytes: int
    physical_bytes: int
    read_requests: int
    coalesced_requests: int
    direct_fallbacks: int
    checksum: int
    elapsed_ms: float


def _extents(extents) -> tuple:
    arr = (L.Extent * max(len(extents), 1))()
    for i, (off, size) in enumerate(extents):
        arr[i].offset, arr[i].size = int(off), int(size)
    return arr, len(extents)


def coalesce_extents(extents, max_gap: int):
    """coalesce_extents (src/io.cpp:46-78) through the C ABI (host only):
    [(offset, end, [extent indices])]."""
    lib = L.load()
    arr, n = _extents(extents)
    go = (C.c_uint64 * max(n, 1))()
    ge = (C.c_uint64 * max(n, 1))()
    gof = (C.c_uint32 * max(n, 1))()
    ng = C.c_uint32()
    L.check(lib.fmcuda_coalesce_extents(arr, n, max_gap, go, ge, gof, C.byref(ng)))
    return [(go[j], ge[j], [i for i in range(n) if gof[i] == j]) for j in range(ng.value)]


def file_identity(path) -> tuple:
    """current_identity (src/common.cpp:79-119) through the C ABI:
    (size, dev, ino, mtime_ns, ctime_ns, content_probe)."""
    fid = L.FileIdentity()
    L.check(L.load().fmcuda_file_identity_get(str(path).encode(), C.byref(fid)))
    return (fid.size, fid.dev, fid.ino, fid.mtime_ns, fid.ctime_ns, fid.content_probe)


def fnv1a64(data: torch.Tensor, stream: torch.cuda.Stream | None = None) -> int:
    """FNV-1a 64 (include/fm/common.hpp:73-81) of a CUDA tensor's bytes, on the device."""
    if not data.is_cuda or not data.is_contiguous():
        raise L.FmError(26, "fnv1a64 takes a contiguous CUDA tensor")
    lib = L.load()
    n = data.numel() * data.element_size()
    out = torch.empty(1, dtype=torch.int64, device=data.device)
    ws = torch.empty(max(int(lib.fmcuda_fnv1a64_workspace_bytes(n)), 1), dtype=torch.uint8, device=data.device)
    st = stream or torch.cuda.current_stream(data.device)
    L.check(lib.fmcuda_fnv1a64(C.c_void_p(data.data_ptr()), n, C.c_void_p(out.data_ptr()),
                               C.c_void_p(ws.data_ptr()), ws.numel(), C.c_void_p(st.cuda_stream)))
    return int(out.cpu().item()) & ((1 << 64) - 1)


class RecordLoader:
    """A ReadScheduler for expert records whose destination is an HBM slot.

    mode: "buffered" (pread) or "direct" (O_DIRECT aligned spans, falling back
    to buffered reads per group when the file system refuses, counted in
    ``direct_fallbacks``).  ``reader_threads`` threads read chunks of
    ``chunk_bytes`` in parallel, each into its own ring of ``ring_depth``
    pinned chunks.  ``expected_identity`` is the identity the manifest
    was built against (None: the file as it is now); each load re-checks it.
    """

    def __init__(self, path, mode: str = "buffered", coalesce_gap: int = 4096, chunk_bytes: int = 4 << 20,
                 ring_depth: int = 3, reader_threads: int = 8, force_direct_fallback: bool = False,
                 expected_identity: tuple | None = None):
        self._lib = L.load()
        modes = {"buffered": L.READER_BUFFERED, "direct": L.READER_DIRECT}
        if mode not in modes:
            raise L.FmError(26, f"reader mode {mode!r}: buffered or direct")
        ident = None
        if expected_identity is not None:
            ident = L.FileIdentity(*expected_identity)
        h = C.c_void_p()
        L.check(self._lib.fmcuda_record_loader_create(str(path).encode(), modes[mode], coalesce_gap, chunk_bytes,
                                                      ring_depth, reader_threads, 1 if force_direct_fallback else 0,
                                                      C.byref(ident) if ident is not None else None, C.byref(h)))
        self._h = h
        self._ws = None

    def workspace_bytes(self, payload_bytes: int) -> int:
        return int(self._lib.fmcuda_record_load_workspace_bytes(payload_bytes))

    def read_record_into(self, extents, slot: torch.Tensor, checksum: int | None = None,
                         stream: torch.cuda.Stream | None = None, timeout_ms: int = 60000) -> LoadStats:
        """Reads the record's extents (in record order) into ``slot`` (a CUDA
        uint8 tensor), checks FNV-1a 64 of the slot against ``checksum`` when
        given, and returns the load's statistics (``checksum`` = the slot's
        FNV-1a 64)."""
        if not slot.is_cuda or not slot.is_contiguous():
            raise L.FmError(26, "the slot must be a contiguous CUDA tensor")
        arr, n = _extents(extents)
        payload = sum(int(s) for _, s in extents)
        need = self.workspace_bytes(payload)
        if self._ws is None or self._ws.numel() < need or self._ws.device != slot.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=slot.device)
        st = stream or torch.cuda.current_stream(slot.device)
        stats = L.RecordLoadStats()
        L.check(self._lib.fmcuda_record_load(self._h, arr, n, C.c_void_p(slot.data_ptr()),
                                             slot.numel() * slot.element_size(), 1 if checksum is not None else 0,
                                             (checksum or 0) & ((1 << 64) - 1), C.c_void_p(self._ws.data_ptr()),
                                             self._ws.numel(), C.c_void_p(st.cuda_stream), timeout_ms,
                                             C.byref(stats)))
        return LoadStats(stats.payload_bytes, stats.physical_bytes, stats.read_requests, stats.coalesced_requests,
                         stats.direct_fallbacks, stats.checksum, stats.elapsed_ms)

    def close(self) -> None:
        if self._h:
            self._lib.fmcuda_record_loader_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
