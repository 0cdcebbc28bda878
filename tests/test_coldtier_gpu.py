"""Cold -> warm expert loads on the GPU, through the C ABI.

Bars: the device FNV-1a 64 is bit-exact against the reference's fm::fnv1a64
(golden vectors made by the reference) and the oracle restatement, at every
size, alignment and chunk boundary; a loaded slot holds exactly the file bytes
of the record's extents in record order; the statistics and every error code
follow the reference's reader (src/io.cpp) and load_slot (src/residency.cpp).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN

from freemoe_b200 import _lib as L
from freemoe_b200 import coldtier

pytestmark = pytest.mark.gpu


def seeded(seed: int, size: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, size, dtype=np.uint8)


def on_gpu(a: np.ndarray, offset: int = 0) -> torch.Tensor:
    """The bytes of `a` on the device, starting `offset` bytes past a 256-byte boundary."""
    buf = torch.empty(a.size + offset + 16, dtype=torch.uint8, device="cuda")
    view = buf[offset:offset + a.size]
    if a.size:
        view.copy_(torch.from_numpy(a))
    return view


# ------------------------------------------------------------------ device FNV-1a

def test_device_fnv_golden():
    g = json.loads((GOLDEN / "fnv_vectors.json").read_text())
    for item in g["strings"]:
        a = np.frombuffer(item["text"].encode(), dtype=np.uint8).copy()
        assert coldtier.fnv1a64(on_gpu(a)) == int(item["fnv1a64"], 16), item["text"]
    for item in g["seeded"]:
        a = seeded(item["seed"], item["size"])
        for off in (0, 1, 8):
            assert coldtier.fnv1a64(on_gpu(a, off)) == int(item["fnv1a64"], 16), (item["size"], off)


@pytest.mark.parametrize("size", [512 * 256 - 1, 512 * 256, 512 * 256 + 1, 512 * 256 * 3 + 77,
                                  (16 << 20) + 3, (64 << 20) + 1])
@pytest.mark.parametrize("off", [0, 3])
def test_device_fnv_matches_oracle(oracle, size, off):
    a = seeded(size + off, size)
    assert coldtier.fnv1a64(on_gpu(a, off)) == oracle.fnv1a64(a)


def test_device_fnv_constant_inputs(oracle):
    # long runs of one byte value keep the low-byte state on short cycles
    for v in (0, 1, 0x25, 0xFF):
        a = np.full(3 * 512 * 256 + 5, v, dtype=np.uint8)
        assert coldtier.fnv1a64(on_gpu(a)) == oracle.fnv1a64(a), v


def test_device_fnv_ignores_stale_workspace(oracle):
    # the workspace is scratch: whatever it holds from earlier use must not matter
    lib = L.load()
    a = seeded(71, 512 * 256 * 2 + 9)
    src = on_gpu(a)
    ws = torch.full((int(lib.fmcuda_fnv1a64_workspace_bytes(a.size)),), 0xFF, dtype=torch.uint8, device="cuda")
    out = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    for _ in range(2):
        assert lib.fmcuda_fnv1a64(src.data_ptr(), a.size, out.data_ptr(), ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream().cuda_stream) == 0
        assert int(out.cpu().item()) & ((1 << 64) - 1) == oracle.fnv1a64(a)


def test_device_fnv_rejects_bad_arguments():
    lib = L.load()
    out = torch.zeros(2, dtype=torch.int64, device="cuda")
    src = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    ws = torch.empty(int(lib.fmcuda_fnv1a64_workspace_bytes(1024)), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    # result word not 8-byte aligned
    assert lib.fmcuda_fnv1a64(src.data_ptr(), 1024, out.data_ptr() + 4, ws.data_ptr(), ws.numel(), st) == 26
    # workspace too small
    assert lib.fmcuda_fnv1a64(src.data_ptr(), 1024, out.data_ptr(), ws.data_ptr(), 1, st) == 26


# ------------------------------------------------------------------ record loads

MODEL_BYTES = 24 << 20


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    d = tmp_path_factory.mktemp("coldtier")
    data = seeded(9, MODEL_BYTES)
    p = d / "experts.gguf"
    p.write_bytes(data.tobytes())
    return p, data


def record_extents(seed: int):
    """Three extents like one expert's gate, up and down slices of three stacked
    tensors: unaligned offsets, Q4_K / Q6_K sized, not in file order."""
    rng = np.random.default_rng(seed)
    sizes = [144 * 4096, 144 * 4096, 210 * 2048 + 17]
    starts = [int(rng.integers(0, MODEL_BYTES // 3 - s)) + j * (MODEL_BYTES // 3) for j, s in enumerate(sizes)]
    ext = list(zip(starts, sizes))
    return [ext[1], ext[0], ext[2]]


def payload_of(data: np.ndarray, extents) -> np.ndarray:
    return np.concatenate([data[o:o + s] for o, s in extents])


def check_load(oracle, loader, data, extents, slot_bytes=None, **kw):
    payload = payload_of(data, extents)
    slot = torch.full((slot_bytes or payload.size + 4096,), 0xA5, dtype=torch.uint8, device="cuda")
    stats = loader.read_record_into(extents, slot, **kw)
    torch.cuda.synchronize()
    got = slot.cpu().numpy()
    assert np.array_equal(got[:payload.size], payload)
    assert np.all(got[payload.size:] == 0xA5)  # nothing past the record
    assert stats.payload_bytes == payload.size
    assert stats.checksum == oracle.fnv1a64(payload)
    groups = oracle.coalesce_extents(extents, 4096)
    assert stats.read_requests == len(groups)
    assert stats.coalesced_requests == sum(len(m) - 1 for *_, m in groups)
    return stats, groups


@pytest.mark.parametrize("chunk,depth,threads", [(1 << 16, 2, 1), (1 << 16, 3, 4), (1 << 20, 4, 8), (8 << 20, 4, 4),
                                                 (8 << 20, 2, 32)])
def test_buffered_load(oracle, model_file, chunk, depth, threads):
    p, data = model_file
    with coldtier.RecordLoader(p, "buffered", chunk_bytes=chunk, ring_depth=depth, reader_threads=threads) as ld:
        for seed in range(3):  # the ring carries over between records
            stats, groups = check_load(oracle, ld, data, record_extents(seed))
            assert stats.physical_bytes == sum(e - o for o, e, _ in groups)
            assert stats.direct_fallbacks == 0


@pytest.mark.parametrize("chunk,threads", [(1 << 16, 1), (1 << 16, 4), (4 << 20, 4)])
def test_direct_load(oracle, model_file, chunk, threads):
    p, data = model_file
    with coldtier.RecordLoader(p, "direct", chunk_bytes=chunk, ring_depth=3, reader_threads=threads) as ld:
        for seed in range(3):
            stats, groups = check_load(oracle, ld, data, record_extents(10 + seed))
            # O_DIRECT reads whole aligned blocks; a file system without it falls back per group
            assert stats.direct_fallbacks in (0, len(groups))
            if stats.direct_fallbacks == 0:
                assert stats.physical_bytes >= stats.payload_bytes


def test_forced_direct_fallback(oracle, model_file):
    p, data = model_file
    with coldtier.RecordLoader(p, "direct", force_direct_fallback=True) as ld:
        stats, groups = check_load(oracle, ld, data, record_extents(20))
        assert stats.direct_fallbacks == len(groups)


def test_coalesced_extents(oracle, model_file):
    p, data = model_file
    base = 3 * 4096 + 5
    ext = [(base + 2000 + 100, 3000), (base, 2000), (base + 2000 + 100 + 3000 + 4096, 512), (base + (9 << 20), 999)]
    with coldtier.RecordLoader(p, "buffered", chunk_bytes=1 << 16) as ld:
        stats, groups = check_load(oracle, ld, data, ext)
    assert len(groups) == 2 and stats.coalesced_requests == 2


def test_tail_of_file_and_tiny_records(oracle, model_file):
    p, data = model_file
    with coldtier.RecordLoader(p, "direct", chunk_bytes=1 << 16, ring_depth=2) as ld:
        check_load(oracle, ld, data, [(MODEL_BYTES - 1, 1)])
        check_load(oracle, ld, data, [(MODEL_BYTES - 70000, 70000), (7, 1)])
        check_load(oracle, ld, data, [(0, 1)])


def test_checksum_known(oracle, model_file):
    p, data = model_file
    ext = record_extents(30)
    good = oracle.fnv1a64(payload_of(data, ext))
    with coldtier.RecordLoader(p, "buffered") as ld:
        check_load(oracle, ld, data, ext, checksum=good)
        slot = torch.empty(8 << 20, dtype=torch.uint8, device="cuda")
        with pytest.raises(L.FmError) as e:
            ld.read_record_into(ext, slot, checksum=good ^ 1)
        assert e.value.code == 17  # EXPERT_CHECKSUM_MISMATCH


def test_read_past_end_of_file_moves_nothing(model_file):
    p, _ = model_file
    slot = torch.full((1 << 20,), 0x5A, dtype=torch.uint8, device="cuda")
    with coldtier.RecordLoader(p, "buffered") as ld:
        with pytest.raises(L.FmError) as e:
            ld.read_record_into([(0, 4096), (MODEL_BYTES - 10, 11)], slot)
        assert e.value.code == 12  # SHORT_READ
    torch.cuda.synchronize()
    assert bool((slot == 0x5A).all())


def test_invalid_records(model_file):
    p, _ = model_file
    slot = torch.empty(4096, dtype=torch.uint8, device="cuda")
    with coldtier.RecordLoader(p, "buffered") as ld:
        for ext in ([(0, 0)], [(0, 4097)]):  # zero-sized extent; payload larger than the slot
            with pytest.raises(L.FmError) as e:
                ld.read_record_into(ext, slot)
            assert e.value.code == 26


def test_source_changed(oracle, tmp_path):
    p = tmp_path / "model.gguf"
    data = seeded(41, 1 << 20)
    p.write_bytes(data.tobytes())
    ident = coldtier.file_identity(p)
    with coldtier.RecordLoader(p, "buffered", expected_identity=ident) as ld:
        check_load(oracle, ld, data, [(100, 5000)])
        st = os.stat(p)
        data2 = data.copy()
        data2[:64] ^= 0xFF  # same size; the content probe sees the first 64 bytes
        p.write_bytes(data2.tobytes())
        os.utime(p, ns=(st.st_atime_ns, st.st_mtime_ns))
        slot = torch.empty(8192, dtype=torch.uint8, device="cuda")
        with pytest.raises(L.FmError) as e:
            ld.read_record_into([(100, 5000)], slot)
        assert e.value.code == 10  # SOURCE_CHANGED
