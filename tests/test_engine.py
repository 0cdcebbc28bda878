"""The reference's own, unmodified fm::Engine driving the CUDA backend.

oracle/_ref/fm_engine links the reference sources (compiled from the reference
tree by oracle/Makefile) with freemoe_b200/backend/cuda_backend.cpp; calls to
fm::Backend::create are routed to CudaBackend for --backend gpu.  The
freemoe-tiny-v1 fixture (d 64, 2 layers, 4 heads x 16, 4 experts ffn 128,
top-2, vocab 258, F32 N(0, 0.02) from seed 0) is run with a 128-byte random
prompt and 32 greedy tokens on both backends; greedy ids, prefill logits and
routing must be identical (the device matvec reproduces the CPU backend's
summation order, so the whole forward pass is bit-identical).
"""
from __future__ import annotations

import json
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT

ENGINE = ROOT / "oracle" / "_ref" / "fm_engine"


def run_engine(*args, check=True):
    p = subprocess.run([str(ENGINE), *map(str, args)], capture_output=True, text=True, timeout=600)
    if check and p.returncode:
        raise AssertionError(f"fm_engine {args[0]} failed ({p.returncode}): {p.stderr}")
    return p


def read_result(path):
    b = path.read_bytes()
    pos = 0

    def take(fmt_char, n):
        nonlocal pos
        arr = np.frombuffer(b, dtype=np.dtype(fmt_char), count=n, offset=pos)
        pos += 4 * n
        return arr

    (n,) = struct.unpack_from("<I", b, pos)
    pos += 4
    ids = take("<i4", n)
    (n,) = struct.unpack_from("<I", b, pos)
    pos += 4
    logits = take("<f4", n)
    (n,) = struct.unpack_from("<I", b, pos)
    pos += 4
    routing = take("<u4", n)
    (n,) = struct.unpack_from("<I", b, pos)
    pos += 4
    metrics = json.loads(b[pos:pos + n].decode())
    return ids, logits, routing, metrics


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    assert ENGINE.exists(), f"{ENGINE} is missing (built by __graft_entry__.build())"
    path = tmp_path_factory.mktemp("tiny") / "freemoe-tiny-v1.gguf"
    run_engine("write-tiny", path, 0)
    prompt = np.random.default_rng(0).integers(0, 256, size=128, dtype=np.uint8).tobytes().hex()
    return path, prompt


def test_tiny_fixture_runs_on_cpu_backend(tiny, tmp_path):
    path, prompt = tiny
    out = tmp_path / "cpu.bin"
    run_engine("run", path, "cpu", prompt, 32, 0, 0, out)
    ids, logits, routing, metrics = read_result(out)
    assert ids.size == 32 and logits.size == 258 and routing.size > 0
    assert metrics["name"] == "cpu"


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU failure path")
def test_gpu_backend_fails_loudly_without_a_device(tiny, tmp_path):
    path, prompt = tiny
    p = run_engine("run", path, "gpu", prompt, 4, 0, 0, tmp_path / "gpu.bin", check=False)
    assert p.returncode == 23, p.stderr  # DEVICE_LOSS: no CPU fallback
    assert "no CUDA device" in p.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("scalar,slots", [(0, 0), (1, 0), (0, 1)])
def test_tiny_fixture_identical_on_gpu(tiny, tmp_path, scalar, slots):
    path, prompt = tiny
    cpu, gpu = tmp_path / "cpu.bin", tmp_path / "gpu.bin"
    run_engine("run", path, "cpu", prompt, 32, slots, scalar, cpu)
    run_engine("run", path, "gpu", prompt, 32, slots, scalar, gpu)
    ids_c, lg_c, rt_c, m_c = read_result(cpu)
    ids_g, lg_g, rt_g, m_g = read_result(gpu)
    assert m_g["name"] == "cuda-sm100a"
    assert list(ids_g) == list(ids_c), "greedy tokens differ"
    assert np.array_equal(lg_g.view(np.uint32), lg_c.view(np.uint32)), "prefill logits differ"
    assert np.array_equal(rt_g, rt_c), "routing differs"
    ops = m_g["operations"]
    assert any(o["backend"] == "cuda-sm100a" and o["name"].startswith("expert_") for o in ops)
    assert not any(o["backend"] in ("cpu-fallback",) for o in ops)
    assert m_g["allocations"]["by_tag"]["expert_cache"] > 0
