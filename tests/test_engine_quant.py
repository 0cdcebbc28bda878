"""FreeMoe's own engine fixtures through the reference's unmodified fm::Engine
on the CUDA backend (oracle/_ref/fm_engine; engine_hooks.cpp routes the
quantised GEMVs and the slot read-back to the device).

* test_quant_model_parity / test_quant_expert_mixed_types
  (tests/unit/tests.cpp:1424-1544): quant-moe-{q8_0,q4_k,q6_k} and
  quant-expert-{separate,fused} give the same greedy tokens as their F32
  twins, and prefill logits within 1e-4 of them; on the GPU every expert GEMV
  is an operation of the CUDA backend (none labelled "cpu-quant").
* test_moe_readers_and_cache_sizes (tests/unit/tests.cpp:958-1046): moe-fm's
  20 prompts within the reference's logit tolerance, identical greedy tokens
  and routing, with one expert slot and with every expert resident.
* test_residency_manager (tests/unit/tests.cpp:794-882): the residency
  manager's slot states and typed faults over the CUDA backend.

The fixtures are the reference's files, copied by tests/golden/make_engine_fixtures.py
with the F32 twins' outputs recorded there.
"""
from __future__ import annotations

import hashlib
import json
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT

ENGINE = ROOT / "oracle" / "_ref" / "fm_engine"
FIX = ROOT / "tests" / "golden" / "engine"
GOLD = json.loads((FIX / "goldens.json").read_text())
LOGIT_TOL = 1e-4  # tests/unit/tests.cpp:1455 and :1506


def engine(*args, timeout=900):
    assert ENGINE.exists(), f"{ENGINE} is missing (built by __graft_entry__.build())"
    p = subprocess.run([str(ENGINE), *map(str, args)], capture_output=True, text=True, timeout=timeout, cwd=ROOT)
    if p.returncode:
        raise AssertionError(f"fm_engine {args[0]} failed ({p.returncode}): {p.stderr[-2000:]}")
    return p.stdout


def run(model, backend, prompt, tokens, slots, tmp_path):
    out = tmp_path / f"{model.stem}-{backend}-{slots}.bin"
    engine("run", model, backend, prompt.encode().hex(), tokens, slots, 0, out)
    b = out.read_bytes()
    n = struct.unpack_from("<I", b, 0)[0]
    ids = np.frombuffer(b, "<i4", n, 4)
    pos = 4 + 4 * n
    m = struct.unpack_from("<I", b, pos)[0]
    logits = np.frombuffer(b, "<f4", m, pos + 4)
    pos += 4 + 4 * m
    r = struct.unpack_from("<I", b, pos)[0]
    pos += 4 + 4 * r
    k = struct.unpack_from("<I", b, pos)[0]
    metrics = json.loads(b[pos + 4:pos + 4 + k].decode())
    return ids, logits, metrics


def test_fixture_files_match_their_manifest():
    for name, digest in GOLD["manifest"].items():
        assert hashlib.sha256((FIX / name).read_bytes()).hexdigest() == digest, name


@pytest.mark.parametrize("variant", sorted(GOLD["quant"]))
def test_quant_fixture_on_cpu_backend_matches_f32_twin(variant, tmp_path):
    # the reference's own test on its CPU backend: pins the fixture and the harness
    g = GOLD["quant"][variant]
    ids, logits, _ = run(FIX / f"{variant}.gguf", "cpu", g["prompt"], g["tokens"], 0, tmp_path)
    assert list(ids) == g["ids"]
    assert float(np.max(np.abs(logits.astype(np.float64) - np.array(g["logits"])))) <= LOGIT_TOL


def test_residency_faults_on_cpu_backend():
    checks = json.loads(engine("residency", FIX / "moe-fm.gguf", "cpu"))["checks"]
    assert len(checks) >= 25 and all(ok for _, ok in checks), [c for c in checks if not c[1]]


@pytest.mark.gpu
@pytest.mark.parametrize("slots", [0, 1])
@pytest.mark.parametrize("variant", sorted(GOLD["quant"]))
def test_quant_fixture_on_gpu_backend(variant, slots, tmp_path):
    g = GOLD["quant"][variant]
    model = FIX / f"{variant}.gguf"
    ids, logits, metrics = run(model, "gpu", g["prompt"], g["tokens"], slots, tmp_path)
    assert metrics["name"] == "cuda-sm100a"
    # test_quant_model_parity's bars against the F32 twin
    assert list(ids) == g["ids"], "greedy tokens differ from the F32 reference"
    assert float(np.max(np.abs(logits.astype(np.float64) - np.array(g["logits"])))) <= LOGIT_TOL
    # and against the same quantised model on the CPU backend
    ids_c, logits_c, _ = run(model, "cpu", g["prompt"], g["tokens"], slots, tmp_path)
    assert list(ids) == list(ids_c)
    assert float(np.max(np.abs(logits - logits_c))) <= LOGIT_TOL
    ops = metrics["operations"]
    expert = [o for o in ops if o["name"].startswith(("expert_gate", "expert_up", "expert_down"))]
    assert expert and all(o["backend"] == "cuda-sm100a" for o in expert)
    assert not any(o["backend"] in ("cpu-quant", "cpu-fallback") for o in ops)
    assert metrics["allocations"]["by_tag"]["expert_cache"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("slots", [1, 16])
def test_moe_fixture_20_prompts_on_gpu_backend(slots):
    d = json.loads(engine("compare", FIX / "moe-fm.gguf", "gpu", FIX / "reference", 20, 16, slots))
    c = d["comparison"]
    assert c["prompts"] == 20
    assert c["prompts_within_tolerance"] == 20 and c["prompts_token_match"] == 20
    assert c["prompts_routing_match"] == 20
    assert d["ops"]["backend"] == "cuda-sm100a"
    assert d["ops"]["expert_gemvs"] > 0 and d["ops"]["expert_gemvs_on_backend"] == d["ops"]["expert_gemvs"]
    cache = d["residency"]["cache"]
    assert cache["checksum_failures"] == 0 and cache["checksum_checks"] > 0
    if slots == 1:
        assert len(d["residency"]["slots"]) == 1
        assert cache["evictions"] > 0  # every expert went through the one slot, read back from HBM each time


@pytest.mark.gpu
def test_residency_faults_on_gpu_backend():
    checks = json.loads(engine("residency", FIX / "moe-fm.gguf", "gpu"))["checks"]
    names = [n for n, _ in checks]
    assert any(n.startswith("CUDA backend:") for n in names)
    assert all(ok for _, ok in checks), [c for c in checks if not c[1]]
