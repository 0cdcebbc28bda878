"""Cold -> warm loads, host side (no GPU): the oracle's FNV-1a against the
golden vectors made by the reference, and the loader's host logic (extent
coalescing, source identity) through the C ABI against the oracle restatement
and the reference's own code (src/io.cpp:46-78, src/common.cpp:79-119)."""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle.oracle import Reference, reference_available

from freemoe_b200 import _lib as L
from freemoe_b200 import coldtier


def seeded(seed: int, size: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, size, dtype=np.uint8)


@pytest.fixture(scope="module")
def fnv_golden():
    return json.loads((GOLDEN / "fnv_vectors.json").read_text())


def test_oracle_fnv_matches_reference_golden(oracle, fnv_golden):
    for item in fnv_golden["strings"]:
        a = np.frombuffer(item["text"].encode(), dtype=np.uint8).copy()
        assert oracle.fnv1a64(a) == int(item["fnv1a64"], 16), item["text"]
    for item in fnv_golden["seeded"]:
        assert oracle.fnv1a64(seeded(item["seed"], item["size"])) == int(item["fnv1a64"], 16), item["size"]


COALESCE_CASES = [
    ([(0, 10)], 0),
    ([(0, 10), (10, 5)], 0),                   # adjacent, gap 0
    ([(0, 10), (11, 5)], 0),                   # one byte apart, gap 0
    ([(0, 10), (11, 5)], 1),                   # within the gap
    ([(100, 10), (0, 10), (50, 10)], 40),      # unsorted input
    ([(0, 100), (20, 10), (200, 8)], 4096),    # contained extent
    ([(5, 10), (5, 3), (5, 10)], 0),           # equal offsets: ordered by size
    ([(4096 * 7 + 3, 144 * 16), (1 << 33, 210), (4096 * 7 + 3 + 144 * 16, 99)], 4096),
]


@pytest.mark.parametrize("extents,gap", COALESCE_CASES)
def test_coalesce_matches_oracle_restatement(oracle, extents, gap):
    got = coldtier.coalesce_extents(extents, gap)
    want = oracle.coalesce_extents(extents, gap)
    assert [(o, e, sorted(m)) for o, e, m in got] == [(o, e, sorted(m)) for o, e, m in want]


def test_coalesce_random_matches_oracle(oracle):
    rng = np.random.default_rng(5)
    for _ in range(200):
        n = int(rng.integers(1, 12))
        ext = [(int(rng.integers(0, 1 << 20)), int(rng.integers(1, 1 << 14))) for _ in range(n)]
        gap = int(rng.choice([0, 1, 512, 4096, 1 << 16]))
        got = coldtier.coalesce_extents(ext, gap)
        want = oracle.coalesce_extents(ext, gap)
        assert [(o, e, sorted(m)) for o, e, m in got] == [(o, e, sorted(m)) for o, e, m in want]


@pytest.mark.skipif(not reference_available(), reason="compiled reference shim not built here")
def test_coalesce_oracle_pinned_to_reference(oracle):
    ref = Reference()
    rng = np.random.default_rng(6)
    cases = [c for c, _ in COALESCE_CASES]
    for _ in range(100):
        n = int(rng.integers(1, 10))
        cases.append([(int(rng.integers(0, 1 << 16)), int(rng.integers(1, 1 << 12))) for _ in range(n)])
    for ext in cases:
        for gap in (0, 1, 4096):
            want = ref.coalesce_extents(ext, gap)
            got = oracle.coalesce_extents(ext, gap)
            assert [(o, e) for o, e, _ in got] == [(o, e) for o, e, _ in want]
            # members of a group: the same set (the reference's sort is not stable)
            assert [sorted(m) for *_, m in got] == [sorted(m) for *_, m in want]


def test_coalesce_rejects_invalid_extents(oracle):
    for ext in ([(0, 0)], [(10, 5), (3, 0)], [((1 << 64) - 4, 8)]):
        with pytest.raises(L.FmError) as e:
            coldtier.coalesce_extents(ext, 0)
        assert e.value.code == 26
        with pytest.raises(ValueError):
            oracle.coalesce_extents(ext, 0)


@pytest.mark.skipif(not reference_available(), reason="compiled reference shim not built here")
@pytest.mark.parametrize("size", [0, 1, 63, 64, 65, 127, 128, 129, 10000])
def test_file_identity_matches_reference(tmp_path, size):
    p = tmp_path / f"model_{size}.gguf"
    p.write_bytes(seeded(77 + size, size).tobytes())
    assert coldtier.file_identity(p) == Reference().file_identity(p)


def test_file_identity_sees_an_edit(tmp_path):
    p = tmp_path / "model.gguf"
    data = seeded(3, 4096)
    p.write_bytes(data.tobytes())
    st = os.stat(p)
    before = coldtier.file_identity(p)
    data[2048 - 32] ^= 1  # inside the middle probe window; same size, same times
    p.write_bytes(data.tobytes())
    os.utime(p, ns=(st.st_atime_ns, st.st_mtime_ns))
    after = coldtier.file_identity(p)
    assert before[0] == after[0] and before[5] != after[5]


def test_file_identity_missing_file(tmp_path):
    with pytest.raises(L.FmError) as e:
        coldtier.file_identity(tmp_path / "absent.gguf")
    assert e.value.code == 11  # IO_ERROR
