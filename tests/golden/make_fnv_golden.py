"""Writes tests/golden/fnv_vectors.json: FNV-1a 64 (include/fm/common.hpp:73-81)
computed by the reference's own fm::fnv1a64, compiled from the reference
sources into oracle/_ref/libfmref.so (``make -C oracle ref``).

Inputs are a few literal strings and seeded byte runs
(``numpy.random.default_rng(seed).integers(0, 256, size, dtype=uint8)``)
whose sizes sit around the 512-byte chunks and 256-thread CTAs of the device
kernel.  Run from the repository root: ``python tests/golden/make_fnv_golden.py``.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle.oracle import Reference, _ptr  # noqa: E402

STRINGS = ["", "a", "foobar", "FreeMoe expert record"]
SIZES = [1, 2, 3, 15, 16, 17, 255, 256, 511, 512, 513, 1023, 1024, 4095, 4097, 131072, 131072 + 512 + 7,
         (1 << 20) + 7]


def seeded(seed: int, size: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, size, dtype=np.uint8)


def main() -> None:
    ref = Reference()
    fnv = lambda a: int(ref.lib.fmr_fnv1a64(_ptr(a), a.size))
    out = {"strings": [], "seeded": []}
    for s in STRINGS:
        a = np.frombuffer(s.encode(), dtype=np.uint8).copy()
        out["strings"].append({"text": s, "fnv1a64": f"{fnv(a):016x}"})
    for i, n in enumerate(SIZES):
        out["seeded"].append({"seed": 1000 + i, "size": n, "fnv1a64": f"{fnv(seeded(1000 + i, n)):016x}"})
    path = ROOT / "tests" / "golden" / "fnv_vectors.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print(path)


if __name__ == "__main__":
    main()
