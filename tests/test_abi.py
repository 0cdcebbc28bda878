"""The C-ABI library loads and exports every symbol include/*.h declares (no GPU needed).

Only host-side validation paths are called here: each returns its typed error
before any CUDA call is made.
"""
from __future__ import annotations

import ctypes as C
import re

import pytest

from conftest import ROOT


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(fmcuda_\w+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    from freemoe_b200 import LIB_PATH, SIGNATURES, load

    lib = load()
    assert LIB_PATH.exists()
    decl = declared_symbols()
    assert len(decl) >= 25
    for name in decl:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    bound = {s[0] for s in SIGNATURES}
    assert set(decl) == bound, "ctypes signatures drift from the header"


def test_status_codes_match_reference_ordinals():
    from freemoe_b200._lib import ERROR_NAMES

    text = (ROOT / "include" / "freemoe_b200.h").read_text()
    for name, val in re.findall(r"FM_STATUS_(\w+) = (\d+)", text):
        assert ERROR_NAMES[int(val)] == name


def test_host_side_validation_without_gpu():
    from freemoe_b200 import load
    from freemoe_b200._lib import MoeArgs

    lib = load()
    assert lib.fmcuda_row_bytes(12, 4096) == 16 * 144
    assert lib.fmcuda_row_bytes(8, 14336) == 448 * 34
    assert lib.fmcuda_row_bytes(0, 7) == 28
    assert lib.fmcuda_row_bytes(12, 100) == 0
    p = C.c_void_p(8)
    # unknown type -> UNSUPPORTED_QUANTISATION, misaligned row -> SHAPE_MISMATCH
    assert lib.fmcuda_gemv(2, p, p, 0, p, 1, 4, 256, None) == 3
    assert lib.fmcuda_gemv(12, p, p, 0, p, 1, 4, 100, None) == 8
    assert lib.fmcuda_gemv(12, None, p, 0, p, 1, 4, 256, None) == 26
    assert lib.fmcuda_dequant(13, p, p, 256, None) == 3
    assert lib.fmcuda_dequant(12, p, p, 255, None) == 8
    # router argument checks (k > E, E = 0)
    assert lib.fmcuda_route(p, 1, 4, 5, 1, 6.1e-5, 1.0, p, p, None, None) == 26
    assert lib.fmcuda_route(p, 1, 0, 1, 1, 6.1e-5, 1.0, p, p, None, None) == 26
    assert b"top-k" in lib.fmcuda_last_error() or b"expert" in lib.fmcuda_last_error()
    # MoE workspace size is pure host arithmetic
    ws = C.c_uint64(0)
    assert lib.fmcuda_moe_workspace_bytes(4, 8, 2, 4096, 14336, C.byref(ws)) == 0
    assert ws.value > 4 * 2 * 14336 * 4
    a = MoeArgs()
    assert lib.fmcuda_moe_block(None, None, 0, None) == 26
    a.tokens, a.experts, a.top_k = 1, 8, 9
    assert lib.fmcuda_moe_block(C.byref(a), None, 0, None) == 26


@pytest.mark.parametrize("fn", ["fmcuda_malloc", "fmcuda_host_alloc"])
def test_null_output_pointer_rejected(fn):
    from freemoe_b200 import load

    assert getattr(load(), fn)(16, None) == 26
