"""Generates the committed golden fixtures for the hot path.

Run where the reference source tree is present (its location comes from
$FM_REFERENCE, with the checker's default otherwise) and the compiled reference shim (``make -C oracle``):

    python tests/golden/make_golden.py

Outputs (small, committed):
  quant_reference_hotpath.bin  the F32 / Q8_0 / Q4_K records of the reference's
                               own golden file tests/fixtures/quant_reference.bin
                               (format FMQR1: u32 type, u32 block_bytes,
                               u32 n_float, payload, expected floats), extracted
                               byte for byte.
  golden_vectors.npz           inputs and outputs of the reference's own code
                               (oracle/_ref/libfmref.so, compiled from source):
                               dequantize_tensor_region, gemv_quant (auto ISA and
                               scalar), gemv_scalar / gemv_isa, Engine::softmax +
                               Engine::topk + renormalisation, silu-gated SwiGLU.
  golden_manifest.json         sha256 of the source fixture and of the outputs.
"""
from __future__ import annotations

import hashlib
import json
import struct
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from oracle.oracle import (REF_TREE, TYPE_F32, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_0, Oracle,  # noqa: E402
                           Reference, bf16_round)

HOT_TYPES = (TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K)


def extract_quant_reference() -> tuple[bytes, str]:
    src = REF_TREE / "tests" / "fixtures" / "quant_reference.bin"
    data = src.read_bytes()
    assert data[:5] == b"FMQR1", "unexpected magic"
    pos = 12
    kept = []
    while pos < len(data):
        type_id, block_bytes, n_float = struct.unpack_from("<III", data, pos)
        end = pos + 12 + block_bytes + 4 * n_float
        if type_id in HOT_TYPES:
            kept.append(data[pos:end])
        pos = end
    out = data[:8] + struct.pack("<I", len(kept)) + b"".join(kept)
    return out, hashlib.sha256(data).hexdigest()


def random_blocks(rng, type_id: int, nb: int) -> np.ndarray:
    bs, bb = {TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}[type_id]
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    offs = {TYPE_Q8_0: [0], TYPE_Q4_K: [0, 2], TYPE_Q6_K: [208]}[type_id]
    for off in offs:
        h = rng.integers(0, 0x7C00, size=nb).astype(np.uint16)
        h |= (rng.integers(0, 2, size=nb).astype(np.uint16) << 15)
        # edge scales: zero, smallest subnormal, largest subnormal, smallest normal, max finite
        specials = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00],
                            dtype=np.uint16)
        h[: len(specials)] = specials
        raw[:, off] = (h & 0xFF).astype(np.uint8)
        raw[:, off + 1] = (h >> 8).astype(np.uint8)
    return raw.reshape(-1)


def main() -> None:
    ref = Reference()
    orc = Oracle()
    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}

    # dequantisation of random-but-valid blocks (all nibble / 6-bit patterns)
    for name, t, nb in (("q8_0", TYPE_Q8_0, 256), ("q4_k", TYPE_Q4_K, 64)):
        bs = 32 if t == TYPE_Q8_0 else 256
        raw = random_blocks(rng, t, nb)
        out[f"dequant_{name}_src"] = raw
        out[f"dequant_{name}_out"] = ref.dequant(t, raw, nb * bs)

    # quantised GEMV: Gaussian weights encoded by the oracle's encoders
    out_dim, in_dim, tokens = 48, 512, 3
    for name, t in (("q8_0", TYPE_Q8_0), ("q4_k", TYPE_Q4_K)):
        w = orc.quantize(t, rng.normal(0, 0.02, size=out_dim * in_dim).astype(np.float32))
        x = bf16_round(rng.normal(0, 1, size=(tokens, in_dim)).astype(np.float32))
        out[f"gemv_{name}_w"] = w
        out[f"gemv_{name}_x"] = x
        out[f"gemv_{name}_y_auto"] = np.stack([ref.gemv_quant(t, w, xt, out_dim, in_dim) for xt in x])
        out[f"gemv_{name}_y_scalar"] = np.stack(
            [ref.gemv_quant(t, w, xt, out_dim, in_dim, scalar=True) for xt in x])
    out["gemv_shape"] = np.array([out_dim, in_dim, tokens], dtype=np.int64)

    # F32 matvec in both reference orders
    fo, fi = 40, 96
    w = rng.normal(0, 0.5, size=(fo, fi)).astype(np.float32)
    x = rng.normal(0, 1, size=fi).astype(np.float32)
    out["f32_w"], out["f32_x"] = w, x
    out["f32_y_scalar"] = ref.gemv_f32(w, x, fo, fi, scalar=True)
    out["f32_y_auto"] = ref.gemv_f32(w, x, fo, fi, scalar=False)

    # router: Engine::softmax / Engine::topk / renormalisation
    for E, k in ((4, 2), (8, 2), (64, 6), (128, 8)):
        lg = rng.normal(0, 1, size=(64, E)).astype(np.float32)
        lg[0, :] = 0.25                      # all equal: ties resolve to the lowest ids
        lg[1, ::2] = lg[1, 1::2]             # pairwise ties
        lg[2, :] = np.round(lg[2, :], 1)     # many ties
        lg[3, :] *= 40.0                     # saturated softmax (underflowing exps)
        rc, ids, wts, probs = ref.route(lg, k)
        assert rc == 0
        out[f"route_E{E}_k{k}_logits"] = lg
        out[f"route_E{E}_k{k}_ids"] = ids
        out[f"route_E{E}_k{k}_weights"] = wts
        out[f"route_E{E}_k{k}_probs"] = probs

    # SwiGLU
    g = np.concatenate([rng.normal(0, 4, size=1000), [0.0, -0.0, 80.0, -80.0, 1e-30, -1e-30]]).astype(np.float32)
    u = rng.normal(0, 1, size=g.size).astype(np.float32)
    out["swiglu_gate"], out["swiglu_up"], out["swiglu_out"] = g, u, ref.swiglu(g, u)

    # Q6_K (the down projection of mixed-type records): decode and GEMV, drawn
    # after everything above so the earlier vectors keep their values
    raw = random_blocks(rng, TYPE_Q6_K, 64)
    out["dequant_q6_k_src"] = raw
    out["dequant_q6_k_out"] = ref.dequant(TYPE_Q6_K, raw, 64 * 256)
    w = orc.quantize(TYPE_Q6_K, rng.normal(0, 0.02, size=out_dim * in_dim).astype(np.float32))
    x = bf16_round(rng.normal(0, 1, size=(tokens, in_dim)).astype(np.float32))
    out["gemv_q6_k_w"] = w
    out["gemv_q6_k_x"] = x
    out["gemv_q6_k_y_auto"] = np.stack([ref.gemv_quant(TYPE_Q6_K, w, xt, out_dim, in_dim) for xt in x])
    out["gemv_q6_k_y_scalar"] = np.stack(
        [ref.gemv_quant(TYPE_Q6_K, w, xt, out_dim, in_dim, scalar=True) for xt in x])

    qr, qr_sha = extract_quant_reference()
    (HERE / "quant_reference_hotpath.bin").write_bytes(qr)
    np.savez_compressed(HERE / "golden_vectors.npz", **out)
    manifest = {
        "generator": "tests/golden/make_golden.py",
        "reference_isa": ref.isa(),
        "source_quant_reference_sha256": qr_sha,
        "quant_reference_hotpath_sha256": hashlib.sha256(qr).hexdigest(),
        "golden_vectors_sha256": hashlib.sha256((HERE / "golden_vectors.npz").read_bytes()).hexdigest(),
    }
    (HERE / "golden_manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
