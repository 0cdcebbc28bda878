"""Engine-level fixtures of the reference, for the GPU-backend engine tests.

Copies, byte for byte, from the reference tree (FM_REFERENCE):
  * tests/fixtures/quant-moe-{q8_0,q4_k,q6_k}.gguf and
    tests/fixtures/quant-expert-{separate,fused}.gguf -- the block-quantised
    fixtures of test_quant_model_parity / test_quant_expert_mixed_types
    (tests/unit/tests.cpp:1424-1544);
  * tests/fixtures/moe-fm.gguf with tests/reference/prompt_XX.txt and
    tests/reference/moe/prompt_XX.{logits,greedy.ids,routing.txt} -- the
    20-prompt MoE comparison (tests/unit/tests.cpp:958-1046).
and records, for each quantised fixture, the greedy ids and prefill logits of
its -f32ref twin run by the reference's own engine on the CPU backend
(oracle/_ref/fm_engine, the reference compiled from source) with the prompt
and token count the reference's test uses.  The twins themselves (3 MB each)
stay out of the repository; only their outputs are kept (goldens.json).

Run from the repository root with FM_REFERENCE set and oracle/_ref built:
    FM_REFERENCE=<reference tree> python tests/golden/make_engine_fixtures.py
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import struct
import subprocess
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = ROOT / "tests" / "golden" / "engine"
ENGINE = ROOT / "oracle" / "_ref" / "fm_engine"

# variant -> (prompt, generated tokens) of the reference's own tests
QUANT = {
    "quant-moe-q8_0": ("quantised conformance", 6),
    "quant-moe-q4_k": ("quantised conformance", 6),
    "quant-moe-q6_k": ("quantised conformance", 6),
    "quant-expert-separate": ("mixed experts", 6),
    "quant-expert-fused": ("mixed experts", 6),
}


def sha256(p: Path) -> str:
    return hashlib.sha256(p.read_bytes()).hexdigest()


def run_cpu(model: Path, prompt: str, tokens: int) -> tuple[list[int], list[float]]:
    with tempfile.TemporaryDirectory() as td:
        out = Path(td) / "r.bin"
        subprocess.run([str(ENGINE), "run", str(model), "cpu", prompt.encode().hex(), str(tokens), "0", "0", str(out)],
                       check=True, capture_output=True)
        b = out.read_bytes()
    n = struct.unpack_from("<I", b, 0)[0]
    ids = list(struct.unpack_from(f"<{n}i", b, 4))
    pos = 4 + 4 * n
    m = struct.unpack_from("<I", b, pos)[0]
    logits = list(struct.unpack_from(f"<{m}f", b, pos + 4))
    return ids, logits


def main() -> None:
    ref = Path(os.environ["FM_REFERENCE"])
    OUT.mkdir(parents=True, exist_ok=True)
    manifest, goldens = {}, {}
    for name in [*QUANT, "moe-fm"]:
        src = ref / "tests" / "fixtures" / f"{name}.gguf"
        dst = OUT / src.name
        shutil.copyfile(src, dst)
        manifest[dst.name] = sha256(dst)
    refdir = OUT / "reference"
    (refdir / "moe").mkdir(parents=True, exist_ok=True)
    for i in range(20):
        stem = f"prompt_{i:02d}"
        shutil.copyfile(ref / "tests" / "reference" / f"{stem}.txt", refdir / f"{stem}.txt")
        manifest[f"reference/{stem}.txt"] = sha256(refdir / f"{stem}.txt")
        for ext in ("logits", "greedy.ids", "routing.txt"):
            p = refdir / "moe" / f"{stem}.{ext}"
            shutil.copyfile(ref / "tests" / "reference" / "moe" / f"{stem}.{ext}", p)
            manifest[f"reference/moe/{stem}.{ext}"] = sha256(p)
    for name, (prompt, tokens) in QUANT.items():
        twin = ref / "tests" / "fixtures" / f"{name}-f32ref.gguf"
        ids, logits = run_cpu(twin, prompt, tokens)
        goldens[name] = {"prompt": prompt, "tokens": tokens, "f32ref": twin.name, "f32ref_sha256": sha256(twin),
                         "ids": ids, "logits": logits}
    (OUT / "goldens.json").write_text(json.dumps({"manifest": manifest, "quant": goldens}, indent=1) + "\n")
    print(f"wrote {len(manifest)} files and {len(goldens)} goldens to {OUT}")


if __name__ == "__main__":
    main()
