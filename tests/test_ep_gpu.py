"""Expert-parallel layer over NCCL on 2+ GPUs against the one-GPU grouped-GEMM
prefill: bit for bit with the per-pair exchange (each pair's expert output does
not depend on which rank computes it), within 1e-5 of max |y| with the
de-duplicated exchange (partial sums grouped by rank).  Skipped when fewer than
two GPUs are visible."""
from __future__ import annotations

import subprocess
import sys

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(16, 4, 256, 256, 512, 12), (128, 8, 4096, 1536, 1024, 12), (64, 6, 2048, 1408, 512, 8)])
@pytest.mark.parametrize("mode", ["pairs", "rows"])
def test_ep_matches_single_gpu(shape, mode):
    n = min(torch.cuda.device_count(), 8)
    n = 2 if shape[0] % n else n
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29731",
           str(ROOT / "tests" / "ep_gpu_worker.py"), *map(str, shape), mode]
    p = subprocess.run(cmd, capture_output=True, text=True, cwd=str(ROOT), env={**__import__("os").environ,
                       "NCCL_NVLS_ENABLE": "0"})
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert ("identical=True" if mode == "pairs" else "max_rel=") in p.stdout
