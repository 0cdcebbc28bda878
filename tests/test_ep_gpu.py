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


def _file_store(tmp_path) -> str:
    """Rendezvous of a one-rank process group through a file (no port to race for)."""
    return f"file://{tmp_path / 'pg_store'}"


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(16, 4, 256, 256, 512, 12), (128, 8, 4096, 1536, 1024, 12), (64, 6, 2048, 1408, 512, 8)])
@pytest.mark.parametrize("mode", ["pairs", "rows", "p2p", "nccl_c"])
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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("shape", [(8, 8, 512, 768, 8, 12), (8, 2, 4096, 14336, 4, 12)])
@pytest.mark.parametrize("mode", ["rows", "p2p", "nccl_c"])
def test_ep_decode_matches_moe_block(shape, mode):
    """Decode-sized batches (one 8-token tile per expert on average): every rank's
    experts run on the tcgen05 decode stage; the gathered output is within 1e-5
    of max |y| of fmcuda_moe_block over all experts on one GPU."""
    n = min(torch.cuda.device_count(), 8)
    n = 2 if shape[0] % n or shape[4] % n else n
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", "--master-port=29733",
           str(ROOT / "tests" / "ep_gpu_worker.py"), *map(str, shape), mode, "block"]
    p = subprocess.run(cmd, capture_output=True, text=True, cwd=str(ROOT), env={**__import__("os").environ,
                       "NCCL_NVLS_ENABLE": "0"})
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    assert "ref=block" in p.stdout and "max_rel=" in p.stdout


def test_p2p_decode_single_rank(cuda, oracle, tmp_path):
    """One rank through the peer-memory exchange with a decode-sized batch (the
    tcgen05 decode stage computes the experts from the fp16 mailbox rows): three
    calls in a row, each within 1e-5 of max |y| of fmcuda_moe_block and within
    1e-3 of the oracle's per-token expert loop."""

    import numpy as np
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200.ep import DeviceOps, EPLayer

    dist.init_process_group("gloo", init_method=_file_store(tmp_path), rank=0, world_size=1)
    try:
        E, k, d, ffn, T, t = 8, 2, 512, 768, 6, 12
        rb = hotpath.row_bytes
        slots = [torch.cat([hotpath.synth_weights(t, ffn, d, 7100 + 3 * e), hotpath.synth_weights(t, ffn, d, 7101 + 3 * e),
                            hotpath.synth_weights(t, d, ffn, 7102 + 3 * e)]) for e in range(E)]
        gb = rb(t, d) * ffn
        rng = np.random.default_rng(4)
        x_np = rng.normal(0, 1, size=(T, d)).astype(np.float32)
        x = torch.from_numpy(x_np).cuda().to(torch.bfloat16)
        lg_np = rng.normal(0, 1, size=(T, E)).astype(np.float32)
        logits = torch.from_numpy(lg_np).cuda()
        ops = DeviceOps(experts_total=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                        local_slots=slots, up_offset=gb, down_offset=2 * gb)
        y_block = hotpath.moe_block(x, logits, slots, top_k=k, ffn=ffn, gate_type=t)
        rc, ids_o, w_o, _ = oracle.route(lg_np, k)
        y_o = oracle.moe_block(x.float().cpu().numpy(), ids_o, w_o, [s.cpu().numpy() for s in slots], d, ffn, t)
        layer = EPLayer(ops, mode="p2p")
        for _ in range(3):
            y = layer.forward(x, logits)
            torch.cuda.synchronize()
            assert cuda.device_status() == 0
            err_b = float((y - y_block).abs().max() / y_block.abs().max())
            assert err_b <= 1e-5, err_b
            err_o = float(np.abs(y.cpu().numpy() - y_o).max() / np.abs(y_o).max())
            assert err_o <= 1e-3, err_o
        layer.close()
        # device epochs: one forward captured in a CUDA graph and replayed, each
        # replay equal to the explicit-epoch calls bit for bit
        g_layer = EPLayer(ops, mode="p2p", device_epoch=True)
        y0 = g_layer.forward(x, logits)
        torch.cuda.synchronize()
        assert torch.equal(y0.view(torch.int32), y.view(torch.int32))
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            g_layer.forward(x, logits)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_g = g_layer.forward(x, logits)
        for _ in range(3):
            y_g.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert cuda.device_status() == 0
            assert torch.equal(y_g.view(torch.int32), y.view(torch.int32))
        del graph
        g_layer.close()
    finally:
        dist.destroy_process_group()


def nccl_c_layer(lib, comm, x, logits, slots_table, *, world, n_local, E, k, d, ffn, t, gb, tokens_max):
    """One fmcuda_ep_layer call through the C ABI (the NCCL-driven layer)."""
    import ctypes as C

    from freemoe_b200._lib import X_BF16, EpLayerArgs, check

    a = EpLayerArgs()
    a.x, a.x_dtype, a.logits = x.data_ptr(), X_BF16, logits.data_ptr()
    a.tokens, a.experts, a.top_k, a.d_model, a.ffn = x.shape[0], E, k, d, ffn
    a.local_slots, a.up_offset, a.down_offset = slots_table.data_ptr(), gb, 2 * gb
    a.gate_type = a.up_type = a.down_type = t
    a.normalise, a.epsilon, a.scale = 1, 6.103515625e-5, 1.0
    y = torch.empty(x.shape[0], d, device=x.device)
    a.y = y.data_ptr()
    nbytes = C.c_uint64()
    check(lib.fmcuda_ep_layer_workspace_bytes(tokens_max, world, n_local, k, d, ffn, C.byref(nbytes)))
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=x.device)
    check(lib.fmcuda_ep_layer(comm, C.byref(a), tokens_max, C.c_void_p(ws.data_ptr()), ws.numel(), None))
    return y


@pytest.mark.parametrize("shape", [(16, 4, 256, 256, 64, 12), (8, 2, 512, 768, 6, 12)])
def test_nccl_c_layer_single_rank(cuda, shape, tmp_path):
    """fmcuda_ep_init / fmcuda_ep_layer with one rank (NCCL sends to itself): the
    layer driven from the C ABI equals the Python layer's "rows" exchange bit for
    bit, twice in a row, for a prefill-sized batch (grouped GEMM) and a
    decode-sized one (tcgen05 decode stage)."""
    import ctypes as C

    import numpy as np
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200._lib import EP_NCCL_ID_BYTES, check, load
    from freemoe_b200.ep import DeviceOps, EPLayer

    E, k, d, ffn, T, t = shape
    lib = load()
    dist.init_process_group("gloo", init_method=_file_store(tmp_path), rank=0, world_size=1)
    comm = C.c_void_p()
    try:
        rb = hotpath.row_bytes
        slots = [torch.cat([hotpath.synth_weights(t, ffn, d, 7200 + 3 * e), hotpath.synth_weights(t, ffn, d, 7201 + 3 * e),
                            hotpath.synth_weights(t, d, ffn, 7202 + 3 * e)]) for e in range(E)]
        gb = rb(t, d) * ffn
        rng = np.random.default_rng(5)
        x = torch.from_numpy(rng.normal(0, 1, size=(T, d)).astype(np.float32)).cuda().to(torch.bfloat16)
        logits = torch.from_numpy(rng.normal(0, 1, size=(T, E)).astype(np.float32)).cuda()
        ops = DeviceOps(experts_total=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                        local_slots=slots, up_offset=gb, down_offset=2 * gb)
        y_rows = EPLayer(ops, mode="rows").forward(x, logits)
        uid = (C.c_uint8 * EP_NCCL_ID_BYTES)()
        check(lib.fmcuda_ep_nccl_unique_id(uid))
        check(lib.fmcuda_ep_init(uid, 0, 1, C.byref(comm)))
        for _ in range(2):
            y = nccl_c_layer(lib, comm, x, logits, ops.table, world=1, n_local=E, E=E, k=k, d=d, ffn=ffn, t=t, gb=gb,
                             tokens_max=T)
            torch.cuda.synchronize()
            assert cuda.device_status() == 0
            assert torch.equal(y.view(torch.int32), y_rows.view(torch.int32))
    finally:
        if comm.value:
            lib.fmcuda_ep_destroy(comm)
        dist.destroy_process_group()


def test_nccl_c_layer_rejects_bad_arguments(cuda):
    """Host-side validation of the NCCL layer: typed INVALID_ARGUMENT, nothing launched."""
    import ctypes as C

    from freemoe_b200._lib import EpLayerArgs, load

    lib = load()
    assert lib.fmcuda_ep_init(None, 0, 1, None) == 26
    uid = (C.c_uint8 * 128)()
    out = C.c_void_p()
    assert lib.fmcuda_ep_init(uid, 2, 2, C.byref(out)) == 26  # rank >= world
    assert lib.fmcuda_ep_layer(None, C.byref(EpLayerArgs()), 1, None, 0, None) == 26


def test_p2p_exchange_single_rank_and_timeout(cuda, tmp_path):
    """One rank (world 1) through the peer-memory exchange: mailbox, IPC handle,
    the count/plan/send/return/combine kernels writing to its own mailbox,
    three calls in a row, each equal bit for bit to fmcuda_moe_prefill.  Then a
    wait whose flag nothing raises gives up after its limit with FENCE_TIMEOUT
    in the device status word (the wait is bounded, the context stays usable)."""
    import ctypes as C

    import numpy as np
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200._lib import load
    from freemoe_b200.ep import DeviceOps, EPLayer

    dist.init_process_group("gloo", init_method=_file_store(tmp_path), rank=0, world_size=1)
    try:
        E, k, d, ffn, T, t = 16, 4, 256, 256, 64, 12
        rb = hotpath.row_bytes
        slots = [torch.cat([hotpath.synth_weights(t, ffn, d, 7000 + 3 * e), hotpath.synth_weights(t, ffn, d, 7001 + 3 * e),
                            hotpath.synth_weights(t, d, ffn, 7002 + 3 * e)]) for e in range(E)]
        gb = rb(t, d) * ffn
        rng = np.random.default_rng(3)
        x = torch.from_numpy(rng.normal(0, 1, size=(T, d)).astype(np.float32)).cuda().to(torch.bfloat16)
        logits = torch.from_numpy(rng.uniform(-1, 1, size=(T, E)).astype(np.float32)).cuda()
        ops = DeviceOps(experts_total=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                        local_slots=slots, up_offset=gb, down_offset=2 * gb)
        y_one = hotpath.moe_prefill(x, logits, slots, top_k=k, ffn=ffn, gate_type=t)
        layer = EPLayer(ops, mode="p2p")
        for _ in range(3):
            y = layer.forward(x, logits)
            torch.cuda.synchronize()
            assert cuda.device_status() == 0
            assert torch.equal(y.view(torch.int32), y_one.view(torch.int32))
        # a combine for an epoch nobody announced: bounded wait, FENCE_TIMEOUT
        row_of = torch.zeros(T, dtype=torch.int32, device="cuda")
        y_bad = torch.empty(T, d, device="cuda")
        rc = load().fmcuda_ep_p2p_combine(C.c_void_p(ops.mailbox), 1, 0, ops.capacity, layer.epoch + 5, k,
                                          C.c_void_p(row_of.data_ptr()), T, d, C.c_void_p(y_bad.data_ptr()), 50, None)
        assert rc == 0
        torch.cuda.synchronize()
        assert cuda.device_status(clear=True) == 22  # FENCE_TIMEOUT
        layer.close()
    finally:
        dist.destroy_process_group()
