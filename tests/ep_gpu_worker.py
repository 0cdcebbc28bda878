"""One rank of the expert-parallel GPU test (launched by test_ep_gpu.py with
torchrun, one process per GPU, NCCL).  Every rank builds the same expert stack
and token batch from seeds, keeps its expert shard and its token shard, runs
EPLayer, and rank 0 compares the gathered output with fmcuda_moe_prefill over
all experts on one GPU: identical bits in the per-pair exchange ("pairs"); in
the de-duplicated exchange ("rows") the terms are summed grouped by rank, so
the bar is 1e-5 of max |y|; the peer-memory exchange ("p2p") must equal "rows"
bit for bit on three successive calls.  With a last argument "block" the
reference is fmcuda_moe_block instead (decode-sized batches, where each rank's
experts run on the tcgen05 decode stage): within 1e-5 of max |y| for "rows"
and "p2p"."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    E, k, d, ffn, T, t = (int(v) for v in sys.argv[1:7])
    mode = sys.argv[7] if len(sys.argv) > 7 else "pairs"
    ref = sys.argv[8] if len(sys.argv) > 8 else "prefill"
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    from freemoe_b200 import hotpath
    from freemoe_b200.ep import DeviceOps, EPLayer

    hotpath.init(local)
    rb = hotpath.row_bytes
    slots = [torch.cat([hotpath.synth_weights(t, ffn, d, 5000 + 3 * e), hotpath.synth_weights(t, ffn, d, 5001 + 3 * e),
                        hotpath.synth_weights(t, d, ffn, 5002 + 3 * e)]) for e in range(E)]
    gb = rb(t, d) * ffn
    rng = np.random.default_rng(11)
    x = torch.from_numpy(rng.normal(0, 1, size=(T, d)).astype(np.float32)).cuda().to(torch.bfloat16)
    logits = torch.from_numpy(rng.uniform(-1, 1, size=(T, E)).astype(np.float32)).cuda()
    per, tp = E // world, T // world
    ops = DeviceOps(experts_total=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                    local_slots=slots[rank * per:(rank + 1) * per], up_offset=gb, down_offset=2 * gb)
    xs, ls = x[rank * tp:(rank + 1) * tp].contiguous(), logits[rank * tp:(rank + 1) * tp].contiguous()
    if mode == "nccl_c":
        # the layer driven from the C ABI over its own NCCL communicator must equal
        # the Python layer's "rows" exchange bit for bit, call after call
        import ctypes as C

        from freemoe_b200._lib import X_BF16, EpLayerArgs, check, load

        lib = load()
        y_rows = EPLayer(ops, mode="rows").forward(xs, ls)
        uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            h = (C.c_uint8 * 128)()
            check(lib.fmcuda_ep_nccl_unique_id(h))
            uid.copy_(torch.tensor(list(h), dtype=torch.uint8))
        dist.broadcast(uid, 0)
        uid_h = (C.c_uint8 * 128)(*uid.cpu().tolist())
        comm = C.c_void_p()
        check(lib.fmcuda_ep_init(uid_h, rank, world, C.byref(comm)))
        a = EpLayerArgs()
        a.x, a.x_dtype, a.logits = xs.data_ptr(), X_BF16, ls.data_ptr()
        a.tokens, a.experts, a.top_k, a.d_model, a.ffn = xs.shape[0], E, k, d, ffn
        a.local_slots, a.up_offset, a.down_offset = ops.table.data_ptr(), gb, 2 * gb
        a.gate_type = a.up_type = a.down_type = t
        a.normalise, a.epsilon, a.scale = 1, 6.103515625e-5, 1.0
        y = torch.empty(xs.shape[0], d, device="cuda")
        a.y = y.data_ptr()
        nbytes = C.c_uint64()
        check(lib.fmcuda_ep_layer_workspace_bytes(tp, world, per, k, d, ffn, C.byref(nbytes)))
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
        for call in range(3):
            check(lib.fmcuda_ep_layer(comm, C.byref(a), tp, C.c_void_p(ws.data_ptr()), ws.numel(), None))
            torch.cuda.synchronize()
            assert hotpath.device_status() == 0
            assert torch.equal(y.view(torch.int32), y_rows.view(torch.int32)), f"call {call} differs from mode rows"
        check(lib.fmcuda_ep_destroy(comm))
    elif mode == "p2p":
        # the peer-memory exchange must reproduce mode "rows" bit for bit, call after call
        y_rows = EPLayer(ops, mode="rows").forward(xs, ls)
        layer = EPLayer(ops, mode="p2p")
        for call in range(3):
            y = layer.forward(xs, ls)
            torch.cuda.synchronize()
            assert hotpath.device_status() == 0
            assert torch.equal(y.view(torch.int32), y_rows.view(torch.int32)), f"call {call} differs from mode rows"
        layer.close()
    else:
        layer = EPLayer(ops, mode=mode)
        y = layer.forward(xs, ls)
    torch.cuda.synchronize()
    assert hotpath.device_status() == 0
    parts = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(parts, y)
    ok = torch.tensor([1], device="cuda")
    if rank == 0:
        y_ep = torch.cat(parts)
        if ref == "block":
            y_one = hotpath.moe_block(x, logits, slots, top_k=k, ffn=ffn, gate_type=t)
        else:
            y_one = hotpath.moe_prefill(x, logits, slots, top_k=k, ffn=ffn, gate_type=t)
        same = torch.equal(y_ep.view(torch.int32), y_one.view(torch.int32))
        err = float((y_ep - y_one).abs().max() / y_one.abs().max())
        print(f"ep world={world} mode={mode} ref={ref}: identical={same} max_rel={err:.3e}", flush=True)
        ok[0] = int(same) if mode == "pairs" else int(err <= 1e-5)  # nccl_c: "rows" checked on every rank above
    dist.broadcast(ok, 0)
    dist.destroy_process_group()
    sys.exit(0 if ok.item() else 1)


if __name__ == "__main__":
    main()
