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
    if mode == "p2p":
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
        ok[0] = int(same) if mode == "pairs" else int(err <= 1e-5)
    dist.broadcast(ok, 0)
    dist.destroy_process_group()
    sys.exit(0 if ok.item() else 1)


if __name__ == "__main__":
    main()
