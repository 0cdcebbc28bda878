"""Expert-parallel exchange logic (freemoe_b200/ep.py) on gloo ranks, CPU only.

Two ranks each own half of the experts and half of the tokens.  The layer's
arithmetic is plugged in as a host implementation built on the oracle (router,
per-row expert FFN, combine), so the test checks what EPLayer itself does: the
grouping by destination, the count and row exchanges with ragged and empty
splits, the return of the outputs and the combine order.  The result must equal
the oracle's single-process MoE block: bit for bit in the per-pair exchange
(mode "pairs"); in the de-duplicated exchange (mode "rows", one row per token and
destination rank, partial sums back) the same terms are summed grouped by rank,
so the bar there is the f32 rounding of that regrouping.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

E, K, D, FFN, T_PER_RANK = 8, 2, 64, 64, 12


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class HostOps:
    """Host arithmetic with the DeviceOps interface (oracle-backed)."""

    def __init__(self, oracle, slots, per_rank_slots, t):
        self.o, self.E, self.k, self.d, self.ffn = oracle, E, K, D, FFN
        self.all_slots, self.slots, self.t = slots, per_rank_slots, t

    def route(self, logits):
        rc, ids, w, _ = self.o.route(logits.numpy(), self.k)
        assert rc == 0
        return torch.from_numpy(ids.astype(np.int32)), torch.from_numpy(w)

    def dispatch(self, ids, x, world):
        from freemoe_b200.ep import Dispatch

        ids_np = ids.numpy().astype(np.int64)
        per_rank = self.E // world
        dest = (ids_np // per_rank).ravel()
        order = np.argsort(dest, kind="stable")
        slot_of = np.empty_like(order)
        slot_of[order] = np.arange(order.size)
        counts = np.bincount(dest, minlength=world)
        send_x = x.numpy()[order // self.k]
        send_e = (ids_np.ravel()[order] % per_rank).astype(np.int32)
        return Dispatch(torch.from_numpy(counts.astype(np.int64)), torch.from_numpy(np.ascontiguousarray(send_x)),
                        torch.from_numpy(send_e), torch.from_numpy(slot_of.astype(np.int32)))

    def empty_rows(self, n, like):
        return torch.zeros(max(n, 1), self.d, dtype=like.dtype)

    def experts(self, rows, expert, n):
        out = np.zeros((max(n, 1), self.d), dtype=np.float32)
        if n:
            ids = expert.numpy()[:n].astype(np.uint32).reshape(-1, 1)
            out[:n] = self.o.moe_block(rows.numpy()[:n], ids, np.ones((n, 1), np.float32), self.slots, self.d,
                                       self.ffn, self.t)
        return torch.from_numpy(out)

    def dispatch_rows(self, ids, w, x, world):
        from freemoe_b200.ep import RowDispatch

        ids_np = ids.numpy().astype(np.int64)
        T, k = ids_np.shape
        per_rank = self.E // world
        dest_of = ids_np // per_rank
        items = [t * world + dst for dst in range(world) for t in range(T) if (dest_of[t] == dst).any()]
        counts = np.bincount([i % world for i in items], minlength=world)
        row_of = np.full(T * world, -1, dtype=np.int32)
        row_of[np.array(items, dtype=np.int64)] = np.arange(len(items))
        xs = x.numpy()
        send_x = np.stack([xs[i // world] for i in items]) if items else np.zeros((1, self.d), np.float32)
        meta_e = np.full((max(len(items), 1), k), -1, dtype=np.int32)
        meta_w = np.zeros((max(len(items), 1), k), dtype=np.float32)
        wn = w.numpy()
        for j, i in enumerate(items):
            t, dst = i // world, i % world
            for r in range(k):
                if dest_of[t, r] == dst:
                    meta_e[j, r] = ids_np[t, r] % per_rank
                    meta_w[j, r] = wn[t, r]
        return RowDispatch(torch.from_numpy(counts.astype(np.int64)), torch.from_numpy(np.ascontiguousarray(send_x)),
                           torch.from_numpy(meta_e), torch.from_numpy(meta_w), torch.from_numpy(row_of))

    def experts_partial(self, rows, meta_e, meta_w, n):
        out = np.zeros((max(n, 1), self.d), dtype=np.float32)
        me, mw, xr = meta_e.numpy(), meta_w.numpy(), rows.numpy()
        for j in range(n):
            acc = np.zeros(self.d, dtype=np.float32)
            for r in range(self.k):
                if me[j, r] >= 0:
                    o = self.o.moe_block(xr[j:j + 1], np.array([[me[j, r]]], np.uint32), np.ones((1, 1), np.float32),
                                         self.slots, self.d, self.ffn, self.t)[0]
                    acc = acc + np.float32(mw[j, r]) * o
            out[j] = acc
        return torch.from_numpy(out)

    def combine_rows(self, back, row_of, tokens, world):
        b, ro = back.numpy(), row_of.numpy()
        y = np.zeros((tokens, self.d), dtype=np.float32)
        for t in range(tokens):
            for r in range(world):
                if ro[t * world + r] >= 0:
                    y[t] = y[t] + b[ro[t * world + r]]
        return torch.from_numpy(y)

    def combine(self, back, w, slot_of):
        back, w, s = back.numpy(), w.numpy(), slot_of.numpy()
        T = w.shape[0]
        y = np.zeros((T, self.d), dtype=np.float32)
        for t in range(T):
            for r in range(self.k):
                y[t] = y[t] + np.float32(w[t, r]) * back[s[t * self.k + r]]
        return torch.from_numpy(y)


def problem(oracle, case):
    from oracle.oracle import TYPE_Q8_0

    rng = np.random.default_rng(5 + case)
    t = TYPE_Q8_0
    slots = [np.concatenate([oracle.quantize(t, rng.normal(0, 0.02, size=n).astype(np.float32))
                             for n in (FFN * D, FFN * D, D * FFN)]) for _ in range(E)]
    T = 2 * T_PER_RANK
    x = rng.normal(0, 1, size=(T, D)).astype(np.float32)
    logits = rng.normal(0, 1, size=(T, E)).astype(np.float32)
    if case == 1:
        logits[:, : E // 2] += 20.0  # every pair goes to rank 0: rank 1 receives nothing
    return t, slots, x, logits


def worker(rank, world, port, case, out_dir, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    sys.path.insert(0, str(ROOT))
    from freemoe_b200.ep import EPLayer
    from oracle.oracle import Oracle

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        oracle = Oracle()
        t, slots, x, logits = problem(oracle, case)
        per = E // world
        ops = HostOps(oracle, slots, slots[rank * per:(rank + 1) * per], t)
        layer = EPLayer(ops, mode=mode)
        sl = slice(rank * T_PER_RANK, (rank + 1) * T_PER_RANK)
        y = layer.forward(torch.from_numpy(x[sl]), torch.from_numpy(logits[sl]))
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["pairs", "rows"])
@pytest.mark.parametrize("case", [0, 1])
def test_ep_two_gloo_ranks_match_single_process(oracle, tmp_path, case, mode):
    world = 2
    mp.start_processes(worker, args=(world, free_port(), case, str(tmp_path), mode), nprocs=world,
                       start_method="spawn", join=True)
    y = np.concatenate([np.load(tmp_path / f"y{r}.npy") for r in range(world)])
    t, slots, x, logits = problem(oracle, case)
    rc, ids, w, _ = oracle.route(logits, K)
    y_ref = oracle.moe_block(x, ids, w, slots, D, FFN, t)
    if mode == "pairs":
        assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
    else:
        assert np.max(np.abs(y - y_ref)) <= 1e-6 * np.max(np.abs(y_ref))
