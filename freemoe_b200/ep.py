"""Expert-parallel MoE layer: experts sharded over the ranks of a process group,
token rows dispatched to the experts' owners and the outputs combined back.

No counterpart in the reference (FreeMoe runs every expert in one process);
the per-rank arithmetic is the reference's expert loop (src/engine.cpp:1711-1772)
on the grouped GEMM.  Expert e lives on rank e // (E / world).  One layer call:

  route          ids, weights of this rank's tokens            (fmcuda_route)
  dispatch       pairs grouped by destination rank, fp16 rows   (fmcuda_ep_dispatch)
  all-to-all     counts, then rows and local expert ids
  experts        the received rows through this rank's experts (fmcuda_moe_experts)
  all-to-all     the f32 outputs back to the tokens' owners
  combine        y[t] = sum over r of w[t, r] * out[slot_of(t, r)] in top-k order

That is ``mode="pairs"``: one row per (token, expert) pair each way, and a result
equal to the one-GPU block bit for bit.  ``mode="rows"`` (the default) sends a
token once to each rank that owns any of its experts (fmcuda_ep_dispatch_rows)
and gets back one f32 partial sum per (token, rank) (fmcuda_moe_experts_partial,
fmcuda_ep_combine_rows): less traffic, the same terms summed grouped by rank.

The exchange uses ``torch.distributed.all_to_all_single`` on the group (NCCL
over NVLink on GPUs).  ``mode="p2p"`` (one node, CUDA devices) does the
de-duplicated exchange with no collective call in the data path: every rank
owns a mailbox shared over CUDA IPC, the dispatch kernel writes the token rows
straight into the destinations' mailboxes and the partial-sum kernel writes its
results straight back (fmcuda_ep_p2p_*); the result is that of ``mode="rows"``
bit for bit.  The arithmetic is pluggable (``ops``): :class:`DeviceOps` calls
the sm_100a library; the CPU tests plug in a host implementation to check the
exchange and ordering logic with gloo ranks.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class RowDispatch:
    send_counts: torch.Tensor  # [world] int64
    send_x: torch.Tensor       # [>= S, d] token rows, one per (token, destination)
    meta_e: torch.Tensor       # [>= S, k] int32 local expert per top-k slot, -1 elsewhere
    meta_w: torch.Tensor       # [>= S, k] f32 routing weight per slot, 0 elsewhere
    row_of: torch.Tensor       # [T * world] int32 send row of (t, dest), -1 if none


@dataclass
class Dispatch:
    send_counts: torch.Tensor  # [world] int64, on the exchange device
    send_x: torch.Tensor       # [>= S, d] rows in send order (fp16 on the device)
    send_expert: torch.Tensor  # [>= S] int32 local expert ids
    slot_of: torch.Tensor      # [T*k] int32: send row of pair t*k + r


class DeviceOps:
    """The sm_100a kernels through the C ABI (all tensors on one CUDA device)."""

    def __init__(self, *, experts_total: int, top_k: int, d_model: int, ffn: int, gate_type: int,
                 up_type: int, down_type: int, local_slots, up_offset: int, down_offset: int):
        from . import hotpath
        from ._lib import X_BF16, X_F32, check, load

        self.h, self.lib, self.check = hotpath, load(), check
        self.X_BF16, self.X_F32 = X_BF16, X_F32
        self.E, self.k, self.d, self.ffn = experts_total, top_k, d_model, ffn
        self.types = (gate_type, up_type, down_type)
        self.up_offset, self.down_offset = up_offset, down_offset
        self.slots = local_slots
        self.table = hotpath.slot_table(local_slots, local_slots[0].device) if local_slots else None
        self._ws = {}

    def _buf(self, name, nbytes, device):
        b = self._ws.get(name)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
            self._ws[name] = b
        return b

    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def route(self, logits: torch.Tensor):
        T = logits.shape[0]
        ids = torch.empty(T, self.k, dtype=torch.int32, device=logits.device)
        w = torch.empty(T, self.k, dtype=torch.float32, device=logits.device)
        self.check(self.lib.fmcuda_route(C.c_void_p(logits.data_ptr()), T, self.E, self.k, 1, 6.103515625e-5, 1.0,
                                         C.c_void_p(ids.data_ptr()), C.c_void_p(w.data_ptr()), None, self._stream()))
        return ids, w

    def dispatch(self, ids: torch.Tensor, x: torch.Tensor, world: int) -> Dispatch:
        T, k = ids.shape
        P, dev, d = T * k, ids.device, self.d
        per_rank = self.E // world
        counts32 = torch.empty(world, dtype=torch.int32, device=dev)
        offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
        send_pairs = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        slot_of = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        send_x = torch.empty(max(P, 1), d, dtype=torch.float16, device=dev)
        send_e = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
        scratch = self._buf("dispatch", self.lib.fmcuda_ep_dispatch_scratch_bytes(T, k, world), dev)
        xdt = self.X_BF16 if x.dtype == torch.bfloat16 else self.X_F32
        self.check(self.lib.fmcuda_ep_dispatch(
            C.c_void_p(ids.data_ptr()), T, k, per_rank, world, C.c_void_p(x.data_ptr()), xdt, d,
            C.c_void_p(counts32.data_ptr()), C.c_void_p(offsets.data_ptr()), C.c_void_p(send_pairs.data_ptr()),
            C.c_void_p(slot_of.data_ptr()), C.c_void_p(send_x.data_ptr()), C.c_void_p(send_e.data_ptr()),
            C.c_void_p(scratch.data_ptr()), self._stream()))
        return Dispatch(counts32.to(torch.int64), send_x, send_e, slot_of)

    def empty_rows(self, n: int, like: torch.Tensor) -> torch.Tensor:
        return torch.empty(max(n, 1), self.d, dtype=like.dtype, device=like.device)

    def experts(self, rows: torch.Tensor, expert: torch.Tensor, n: int) -> torch.Tensor:
        dev = rows.device
        out = torch.empty(max(n, 1), self.d, dtype=torch.float32, device=dev)
        if n == 0:
            return out
        per_rank = len(self.slots)
        ws = self._buf("experts", self.lib.fmcuda_moe_experts_workspace_bytes(n, per_rank, self.d, self.ffn), dev)
        g, u, dn = self.types
        self.check(self.lib.fmcuda_moe_experts(
            C.c_void_p(rows.data_ptr()), C.c_void_p(expert.data_ptr()), n, per_rank, C.c_void_p(self.table.data_ptr()),
            self.up_offset, self.down_offset, g, u, dn, self.d, self.ffn, C.c_void_p(out.data_ptr()),
            C.c_void_p(ws.data_ptr()), ws.numel(), self._stream()))
        return out

    def dispatch_rows(self, ids: torch.Tensor, w: torch.Tensor, x: torch.Tensor, world: int) -> RowDispatch:
        T, k = ids.shape
        n, dev, d = T * world, ids.device, self.d
        counts32 = torch.empty(world, dtype=torch.int32, device=dev)
        offsets = torch.empty(world + 1, dtype=torch.int32, device=dev)
        items = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        row_of = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        send_x = torch.empty(max(n, 1), d, dtype=torch.float16, device=dev)
        meta_e = torch.empty(max(n, 1), k, dtype=torch.int32, device=dev)
        meta_w = torch.empty(max(n, 1), k, dtype=torch.float32, device=dev)
        scratch = self._buf("dispatch_rows", self.lib.fmcuda_ep_dispatch_rows_scratch_bytes(T, world), dev)
        xdt = self.X_BF16 if x.dtype == torch.bfloat16 else self.X_F32
        P = C.c_void_p
        self.check(self.lib.fmcuda_ep_dispatch_rows(
            P(ids.data_ptr()), P(w.data_ptr()), T, k, self.E // world, world, P(x.data_ptr()), xdt, d,
            P(counts32.data_ptr()), P(offsets.data_ptr()), P(items.data_ptr()), P(row_of.data_ptr()),
            P(send_x.data_ptr()), P(meta_e.data_ptr()), P(meta_w.data_ptr()), P(scratch.data_ptr()),
            self._stream()))
        return RowDispatch(counts32.to(torch.int64), send_x, meta_e, meta_w, row_of)

    def experts_partial(self, rows: torch.Tensor, meta_e: torch.Tensor, meta_w: torch.Tensor, n: int):
        dev = rows.device
        out = torch.empty(max(n, 1), self.d, dtype=torch.float32, device=dev)
        if n == 0:
            return out
        per_rank = len(self.slots)
        ws = self._buf("experts_partial", self.lib.fmcuda_moe_experts_partial_workspace_bytes(
            n, self.k, per_rank, self.d, self.ffn), dev)
        g, u, dn = self.types
        P = C.c_void_p
        self.check(self.lib.fmcuda_moe_experts_partial(
            P(rows.data_ptr()), P(meta_e.data_ptr()), P(meta_w.data_ptr()), n, self.k, per_rank,
            P(self.table.data_ptr()), self.up_offset, self.down_offset, g, u, dn, self.d, self.ffn,
            P(out.data_ptr()), P(ws.data_ptr()), ws.numel(), self._stream()))
        return out

    def combine_rows(self, back: torch.Tensor, row_of: torch.Tensor, tokens: int, world: int) -> torch.Tensor:
        y = torch.empty(tokens, self.d, dtype=torch.float32, device=back.device)
        self.check(self.lib.fmcuda_ep_combine_rows(C.c_void_p(back.data_ptr()), C.c_void_p(row_of.data_ptr()),
                                                   tokens, world, self.d, C.c_void_p(y.data_ptr()), self._stream()))
        return y

    # ---- exchange over peer memory (mode "p2p") ------------------------------

    def p2p_setup(self, world: int, rank: int, capacity: int, group=None, timeout_ms: int = 0):
        """Allocates this rank's mailbox, swaps IPC handles with the group and
        opens the peers' mailboxes (collective over `group`)."""
        dev = torch.device("cuda", torch.cuda.current_device())
        self.world, self.rank, self.capacity, self.timeout_ms = world, rank, capacity, timeout_ms
        nbytes = self.lib.fmcuda_ep_mailbox_bytes(world, capacity, self.k, self.d)
        mine, handle = C.c_void_p(), (C.c_ubyte * 64)()
        self.check(self.lib.fmcuda_ep_mailbox_alloc(nbytes, C.byref(mine), handle))
        self.mailbox = mine.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened, ptrs = [], []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(self.mailbox)
                continue
            buf, p = (C.c_ubyte * 64).from_buffer_copy(h), C.c_void_p()
            self.check(self.lib.fmcuda_ep_mailbox_open(buf, C.byref(p)))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=dev)
        dist.barrier(group=group)  # every mailbox is open before any rank writes

    def p2p_close(self, group=None):
        torch.cuda.synchronize()
        dist.barrier(group=group)  # nobody writes into a mailbox that is going away
        for p in getattr(self, "opened", []):
            self.lib.fmcuda_ep_mailbox_close(C.c_void_p(p))
        if getattr(self, "mailbox", None):
            self.lib.fmcuda_ep_mailbox_free(C.c_void_p(self.mailbox))
        self.opened, self.mailbox = [], None

    def p2p_dispatch(self, ids, w, x, epoch: int) -> torch.Tensor:
        T, k = ids.shape
        dev, world = ids.device, self.world
        row_of = torch.empty(max(T * world, 1), dtype=torch.int32, device=dev)
        scratch = self._buf("p2p_dispatch", self.lib.fmcuda_ep_p2p_dispatch_scratch_bytes(T, world), dev)
        xdt = self.X_BF16 if x.dtype == torch.bfloat16 else self.X_F32
        P = C.c_void_p
        self.check(self.lib.fmcuda_ep_p2p_dispatch(
            P(ids.data_ptr()), P(w.data_ptr()), T, k, self.E // world, world, self.rank, P(x.data_ptr()), xdt, self.d,
            P(self.mailbox), P(self.peers.data_ptr()), self.capacity, epoch, P(row_of.data_ptr()), P(scratch.data_ptr()),
            self.timeout_ms, self._stream()))
        return row_of

    def p2p_experts(self, epoch: int):
        dev = self.peers.device
        per_rank = len(self.slots)
        ws = self._buf("p2p_experts", self.lib.fmcuda_ep_p2p_experts_workspace_bytes(
            self.capacity, self.k, per_rank, self.d, self.ffn), dev)
        g, u, dn = self.types
        P = C.c_void_p
        self.check(self.lib.fmcuda_ep_p2p_experts(
            P(self.mailbox), P(self.peers.data_ptr()), self.world, self.rank, self.capacity, epoch, self.k, per_rank,
            P(self.table.data_ptr()), self.up_offset, self.down_offset, g, u, dn, self.d, self.ffn, P(ws.data_ptr()),
            ws.numel(), self.timeout_ms, self._stream()))

    def p2p_combine(self, row_of, tokens: int, epoch: int) -> torch.Tensor:
        y = torch.empty(tokens, self.d, dtype=torch.float32, device=row_of.device)
        self.check(self.lib.fmcuda_ep_p2p_combine(
            C.c_void_p(self.mailbox), self.world, self.rank, self.capacity, epoch, self.k, C.c_void_p(row_of.data_ptr()),
            tokens, self.d, C.c_void_p(y.data_ptr()), self.timeout_ms, self._stream()))
        return y

    def combine(self, back: torch.Tensor, w: torch.Tensor, slot_of: torch.Tensor) -> torch.Tensor:
        T = w.shape[0]
        y = torch.empty(T, self.d, dtype=torch.float32, device=w.device)
        self.check(self.lib.fmcuda_moe_combine(C.c_void_p(back.data_ptr()), C.c_void_p(w.data_ptr()),
                                               C.c_void_p(slot_of.data_ptr()), T, self.k, self.d,
                                               C.c_void_p(y.data_ptr()), self._stream()))
        return y


class EPLayer:
    """One expert-parallel MoE layer on the ranks of ``group``."""

    PHASES = ("route", "dispatch", "counts", "rows_out", "experts", "rows_back", "combine")

    def __init__(self, ops, group=None, record_timing: bool = False, mode: str = "rows", capacity: int = 0,
                 timeout_ms: int = 0, device_epoch: bool = False):
        if mode not in ("rows", "pairs", "p2p"):
            raise ValueError(f"unknown exchange mode {mode!r}")
        self.ops, self.group, self.mode = ops, group, mode
        self.record_timing = record_timing and torch.cuda.is_available()
        self._events = []
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if ops.E % self.world:
            raise ValueError(f"{ops.E} experts do not shard evenly over {self.world} ranks")
        self.timing = {}
        # mode "p2p": mailboxes are set up on the first call (capacity = the
        # largest tokens per rank of that call x world unless given)
        self.capacity, self.timeout_ms, self.epoch = capacity, timeout_ms, 0
        # mode "p2p" with device_epoch: the kernels number the calls themselves
        # (epoch 0 to the library), so forward() can be captured in a CUDA graph
        # once the mailboxes exist (after the first call) and replayed
        self.device_epoch = device_epoch

    def close(self):
        """Releases the peer mailboxes (mode "p2p"); collective over the group."""
        if self.mode == "p2p" and self.epoch:
            self.ops.p2p_close(self.group)
            self.epoch = 0

    def _forward_p2p(self, x, logits):
        ops = self.ops
        if self.epoch == 0:
            if not self.capacity:
                t = torch.tensor([x.shape[0]], dtype=torch.int64, device=x.device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
                self.capacity = int(t.item()) * self.world
            ops.p2p_setup(self.world, self.rank, self.capacity, self.group, self.timeout_ms)
        self.epoch += 1
        ep = 0 if self.device_epoch else self.epoch
        self._mark()
        ids, w = ops.route(logits)
        self._mark()
        row_of = ops.p2p_dispatch(ids, w, x, ep)
        self._mark()
        self._mark()  # counts: inside the dispatch kernels
        self._mark()  # rows out: written by the dispatch kernel
        ops.p2p_experts(ep)
        self._mark()  # the partial sums go back from the experts call
        self._mark()
        y = ops.p2p_combine(row_of, x.shape[0], ep)
        self._mark()
        return y

    def _mark(self):
        if self.record_timing:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append(e)

    def phase_ms(self) -> dict:
        """Mean milliseconds per phase over the calls since the last reset
        (record_timing=True); synchronises the device."""
        torch.cuda.synchronize()
        n = len(self.PHASES) + 1
        calls = [self._events[i:i + n] for i in range(0, len(self._events) - n + 1, n)]
        out = {ph: sum(c[j].elapsed_time(c[j + 1]) for c in calls) / max(len(calls), 1)
               for j, ph in enumerate(self.PHASES)}
        self._events = []
        return out

    def _exchange_counts(self, send_counts):
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = send_counts.cpu().tolist()  # the host needs both sides' sizes
        rc = recv_counts.cpu().tolist()
        return sc, rc

    def _a2a(self, out, inp, out_splits, in_splits):
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=self.group)

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        if self.mode == "p2p":
            return self._forward_p2p(x, logits)
        ops = self.ops
        self._mark()
        ids, w = ops.route(logits)
        self._mark()
        if self.mode == "pairs":
            plan = ops.dispatch(ids, x, self.world)
            self._mark()
            sc, rc = self._exchange_counts(plan.send_counts)
            S, R = int(sum(sc)), int(sum(rc))
            self._mark()
            recv_x = ops.empty_rows(R, plan.send_x)
            recv_e = torch.empty(max(R, 1), dtype=plan.send_expert.dtype, device=plan.send_expert.device)
            self._a2a(recv_x[:R], plan.send_x[:S], rc, sc)
            self._a2a(recv_e[:R], plan.send_expert[:S], rc, sc)
            self._mark()
            out = ops.experts(recv_x, recv_e, R)
            self._mark()
            back = torch.empty(max(S, 1), out.shape[1], dtype=out.dtype, device=out.device)
            self._a2a(back[:S], out[:R], sc, rc)
            self._mark()
            y = ops.combine(back, w, plan.slot_of)
        else:
            plan = ops.dispatch_rows(ids, w, x, self.world)
            self._mark()
            sc, rc = self._exchange_counts(plan.send_counts)
            S, R = int(sum(sc)), int(sum(rc))
            self._mark()
            k = plan.meta_e.shape[1]
            recv_x = ops.empty_rows(R, plan.send_x)
            recv_e = torch.empty(max(R, 1), k, dtype=plan.meta_e.dtype, device=plan.meta_e.device)
            recv_w = torch.empty(max(R, 1), k, dtype=plan.meta_w.dtype, device=plan.meta_w.device)
            self._a2a(recv_x[:R], plan.send_x[:S], rc, sc)
            self._a2a(recv_e[:R], plan.meta_e[:S], rc, sc)
            self._a2a(recv_w[:R], plan.meta_w[:S], rc, sc)
            self._mark()
            part = ops.experts_partial(recv_x, recv_e, recv_w, R)
            self._mark()
            back = torch.empty(max(S, 1), part.shape[1], dtype=part.dtype, device=part.device)
            self._a2a(back[:S], part[:R], sc, rc)
            self._mark()
            y = ops.combine_rows(back, plan.row_of, x.shape[0], self.world)
        self._mark()
        return y
