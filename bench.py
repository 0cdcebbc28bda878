#!/usr/bin/env python
"""Benchmark of the routed-expert MoE hot path on B200.

Workload (the fused dequant+GEMV microbench): one stack of
8 experts, each gate/up [14336 x 4096] and down [4096 x 14336] in GGUF Q4_K
(or Q8_0 with --type q8_0), seeded Gaussian weights N(0, 0.02) encoded on the
device; x = T bf16 tokens N(0, 1) (T = 8 by default, the top of the 1..8
range).  One step = one MoE block over the whole stack: router (softmax,
top-8 of 8), grouping, fused gate/up GEMV + SwiGLU, down GEMV, weighted combine
-- every expert's rows are streamed from HBM once.  The 792.7 MB Q4_K stack is
far larger than the 126 MB L2, so no flush is needed between steps.

metric/value: algorithmic HBM bytes of the step (stack bytes + x + y) / step
time, whole job over all ranks (weak scaling: every rank owns its own stack,
an expert-parallel partition with no data-path exchange for this workload).
e2e: the same metric through the C ABI with host buffers: pinned H2D of x and
the router logits and D2H of y inside every timed step, pipelined the way a
serving loop runs them: double-buffered device tensors, the H2D of step i+1 and
the D2H of step i-1 on two copy streams while step i computes.

--impl reference: the reference's own CPU code for the same step (its
gemv_quant and silu in the engine's per-token expert loop, compiled from
source into oracle/_ref; the C restatement if that is absent), on all host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "MoE-layer tokens/s + fused dequant-GEMV HBM GB/s (% of 8 TB/s), 1–8 B200"
D_MODEL, FFN, EXPERTS = 4096, 14336, 8
TYPES = {"q4_k": 12, "q8_0": 8}


def row_bytes(t, n):
    return n // 256 * 144 if t == 12 else n // 32 * 34


def expert_bytes(t):
    return 2 * FFN * row_bytes(t, D_MODEL) + D_MODEL * row_bytes(t, FFN)


def step_bytes(t, tokens):
    # weights streamed once + bf16 x read + f32 y written
    return EXPERTS * expert_bytes(t) + tokens * D_MODEL * 2 + tokens * D_MODEL * 4


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def stack_config(type_name: str, tokens: int, world: int) -> dict:
    """The headline workload's config, one dict for both arms (same keys, same
    strings), so that the two JSON lines name the same configuration."""
    t = TYPES[type_name]
    mb = EXPERTS * expert_bytes(t) / 1e6
    return {"workload": f"{type_name} 8-expert stack [{FFN}x{D_MODEL}]x2+[{D_MODEL}x{FFN}], "
                        f"T={tokens} bf16 tokens, top-8 of 8", "tokens": tokens,
            "parallelism": f"ep{world}",
            "l2": f"inputs larger than L2 ({mb:.1f} MB {type_name.upper()} stack vs 126 MB L2)"}


def host_cpu() -> dict:
    """The host CPU the baseline ran on: model name and the vector extensions
    the reference's kernels can use, plus the ISA the reference itself resolved
    (fm::resolved_isa) when its compiled code is present."""
    model, flags = None, set()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if model is None and line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                elif not flags and line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                if model and flags:
                    break
    except OSError:
        pass
    out = {"cpu_model": model, "cpu_flags": [f for f in ("avx2", "fma", "f16c", "avx512f") if f in flags]}
    try:
        from oracle.oracle import Reference, reference_available

        if reference_available():
            out["isa"] = Reference().isa()
    except Exception:  # noqa: BLE001 - the ISA is informative only
        pass
    return out


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.lines, self.proc = gpu, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def pipelined_e2e(call, hx, hl, like_x, like_l, like_y, steps, stream):
    """ms per step of `steps` calls that each take x and logits from pinned host
    memory and return y to pinned host memory: H2D on one copy stream, D2H on
    another, compute on `stream`, two buffers of each so step i+1's inputs and
    step i-1's result move while step i computes.  Returns (ms, host y)."""
    import torch

    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()
    dx = [torch.empty_like(like_x) for _ in range(2)]
    dl = [torch.empty_like(like_l) for _ in range(2)]
    dy = [torch.empty_like(like_y) for _ in range(2)]
    hy = [torch.empty(like_y.shape, dtype=like_y.dtype).pin_memory() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    returned = [torch.cuda.Event() for _ in range(2)]
    for b in range(2):  # every event recorded once, so the first waits are satisfied
        computed[b].record(stream)
        returned[b].record(stream)

    def step(i):
        b = i & 1
        with torch.cuda.stream(h2d_s):
            h2d_s.wait_event(computed[b])  # step i-2 has read dx[b], dl[b]
            dx[b].copy_(hx, non_blocking=True)
            dl[b].copy_(hl, non_blocking=True)
            in_ready[b].record(h2d_s)
        stream.wait_event(in_ready[b])
        stream.wait_event(returned[b])  # step i-2's y has left dy[b]
        call(dx[b], dl[b], dy[b])
        computed[b].record(stream)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(computed[b])
            hy[b].copy_(dy[b], non_blocking=True)
            returned[b].record(d2h_s)

    for i in range(2):
        step(i)
    torch.cuda.synchronize()
    e0, e1, start = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
                     torch.cuda.Event())
    e0.record(stream)
    start.record(stream)
    h2d_s.wait_event(start)
    for i in range(steps):
        step(i)
    stream.wait_event(returned[(steps - 1) & 1])
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps, hy[(steps - 1) & 1]


def report_stages(stage_ms: dict, tokens: int, experts: int = EXPERTS) -> dict:
    """Per-stage device times of one decode MoE block.  Up to 64 tokens and 64
    experts (plain router) the router, grouping and x planes (Q4_K: B images)
    are one launch and the down projection's x planes (images) are written by
    the gate/up epilogue, so the library's events between those stages time
    nothing: report the launches."""
    if tokens <= 64 and experts <= 64:
        return {"front": stage_ms["router"] + stage_ms["grouping"] + stage_ms["x_planes"],
                "gate_up": stage_ms["gate_up"] + stage_ms["act_planes"], "down": stage_ms["down"],
                "combine": stage_ms["combine"]}
    return dict(stage_ms)


# Further configurations measured by the default run after the headline, each
# in a child process of its own (BASELINE configs[1] in Q8_0 and at T = 1, the
# Mixtral-shaped decode layer at T = 1, 4, 16, 64, the DeepSeek- and
# Qwen3-shaped prefill layers); their lines are attached under "configs".
EXTRA_RUNS = (
    ("stack_q8_0_T8", ["--type", "q8_0"]),
    ("stack_q4_k_T1", ["--tokens", "1"]),
    ("mixtral_T1", ["--config", "mixtral", "--tokens", "1"]),
    ("mixtral_T4", ["--config", "mixtral", "--tokens", "4"]),
    ("mixtral_T16", ["--config", "mixtral", "--tokens", "16"]),
    ("mixtral_T64", ["--config", "mixtral", "--tokens", "64"]),
    ("deepseek_prefill_T4096", ["--config", "deepseek"]),
    ("qwen3_prefill_T8192", ["--config", "qwen3"]),
)
EXTRA_KEYS = ("metric", "value", "unit", "ms_per_step", "dtype", "config", "stage_ms", "roofline", "e2e",
              "cpu_baseline", "hbm_gbs", "tokens_per_s", "gpu_launches", "clocks", "steps", "warmup")


def run_extras(args) -> dict:
    env = {k: v for k, v in os.environ.items()
           if k not in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT")}
    out = {}
    for name, extra in EXTRA_RUNS:
        cmd = [sys.executable, str(Path(__file__).resolve()), "--steps", str(args.extra_steps), "--warmup", "3",
               "--no-extras", "--cpu-seconds", "3", *(["--no-cpu"] if args.no_cpu else []), *extra]
        try:
            p = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(ROOT))
        except subprocess.TimeoutExpired:
            out[name] = {"error": "timed out after 600 s"}
            continue
        lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
        if p.returncode or not lines:
            tail = (p.stderr or p.stdout).strip().splitlines()[-3:]
            out[name] = {"error": f"exit {p.returncode}: {' | '.join(tail)}"}
            continue
        d = json.loads(lines[-1])
        out[name] = {k: d[k] for k in EXTRA_KEYS if k in d}
    return out


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_step_reference(ref, type_id, host_slots, x, logits, tokens, threads, ffn=FFN):
    """One reference step on the CPU: router + per-token expert loop (engine.cpp:1603-1772)."""
    rc, ids, w, _ = ref.route(logits, EXPERTS)
    if rc:
        raise RuntimeError(f"reference router failed: {rc}")
    gb = ffn * row_bytes(type_id, D_MODEL)
    return ref.moe_block(type_id, host_slots, gb, 2 * gb, x, ids, w, D_MODEL, ffn, threads=threads)


def make_cpu_runner(type_id, host_slots, ffn=FFN):
    """The reference's own code when it was compiled here, else the C restatement."""
    from oracle.oracle import Oracle, Reference, reference_available

    if reference_available():
        ref = Reference()
        return "reference", lambda x, lg, T, th: cpu_step_reference(ref, type_id, host_slots, x, lg, T, th, ffn)
    orc = Oracle()

    def port(x, lg, T, th):
        rc, ids, w, _ = orc.route(lg, EXPERTS)
        return orc.moe_block(x, ids, w, host_slots, D_MODEL, ffn, type_id)
    return "port", port


def row_sample_slots(type_id, host_slots, ffn):
    """The first `ffn` feature rows of every expert: gate/up rows 0..ffn-1 and the
    matching leading blocks of each down row (a bounded sample of the step)."""
    import numpy as np

    gb = FFN * row_bytes(type_id, D_MODEL)
    sb = ffn * row_bytes(type_id, D_MODEL)
    out = []
    for s in host_slots:
        down = s[2 * gb:].reshape(D_MODEL, row_bytes(type_id, FFN))[:, :row_bytes(type_id, ffn)]
        out.append(np.concatenate([s[:sb], s[gb:gb + sb], down.reshape(-1)]))
    return out


def host_inputs(tokens, seed=0):
    import numpy as np
    from oracle.oracle import bf16_round

    rng = np.random.default_rng(seed)
    x = bf16_round(rng.normal(0, 1, size=(tokens, D_MODEL)).astype(np.float32))
    logits = rng.normal(0, 1, size=(tokens, EXPERTS)).astype(np.float32)
    return x, logits


def synth_host_slots(type_id, seed):
    """Expert payloads on the host: the device encoder when a GPU is present
    (identical bytes to the GPU arm), else the C restatement's encoder."""
    import numpy as np

    try:
        import torch

        if torch.cuda.is_available():
            from freemoe_b200 import hotpath

            hotpath.init(0)
            out = []
            for e in range(EXPERTS):
                parts = [hotpath.synth_weights(type_id, rows, cols, seed=seed * 1000 + 3 * e + j)
                         for j, (rows, cols) in enumerate(((FFN, D_MODEL), (FFN, D_MODEL), (D_MODEL, FFN)))]
                out.append(torch.cat(parts).cpu().numpy())
            return out
    except Exception:  # noqa: BLE001 - no usable GPU: fall back to the host encoder
        pass
    from oracle.oracle import Oracle

    orc = Oracle()
    rng = np.random.default_rng(seed)
    return [np.concatenate([orc.quantize(type_id, rng.normal(0, 0.02, n).astype(np.float32))
                            for n in (FFN * D_MODEL, FFN * D_MODEL, D_MODEL * FFN)]) for _ in range(EXPERTS)]


REF_BUDGET_S = 60.0


def run_reference(args):
    world, rank, local = dist_setup(args)
    if rank != 0:
        return
    type_id = TYPES[args.type]
    threads = os.cpu_count() or 1
    host_slots = synth_host_slots(type_id, seed=1)
    kind, runner = make_cpu_runner(type_id, host_slots)
    x, logits = host_inputs(args.tokens)
    # each step is a bounded sample: the full step, or the leading 1/2, 1/4 or
    # 1/8 of every expert's feature rows when K full steps would exceed
    # REF_BUDGET_S (same experts, tokens and threads; bytes scale with the rows)
    t0 = time.perf_counter()
    runner(x, logits, args.tokens, threads)
    t_full = time.perf_counter() - t0
    frac = 1
    while frac < 8 and args.steps * t_full / frac > REF_BUDGET_S:
        frac *= 2
    ffn = FFN // frac
    if frac > 1:
        kind, runner = make_cpu_runner(type_id, row_sample_slots(type_id, host_slots, ffn), ffn)
    for _ in range(args.warmup):
        runner(x, logits, args.tokens, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        runner(x, logits, args.tokens, threads)
    dt = (time.perf_counter() - t0) / args.steps
    nbytes = EXPERTS * 3 * ffn * row_bytes(type_id, D_MODEL) + args.tokens * D_MODEL * 6
    value = nbytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": args.type, "data": "synthetic",
        "config": stack_config(args.type, args.tokens, args.gpus),
        "tokens_per_s": args.tokens / (dt * frac),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": kind,
                         "sample": f"{EXPERTS} experts x {args.tokens} tokens, feature rows 0..{ffn - 1} of "
                                   f"{FFN} per step (full step {t_full * 1e3:.0f} ms)", **host_cpu()},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200._lib import MOE_STAGES, check, load

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    hotpath.init(local)
    type_id = TYPES[args.type]
    T = args.tokens
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()

    # expert slots: one 256-aligned HBM slab per expert holding gate || up || down
    eb = expert_bytes(type_id)
    gb = FFN * row_bytes(type_id, D_MODEL)
    slots = []
    for e in range(EXPERTS):
        slab = torch.empty(eb, dtype=torch.uint8, device=dev)
        off = 0
        for j, (rows, cols) in enumerate(((FFN, D_MODEL), (FFN, D_MODEL), (D_MODEL, FFN))):
            n = rows * row_bytes(type_id, cols)
            check(load().fmcuda_synth_weights(type_id, C.c_void_p(slab.data_ptr() + off), rows, cols,
                                              1000 * (rank + 1) + 3 * e + j, 0.02, stream.cuda_stream))
            off += n
        slots.append(slab)
    table = hotpath.slot_table(slots, dev)
    x_np, lg_np = host_inputs(T, seed=rank)
    x = torch.from_numpy(x_np).to(dev).to(torch.bfloat16)
    logits = torch.from_numpy(lg_np).to(dev)
    y = torch.empty(T, D_MODEL, dtype=torch.float32, device=dev)
    ws = torch.empty(hotpath.moe_workspace_bytes(T, EXPERTS, EXPERTS, D_MODEL, FFN), dtype=torch.uint8,
                     device=dev)
    n_ev = len(MOE_STAGES) + 1
    lib = load()

    def timing_event():
        h = C.c_void_p()
        check(lib.fmcuda_event_create_timing(C.byref(h)))
        return h.value

    # library-owned timing events, recorded by fmcuda_moe_block between its stages
    ev_pool = [[timing_event() for _ in range(n_ev)] for _ in range(min(args.steps, 500))]
    ev_arrays = [(C.c_void_p * n_ev)(*evs) for evs in ev_pool]

    def elapsed(a, b):
        v = C.c_float()
        check(lib.fmcuda_event_elapsed_ms(C.c_void_p(a), C.c_void_p(b), C.byref(v)))
        return v.value
    ws_ptr, ws_n, sptr = C.c_void_p(ws.data_ptr()), ws.numel(), stream.cuda_stream

    arg_cache = {}

    def call(xt, lgt, yt, events=None):
        key = (xt.data_ptr(), lgt.data_ptr(), yt.data_ptr())
        a = arg_cache.get(key)
        if a is None:
            a = hotpath.moe_args(xt, lgt, table, experts=EXPERTS, top_k=EXPERTS, d_model=D_MODEL, ffn=FFN,
                                 gate_type=type_id, up_type=type_id, down_type=type_id, up_offset=gb,
                                 down_offset=2 * gb, y=yt)
            arg_cache[key] = a
        a.stage_events = C.cast(events, C.c_void_p) if events is not None else None
        check(lib.fmcuda_moe_block(C.byref(a), ws_ptr, ws_n, sptr))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # correctness guard on a slice: the step's routing must be every expert
    for _ in range(args.warmup):
        call(x, logits, y)
    barrier()
    assert hotpath.device_status() == 0

    # ---- device-resident timing (value): no per-stage events in this loop ----
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record(stream)
        for i in range(args.steps):
            call(x, logits, y)
        end.record(stream)
        barrier()
    ms = start.elapsed_time(end) / args.steps

    # ---- per-stage device times (library-recorded events), a second pass -------
    n_stage_steps = len(ev_pool)
    barrier()
    for i in range(n_stage_steps):
        call(x, logits, y, ev_arrays[i])
    barrier()
    stage_ms = {s: statistics.mean(elapsed(ev_pool[i][j], ev_pool[i][j + 1]) for i in range(n_stage_steps))
                for j, s in enumerate(MOE_STAGES)}
    for evs in ev_pool:
        for e in evs:
            lib.fmcuda_event_destroy(C.c_void_p(e))

    # ---- end to end through the C ABI with host buffers ----------------------
    hx = torch.from_numpy(x_np).to(torch.bfloat16).pin_memory()
    hl = torch.from_numpy(lg_np).pin_memory()
    h2d = hx.numel() * 2 + hl.numel() * 4
    d2h = y.numel() * 4
    barrier()
    ms_e2e, hy = pipelined_e2e(call, hx, hl, x, logits, y, args.steps, stream)
    barrier()
    assert np.isfinite(hy.numpy()).all()
    assert hotpath.device_status() == 0

    # ---- max over ranks --------------------------------------------------------
    vals = torch.tensor([ms, ms_e2e, stage_ms["gate_up"], stage_ms["down"]], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, ms_e2e, gu_ms, dn_ms = vals.tolist()
    nbytes = step_bytes(type_id, T)
    value = world * nbytes / (ms / 1e3) / 1e9
    e2e = world * nbytes / (ms_e2e / 1e3) / 1e9

    peak, peak_kind = load_peaks()
    # dominant kernel: the fused gate/up GEMV + SwiGLU over the 8 experts
    gu_bytes = EXPERTS * 2 * FFN * row_bytes(type_id, D_MODEL) + T * D_MODEL * 2 + EXPERTS * T * FFN * 4
    gu_achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    traffic = None
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get(f"gate_up_{args.type}_T{T}")

    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.type, "data": "synthetic",
        "config": stack_config(args.type, T, world),
        "entry_point": "fmcuda_moe_block (one call per step)",
        "tokens_per_s": world * T / (ms / 1e3),
        "pct_of_8tbs": value / world / 8000.0 * 100.0,
        "stage_ms": report_stages(stage_ms, T),
        "roofline": {"bound": "hbm", "kernel": ("tgemv_kernel<0> gate/up + SwiGLU (tcgen05), 8 experts" if type_id == 12
                                                else "qgemv_async_kernel gate/up + SwiGLU (mma.sync), 8 experts"),
                     "achieved": gu_achieved,
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s", "frac": gu_achieved / peak,
                     "traffic": traffic, "algorithmic_bytes": gu_bytes,
                     "down_achieved": (EXPERTS * D_MODEL * row_bytes(type_id, FFN)) / (dn_ms / 1e3) / 1e9},
        "e2e": {"value": e2e, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": ms_e2e},
        # Q4_K: router + grouping + B images, gate/up (+ down's B images), down, combine;
        # Q8_0: router + grouping + x planes, gate/up (+ down's x planes), down, combine
        "gpu_launches": 4 * args.steps,
        "clocks": clocks.summary(),
    }

    # ---- CPU baseline (rank 0, N = 1): bounded sample on the host cores -------
    if rank == 0 and world == 1 and not args.no_cpu:
        host_slots = [s.cpu().numpy() for s in slots]
        kind, runner = make_cpu_runner(type_id, host_slots)
        threads = os.cpu_count() or 1
        runner(x_np, lg_np, T, threads)
        n, t0 = 0, time.perf_counter()
        while n < 3 or (time.perf_counter() - t0 < args.cpu_seconds and n < 50):
            runner(x_np, lg_np, T, threads)
            n += 1
        dt = (time.perf_counter() - t0) / n
        line["cpu_baseline"] = {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
                                "sample": f"{n} full steps ({EXPERTS} experts x {T} tokens), "
                                          f"{dt * 1e3:.1f} ms each", **host_cpu()}
    if rank == 0 and world == 1 and not args.no_extras:
        line["configs"] = run_extras(args)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Layer configurations beside the headline stack (BASELINE configs[2..4]):
# prefill of a DeepSeek-shaped layer and a Qwen3-shaped layer on the tcgen05
# grouped GEMM (fmcuda_moe_prefill), and the Mixtral-shaped decode layer on the
# GEMV path (fmcuda_moe_block).  One step = one MoE block over the config's
# tokens; value = tokens/s; roofline of the dominant kernel against the
# measured dense bf16 peak (tensor-bound prefill) or HBM (decode).
# ---------------------------------------------------------------------------

LAYERS = {
    # name: experts, top_k, d_model, ffn, type, tokens, logits, shared_ffn
    "deepseek": dict(E=64, k=6, d=2048, ffn=1408, t=8, T=4096, logits="zipf", shared=2816),
    "qwen3": dict(E=128, k=8, d=4096, ffn=1536, t=12, T=8192, logits="uniform", shared=0),
    "mixtral": dict(E=8, k=2, d=4096, ffn=14336, t=12, T=16, logits="normal", shared=0),
}


def layer_inputs(cfg, tokens, seed):
    import numpy as np
    from oracle.oracle import bf16_round

    rng = np.random.default_rng(seed)
    x = bf16_round(rng.normal(0, 1, size=(tokens, cfg["d"])).astype(np.float32))
    E = cfg["E"]
    if cfg["logits"] == "zipf":
        # Zipf(1.1) expert popularity, ranks permuted, Gumbel-top-k sampling
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        logp = np.log(p / p.sum())[rng.permutation(E)]
        lg = logp[None, :] + rng.gumbel(size=(tokens, E))
    elif cfg["logits"] == "uniform":
        lg = rng.uniform(-1, 1, size=(tokens, E))
    else:
        lg = rng.normal(0, 1, size=(tokens, E))
    return x, lg.astype(np.float32)


def layer_flops(cfg, pairs, tokens):
    routed = 2 * pairs * 3 * cfg["d"] * cfg["ffn"]
    shared = 2 * tokens * 3 * cfg["d"] * cfg["shared"]
    return routed, shared


def run_layer(args):
    import numpy as np
    import torch

    from freemoe_b200 import hotpath
    from freemoe_b200._lib import PREFILL_STAGES, MOE_STAGES, check, load

    cfg = dict(LAYERS[args.config])
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    hotpath.init(local)
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream()
    lib = load()
    E, k, d, ffn, t = cfg["E"], cfg["k"], cfg["d"], cfg["ffn"], cfg["t"]
    T = args.tokens if args.tokens_set else cfg["T"]
    prefill = args.config != "mixtral"
    rb_in, rb_ffn = row_bytes(t, d), row_bytes(t, ffn)
    gb = ffn * rb_in
    slots = []
    for e in range(E):
        slab = torch.empty(2 * gb + d * rb_ffn, dtype=torch.uint8, device=dev)
        off = 0
        for j, (rows, cols) in enumerate(((ffn, d), (ffn, d), (d, ffn))):
            check(lib.fmcuda_synth_weights(t, C.c_void_p(slab.data_ptr() + off), rows, cols,
                                           1000 * (rank + 1) + 3 * e + j, 0.02, stream.cuda_stream))
            off += rows * row_bytes(t, cols)
        slots.append(slab)
    table = hotpath.slot_table(slots, dev)
    shared = None
    if cfg["shared"]:
        sf = cfg["shared"]
        sh_slab = torch.cat([hotpath.synth_weights(t, sf, d, 77001), hotpath.synth_weights(t, sf, d, 77002),
                             hotpath.synth_weights(t, d, sf, 77003)])
        shared = hotpath.shared_expert_args(sh_slab, d_model=d, ffn=sf, gate_type=t)
    x_np, lg_np = layer_inputs(cfg, T, seed=rank + 1)
    x = torch.from_numpy(x_np).to(dev).to(torch.bfloat16)
    logits = torch.from_numpy(lg_np).to(dev)
    y = torch.empty(T, d, dtype=torch.float32, device=dev)
    ids = torch.empty(T, k, dtype=torch.int32, device=dev)
    if prefill:
        need = hotpath.moe_prefill_workspace_bytes(T, E, k, d, ffn, cfg["shared"])
    else:
        need = hotpath.moe_workspace_bytes(T, E, k, d, ffn)
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    n_ev = len(MOE_STAGES) + 1

    def timing_event():
        h = C.c_void_p()
        check(lib.fmcuda_event_create_timing(C.byref(h)))
        return h.value

    ev_pool = [[timing_event() for _ in range(n_ev)] for _ in range(min(args.steps, 200))]
    ev_arrays = [(C.c_void_p * n_ev)(*evs) for evs in ev_pool]

    def elapsed(a, b):
        v = C.c_float()
        check(lib.fmcuda_event_elapsed_ms(C.c_void_p(a), C.c_void_p(b), C.byref(v)))
        return v.value

    arg_cache = {}
    sh_ref = C.byref(shared) if shared is not None else None

    def call(xt, lgt, yt, events=None):
        key = (xt.data_ptr(), lgt.data_ptr(), yt.data_ptr())
        a = arg_cache.get(key)
        if a is None:
            a = hotpath.moe_args(xt, lgt, table, experts=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t,
                                 down_type=t, up_offset=gb, down_offset=2 * gb, y=yt, ids_out=ids)
            arg_cache[key] = a
        a.stage_events = C.cast(events, C.c_void_p) if events is not None else None
        if prefill:
            check(lib.fmcuda_moe_prefill(C.byref(a), sh_ref, C.c_void_p(ws.data_ptr()), ws.numel(),
                                         stream.cuda_stream))
        else:
            check(lib.fmcuda_moe_block(C.byref(a), C.c_void_p(ws.data_ptr()), ws.numel(), stream.cuda_stream))

    for _ in range(args.warmup):
        call(x, logits, y)
    torch.cuda.synchronize()
    assert hotpath.device_status() == 0
    ids_np = ids.cpu().numpy()
    counts = np.bincount(ids_np.ravel(), minlength=E)
    pairs = int(counts.sum())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(args.steps):
            call(x, logits, y)
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    # per-stage device times from the library's events, in a second pass
    for i in range(len(ev_pool)):
        call(x, logits, y, ev_arrays[i])
    torch.cuda.synchronize()
    names = PREFILL_STAGES if prefill else MOE_STAGES
    stage_ms = {s: statistics.mean(elapsed(ev_pool[i][j], ev_pool[i][j + 1]) for i in range(len(ev_pool)))
                for j, s in enumerate(names) if s != "none"}
    for evs in ev_pool:
        for e in evs:
            lib.fmcuda_event_destroy(C.c_void_p(e))

    # end to end with host buffers
    hx = torch.from_numpy(x_np).to(torch.bfloat16).pin_memory()
    hl = torch.from_numpy(lg_np).pin_memory()
    ms_e2e, hy = pipelined_e2e(call, hx, hl, x, logits, y, args.steps, stream)
    assert np.isfinite(hy.numpy()).all()
    assert hotpath.device_status() == 0

    line = {"metric": METRIC, "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": {8: "q8_0", 12: "q4_k"}[t] + (" -> fp16 tensor cores" if prefill else ""),
            "data": "synthetic",
            "config": {"workload": f"{args.config}: {E} experts d {d} ffn {ffn} top-{k}"
                                   + (f" + shared ffn {cfg['shared']}" if cfg["shared"] else "")
                                   + f", T={T} bf16 tokens, {cfg['logits']} router logits",
                       "tokens": T, "pairs": pairs, "experts_hit": int((counts > 0).sum()),
                       "max_group": int(counts.max()), "min_group": int(counts.min()),
                       "l2": "expert weights larger than L2"},
            "stage_ms": stage_ms if prefill else report_stages(stage_ms, T, E),
            "e2e": {"value": T / (ms_e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": hx.numel() * 2 + hl.numel() * 4,
                    "d2h_bytes_per_step": y.numel() * 4, "ms_per_step": ms_e2e},
            "gpu_launches": None, "clocks": clocks.summary()}
    if prefill:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        peak = float(peaks.get("bf16_tflops", 1590.0))
        routed, sh = layer_flops(cfg, pairs, T)
        gu_flops = 2 * pairs * 2 * d * ffn
        gu_ms = stage_ms["gate_up"]
        line["roofline"] = {"bound": "tensor", "kernel": "grouped GEMM gate/up + SwiGLU (tcgen05)",
                            "achieved": gu_flops / (gu_ms / 1e3) / 1e12, "peak": peak,
                            "peak_kind": "measured" if peaks else "fallback", "unit": "TFLOP/s",
                            "frac": gu_flops / (gu_ms / 1e3) / 1e12 / peak, "traffic": None,
                            "algorithmic_flops": gu_flops,
                            "down_achieved": 2 * pairs * d * ffn / (stage_ms["down"] / 1e3) / 1e12,
                            "step_achieved": (routed + sh) / (ms / 1e3) / 1e12,
                            "step_frac": (routed + sh) / (ms / 1e3) / 1e12 / peak}
        # 3 launches before the GEMMs (route, group, gather), 2 GEMMs, combine,
        # and for the shared expert: group, 2 GEMMs, add
        line["gpu_launches"] = (6 + (4 if cfg["shared"] else 0)) * args.steps
    else:
        hit = int((counts > 0).sum())
        wbytes = hit * (2 * gb + d * rb_ffn)
        peak, kind = load_peaks()
        line["hbm_gbs"] = wbytes / (ms / 1e3) / 1e9
        line["roofline"] = {"bound": "hbm", "kernel": "MoE block (distinct experts' bytes)",
                            "achieved": line["hbm_gbs"], "peak": peak, "peak_kind": kind, "unit": "GB/s",
                            "frac": line["hbm_gbs"] / peak, "traffic": None, "algorithmic_bytes": wbytes}
        line["gpu_launches"] = 4 * args.steps

    if not args.no_cpu:
        # the reference's CPU code on a bounded sample of the same tokens
        from oracle.oracle import Reference, reference_available

        if reference_available():
            ref = Reference()
            host_slots = [s.cpu().numpy() for s in slots]
            threads = os.cpu_count() or 1
            n_s = min(T, 64 if prefill else T)
            rc, ids_r, w_r, _ = ref.route(lg_np[:n_s], k)
            t0 = time.perf_counter()
            ref.moe_block(t, host_slots, gb, 2 * gb, x_np[:n_s], ids_r, w_r, d, ffn, threads=threads)
            dt = time.perf_counter() - t0
            line["cpu_baseline"] = {"value": n_s / dt, "unit": "tokens/s", "cores": threads, "kind": "reference",
                                    "sample": f"{n_s} of the {T} tokens (routed experts only), {dt:.2f} s",
                                    **host_cpu()}
    print(json.dumps(line), flush=True)


# The quantised GEMV shapes of the reference's own kernel benchmark
# (`freemoe bench`, src/main.cpp:631-637): attention projections, a small
# expert and the output head, one token.
GEMV_SHAPES = (
    ("qkv_1280x1280_q8_0", 1280, 1280, 8),
    ("qkv_1280x1280_q4_k", 1280, 1280, 12),
    ("expert_gate_1792x1280_q4_k", 1792, 1280, 12),
    ("expert_down_1280x1792_q4_k", 1280, 1792, 12),
    ("output_head_32000x1280_q4_k", 32000, 1280, 12),
)


def run_gemv_shapes(args):
    """fmcuda_gemv on the reference benchmark's quantised GEMV shapes at T=1
    (bf16 x), device-resident and through host buffers, beside the reference's
    own gemv_quant on the host cores."""
    import numpy as np
    import torch

    from freemoe_b200 import hotpath

    hotpath.init(0)
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    rows = []
    ref = None
    if not args.no_cpu:
        from oracle.oracle import Reference, reference_available

        ref = Reference() if reference_available() else None
    with ClockSampler(0) as clocks:
        for label, out_dim, in_dim, t in GEMV_SHAPES:
            w = hotpath.synth_weights(t, out_dim, in_dim, seed=11)
            x = torch.randn(1, in_dim, device=dev).to(torch.bfloat16)
            y = torch.empty(1, out_dim, dtype=torch.float32, device=dev)
            lib = hotpath.load()
            gs = torch.cuda.Stream()
            call = (t, C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()), 1, C.c_void_p(y.data_ptr()), 1, out_dim,
                    in_dim, C.c_void_p(gs.cuda_stream))
            with torch.cuda.stream(gs):
                for _ in range(max(args.warmup, 3)):
                    hotpath.check(lib.fmcuda_gemv(*call))
            torch.cuda.synchronize()
            # device time: the calls captured once into a CUDA graph (host launch
            # overhead out of the measurement), replayed
            reps = 100
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=gs):
                for _ in range(reps):
                    hotpath.check(lib.fmcuda_gemv(*call))
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n_rep = max(1, args.steps // reps)
            e0.record(stream)
            for _ in range(n_rep):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / (n_rep * reps) * 1e3
            del graph
            hx = x.cpu().pin_memory()
            hy = torch.empty(1, out_dim, dtype=torch.float32).pin_memory()
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(args.steps):
                dx = hx.to(dev, non_blocking=True)
                y = hotpath.gemv_quant(t, w, dx, out_dim, in_dim)
                hy.copy_(y, non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize()
            us_e2e = e0.elapsed_time(e1) / args.steps * 1e3
            nbytes = out_dim * row_bytes(t, in_dim)
            row = {"shape": label, "us": us, "gbytes_per_s": nbytes / us / 1e3, "e2e_us": us_e2e,
                   "weights_bytes": nbytes, "l2": "weights L2-resident between calls" if nbytes < 100e6 else "HBM"}
            if ref is not None:
                wh = w.cpu().numpy()
                xh = x.float().cpu().numpy().ravel()
                threads = os.cpu_count() or 1
                ref.gemv_quant(t, wh, xh, out_dim, in_dim, threads=threads)
                n, t0 = 0, time.perf_counter()
                while n < 20 or time.perf_counter() - t0 < 1.0:
                    ref.gemv_quant(t, wh, xh, out_dim, in_dim, threads=threads)
                    n += 1
                cpu_us = (time.perf_counter() - t0) / n * 1e6
                row["reference_cpu_us"] = cpu_us
                row["reference_cpu_gbytes_per_s"] = nbytes / cpu_us / 1e3
                row["reference_cpu_threads"] = threads
            rows.append(row)
    head = rows[-1]
    line = {"metric": METRIC, "value": head["gbytes_per_s"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": head["us"] / 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k/q8_0", "data": "synthetic",
            "config": {"workload": "quantised GEMV shapes of the reference kernel benchmark (src/main.cpp:631-637), "
                                   "T=1 bf16; value = output head", "tokens": 1},
            "shapes": rows, "gpu_launches": args.steps * 2, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


COLD_RECORDS = 8
COLD_METRIC = "cold expert-record load GB/s (model file -> HBM slot, FNV-1a checked), Mixtral Q4_K records"


def cold_model_file(records: int):
    """A synthetic model file holding `records` Mixtral-shaped Q4_K expert records
    in three stacked tensors (gate, up, down), like ffn_{gate,up,down}_exps; returns
    (path, [[(offset, size)] * 3] per record, payload bytes, tmp dir).  Random bytes:
    the path moves and checksums bytes, it does not decode them."""
    import tempfile

    import numpy as np

    sizes = [FFN * row_bytes(TYPES["q4_k"], D_MODEL)] * 2 + [D_MODEL * row_bytes(TYPES["q4_k"], FFN)]
    d = tempfile.mkdtemp(prefix="fm_cold_")
    path = os.path.join(d, "experts.gguf")
    header = 4096 + 123  # tensor data starts unaligned
    starts = [header, header + records * sizes[0], header + records * (sizes[0] + sizes[1])]
    total = starts[2] + records * sizes[2]
    rng = np.random.default_rng(7)
    with open(path, "wb") as f:
        left = total
        while left:
            n = min(left, 64 << 20)
            f.write(rng.integers(0, 256, n, dtype=np.uint8).tobytes())
            left -= n
    recs = [[(starts[j] + r * sizes[j], sizes[j]) for j in range(3)] for r in range(records)]
    return path, recs, sum(sizes), d


def cold_checksums(path, recs):
    from oracle.oracle import Oracle

    import numpy as np

    orc = Oracle()
    raw = np.memmap(path, dtype=np.uint8, mode="r")
    return [orc.fnv1a64(np.concatenate([raw[o:o + s] for o, s in rec])) for rec in recs]


def run_coldload(args):
    """--config coldload: one step = one expert record from the model file into an
    HBM slot through the C-ABI loader (pread by 8 reader threads into pinned
    rings, cudaMemcpyAsync, FNV-1a 64 of the slot on the device, checked against
    the record checksum), the demand load of ResidencyManager::load_slot
    (src/residency.cpp:624-724).  Page cache warm: the file is written just
    before; buffered reads."""
    import shutil

    import torch

    from freemoe_b200 import _lib as FL
    from freemoe_b200 import coldtier, hotpath

    world, rank, local = dist_setup(args)
    hotpath.init(local)
    dev = torch.device("cuda", local)
    path, recs, payload, tmp = cold_model_file(COLD_RECORDS)
    try:
        sums = cold_checksums(path, recs)
        slot = torch.empty(payload, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        steps = args.steps if args.steps != 2000 else 200
        with coldtier.RecordLoader(path, "buffered") as ld:
            for i in range(args.warmup):
                ld.read_record_into(recs[i % COLD_RECORDS], slot, checksum=sums[i % COLD_RECORDS])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(local) as clocks:
                e0.record(stream)
                for i in range(steps):
                    ld.read_record_into(recs[i % COLD_RECORDS], slot, checksum=sums[i % COLD_RECORDS])
                e1.record(stream)
                torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / steps
        # the device FNV alone (the loader's only kernels), CUDA events on its stream
        lib = FL.load()
        out = torch.empty(1, dtype=torch.int64, device=dev)
        ws = torch.empty(int(lib.fmcuda_fnv1a64_workspace_bytes(payload)), dtype=torch.uint8, device=dev)
        call = (C.c_void_p(slot.data_ptr()), payload, C.c_void_p(out.data_ptr()), C.c_void_p(ws.data_ptr()),
                ws.numel(), C.c_void_p(stream.cuda_stream))
        for _ in range(3):
            FL.check(lib.fmcuda_fnv1a64(*call))
        reps = 50
        e0.record(stream)
        for _ in range(reps):
            FL.check(lib.fmcuda_fnv1a64(*call))
        e1.record(stream)
        torch.cuda.synchronize()
        fnv_ms = e0.elapsed_time(e1) / reps
        # the ceiling: a plain pinned host -> device copy of one record
        h = torch.empty(payload, dtype=torch.uint8).pin_memory()
        for _ in range(2):
            slot.copy_(h, non_blocking=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(5):
            slot.copy_(h, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        h2d = payload / (e0.elapsed_time(e1) / 5) / 1e6
        del h
        cpu = None
        if not args.no_cpu and rank == 0:
            from oracle.oracle import Reference, reference_available

            if reference_available():
                import numpy as np

                ref = Reference()
                hslot = np.empty(payload, dtype=np.uint8)
                ext = np.array(recs, dtype=np.uint64)
                t0 = time.perf_counter()
                n = ref.load_records_cpu(path, 1, 4096, ext, np.array(sums, np.uint64), hslot)
                dt = time.perf_counter() - t0
                cpu = {"value": n * payload / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
                       "sample": f"{n} records: ReadScheduler::read_record (buffered) + fnv1a64 + memcpy into the "
                                 f"slot + fnv1a64 of the slot copy, the reference's own code"}
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    peak, peak_kind = load_peaks()
    value = payload / ms / 1e6
    fnv_gbs = payload / fnv_ms / 1e6
    line = {"metric": COLD_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": f"{COLD_RECORDS} Mixtral Q4_K expert records of {payload / 1e6:.1f} MB "
                                   f"(3 extents at unaligned offsets), cycled; buffered reads, page cache warm",
                       "record_bytes": payload, "reader_threads": 8, "chunk_bytes": 4 << 20,
                       "l2": "inputs larger than L2 (99 MB record per step, 8 records cycled)"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": payload, "d2h_bytes_per_step": 8},
            "roofline": {"bound": "hbm", "kernel": "fnv_round_kernel x8 + fnv_final_kernel (per record)",
                         "achieved": fnv_gbs, "peak": peak, "unit": "GB/s", "frac": fnv_gbs / peak,
                         "peak_kind": peak_kind, "traffic": None},
            "h2d_ceiling": {"pinned_copy_GBps": h2d, "frac": value / h2d},
            "gpu_launches": steps * 10, "clocks": clocks.summary()}
    if cpu:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference_coldload(args):
    """--impl reference --config coldload: the reference's own demand-load data path
    (fmr_load_records_cpu over ReadScheduler::read_record, fnv1a64, the CPU
    backend's memcpy upload and the slot checksum), on the same records."""
    import shutil

    import numpy as np

    world, rank, local = dist_setup(args)
    if rank != 0:
        return
    from oracle.oracle import Reference

    path, recs, payload, tmp = cold_model_file(COLD_RECORDS)
    try:
        sums = cold_checksums(path, recs)
        ref = Reference()
        hslot = np.empty(payload, dtype=np.uint8)
        one = lambda i: ref.load_records_cpu(path, 1, 4096, np.array([recs[i % COLD_RECORDS]], np.uint64),
                                             np.array([sums[i % COLD_RECORDS]], np.uint64), hslot)
        t0 = time.perf_counter()
        one(0)
        t_one = time.perf_counter() - t0
        steps = max(1, min(args.steps, int(REF_BUDGET_S / max(t_one, 1e-3))))
        for i in range(min(args.warmup, 3)):
            one(i)
        t0 = time.perf_counter()
        for i in range(steps):
            one(i)
        dt = (time.perf_counter() - t0) / steps
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    value = payload / dt / 1e9
    line = {"impl": "reference", "metric": COLD_METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": {"workload": f"{COLD_RECORDS} Mixtral Q4_K expert records of {payload / 1e6:.1f} MB, cycled; "
                                   f"buffered reads, page cache warm", "record_bytes": payload},
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": 1, "kind": "reference",
                             "sample": f"{steps} of the --steps records (the arm is bounded to ~{REF_BUDGET_S:.0f} s)"},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference_layer(args):
    """--impl reference --config deepseek|qwen3|mixtral: the reference's own
    per-token expert loop (gemv_quant + silu, compiled from source into
    oracle/_ref) on the host cores, over a bounded sample of the config's tokens."""
    world, rank, local = dist_setup(args)
    if rank != 0:
        return
    import numpy as np

    from oracle.oracle import Oracle, Reference, reference_available

    cfg = dict(LAYERS[args.config])
    E, k, d, ffn, t = cfg["E"], cfg["k"], cfg["d"], cfg["ffn"], cfg["t"]
    T = args.tokens if args.tokens_set else cfg["T"]
    gb = ffn * row_bytes(t, d)
    slots = None
    try:
        import torch

        if torch.cuda.is_available():
            from freemoe_b200 import hotpath

            hotpath.init(0)
            slots = [torch.cat([hotpath.synth_weights(t, rows, cols, 1000 + 3 * e + j)
                                for j, (rows, cols) in enumerate(((ffn, d), (ffn, d), (d, ffn)))]).cpu().numpy()
                     for e in range(E)]
    except Exception:  # noqa: BLE001 - no usable GPU: encode on the host
        slots = None
    if slots is None:
        orc = Oracle()
        rng = np.random.default_rng(1)
        slots = [np.concatenate([orc.quantize(t, rng.normal(0, 0.02, n).astype(np.float32))
                                 for n in (ffn * d, ffn * d, d * ffn)]) for _ in range(E)]
    x, lg = layer_inputs(cfg, T, seed=1)
    threads = os.cpu_count() or 1
    kind = "reference" if reference_available() else "port"
    ref = Reference() if kind == "reference" else None
    orc = Oracle()
    n_s = min(T, max(1, int(args.sample)))

    def step():
        if ref is not None:
            rc, ids, w, _ = ref.route(lg[:n_s], k)
            return ref.moe_block(t, slots, gb, 2 * gb, x[:n_s], ids, w, d, ffn, threads=threads)
        rc, ids, w, _ = orc.route(lg[:n_s], k)
        return orc.moe_block(x[:n_s], ids, w, slots, d, ffn, t)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = n_s / dt
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": {8: "q8_0", 12: "q4_k"}[t], "data": "synthetic",
            "config": {"workload": f"{args.config}: {E} experts d {d} ffn {ffn} top-{k} (routed experts), "
                                   f"{n_s} of T={T} tokens per step", "tokens": n_s},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                             "sample": f"{n_s} tokens of the {T}-token batch per step", **host_cpu()},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_layer_ep(args):
    """The Qwen3-shaped layer expert-parallel over the torchrun ranks (NCCL):
    experts 128/G per rank, tokens 8192/G per rank (strong scaling), token rows
    dispatched to the experts' owners and the outputs combined back with
    all-to-all (freemoe_b200/ep.py)."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200.ep import DeviceOps, EPLayer

    cfg = dict(LAYERS[args.config])
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    hotpath.init(local)
    E, k, d, ffn, t = cfg["E"], cfg["k"], cfg["d"], cfg["ffn"], cfg["t"]
    T = args.tokens if args.tokens_set else cfg["T"]
    if E % world or T % world:
        raise SystemExit(f"{E} experts / {T} tokens do not shard over {world} ranks")
    per, tp = E // world, T // world
    gb = ffn * row_bytes(t, d)
    slots = []
    for e in range(rank * per, (rank + 1) * per):  # the same seeds as the one-GPU layer
        slots.append(torch.cat([hotpath.synth_weights(t, rows, cols, 1000 + 3 * e + j)
                                for j, (rows, cols) in enumerate(((ffn, d), (ffn, d), (d, ffn)))]))
    x_np, lg_np = layer_inputs(cfg, T, seed=1)
    sl = slice(rank * tp, (rank + 1) * tp)
    x = torch.from_numpy(x_np[sl]).cuda().to(torch.bfloat16)
    logits = torch.from_numpy(lg_np[sl]).cuda()
    ops = DeviceOps(experts_total=E, top_k=k, d_model=d, ffn=ffn, gate_type=t, up_type=t, down_type=t,
                    local_slots=slots, up_offset=gb, down_offset=2 * gb)
    layer = EPLayer(ops, record_timing=True, mode=args.ep_mode)
    for _ in range(args.warmup):
        y = layer.forward(x, logits)
    torch.cuda.synchronize()
    assert hotpath.device_status() == 0
    layer.phase_ms()  # drop the warm-up marks
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            y = layer.forward(x, logits)
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    phases = layer.phase_ms()
    ph_t = torch.tensor([phases[k] for k in EPLayer.PHASES], dtype=torch.float64, device="cuda")
    dist.all_reduce(ph_t, op=dist.ReduceOp.MAX)
    phases = dict(zip(EPLayer.PHASES, ph_t.tolist()))
    layer.record_timing = False
    # e2e: host token rows and logits in, y out, every step; the copies run on
    # two copy streams beside the layer, as in the one-GPU configurations
    hx = torch.from_numpy(x_np[sl]).to(torch.bfloat16).pin_memory()
    hl = torch.from_numpy(lg_np[sl]).pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    ms_loc, hy = pipelined_e2e(lambda dx, dl, dy: dy.copy_(layer.forward(dx, dl)), hx, hl, x, logits,
                               torch.empty(tp, d, dtype=torch.float32, device="cuda"), args.steps, stream)
    ms_e = torch.tensor([ms_loc], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms_e, op=dist.ReduceOp.MAX)
    assert np.isfinite(hy.numpy()).all()
    pairs = T * k
    routed, _ = layer_flops(cfg, pairs, T)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    if rank == 0:
        line = {"metric": METRIC, "value": T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": {8: "q8_0", 12: "q4_k"}[t] + " -> fp16 tensor cores", "data": "synthetic",
                "config": {"workload": f"{args.config} expert-parallel: {E} experts ({per}/rank) d {d} ffn {ffn} "
                                       f"top-{k}, T={T} bf16 tokens ({tp}/rank), {cfg['logits']} router logits",
                           "tokens": T, "parallelism": f"ep{world}",
                           "exchange": {"p2p": "peer-memory stores fused into the dispatch and partial-sum kernels "
                                                "(CUDA IPC mailboxes, no collective in the data path)",
                                        "rows": "NCCL all-to-all (torch.distributed), one row per token and rank",
                                        "pairs": "NCCL all-to-all (torch.distributed), one row per pair"}[args.ep_mode]},
                "phase_ms_max_over_ranks": phases,
                "e2e": {"value": T / (float(ms_e.item()) / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": hx.numel() * 2 + hl.numel() * 4, "d2h_bytes_per_step": hy.numel() * 4,
                        "ms_per_step": float(ms_e.item())},
                "roofline": {"bound": "tensor", "kernel": "whole expert-parallel layer", "unit": "TFLOP/s",
                             "achieved": routed / (ms / 1e3) / 1e12, "peak": peak * world,
                             "peak_kind": "measured x ranks" if peaks else "fallback x ranks",
                             "frac": routed / (ms / 1e3) / 1e12 / (peak * world), "traffic": None},
                "gpu_launches": None, "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def run_stack_ep(args):
    """--gpus N > 1 on the headline stack: expert parallelism over the torchrun
    ranks.  Experts e live on rank e / (8 / N) with the N = 1 line's weights; the
    step's T tokens are split over the ranks (T / N each, strong scaling: the
    same stack and tokens as N = 1); each rank routes its tokens (top-8 of 8),
    sends every token once to each rank over peer memory (mode p2p; NCCL
    all-to-all with --ep-mode rows), runs the received rows through its experts
    (tcgen05 decode stage) and combines the returned partial sums.  value = the
    N = 1 line's bytes (every expert's weights once, x and y) / the step time,
    max over ranks."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from freemoe_b200 import hotpath
    from freemoe_b200.ep import DeviceOps, EPLayer

    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    hotpath.init(local)
    type_id = TYPES[args.type]
    T = args.tokens
    if EXPERTS % world or T % world:
        raise SystemExit(f"{EXPERTS} experts / {T} tokens do not shard over {world} ranks")
    per, tp = EXPERTS // world, T // world
    gb = FFN * row_bytes(type_id, D_MODEL)
    slots = []
    for e in range(rank * per, (rank + 1) * per):  # the N = 1 line's weights (its rank-0 seeds)
        slots.append(torch.cat([hotpath.synth_weights(type_id, rows, cols, 1000 + 3 * e + j)
                                for j, (rows, cols) in enumerate(((FFN, D_MODEL), (FFN, D_MODEL), (D_MODEL, FFN)))]))
    x_np, lg_np = host_inputs(T, seed=0)  # the N = 1 line's tokens
    sl = slice(rank * tp, (rank + 1) * tp)
    x = torch.from_numpy(x_np[sl]).cuda().to(torch.bfloat16)
    logits = torch.from_numpy(lg_np[sl]).cuda()
    ops = DeviceOps(experts_total=EXPERTS, top_k=EXPERTS, d_model=D_MODEL, ffn=FFN, gate_type=type_id,
                    up_type=type_id, down_type=type_id, local_slots=slots, up_offset=gb, down_offset=2 * gb)
    p2p = args.ep_mode == "p2p"
    layer = EPLayer(ops, record_timing=True, mode=args.ep_mode, device_epoch=p2p)
    for _ in range(args.warmup):
        layer.forward(x, logits)
    torch.cuda.synchronize()
    assert hotpath.device_status() == 0
    layer.phase_ms()  # drop the warm-up marks
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # value: timed without the phase events; the phases come from a second pass
    layer.record_timing = False
    graph, xs, ls, y_static = None, x, logits, None
    if p2p:
        # the peer-memory layer numbers its calls on the device, so one captured
        # forward replays as a whole step: every step's 15 launches from one
        # graph launch (the Python layer's host work no longer paces the GPUs)
        xs, ls = x.clone(), logits.clone()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            layer.forward(xs, ls)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_static = layer.forward(xs, ls)
        graph.replay()
        torch.cuda.synchronize()
        assert hotpath.device_status() == 0

    def step():
        if graph is not None:
            graph.replay()
        else:
            layer.forward(x, logits)

    with ClockSampler(local) as clocks:
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
    ms_t = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    layer.record_timing = True
    for _ in range(min(args.steps, 200)):
        layer.forward(x, logits)
    torch.cuda.synchronize()
    phases = layer.phase_ms()
    ph_t = torch.tensor([phases[k] for k in EPLayer.PHASES], dtype=torch.float64, device="cuda")
    dist.all_reduce(ph_t, op=dist.ReduceOp.MAX)
    phases = dict(zip(EPLayer.PHASES, ph_t.tolist()))
    layer.record_timing = False
    # e2e: this rank's tokens and logits from pinned host memory, y back, every step
    hx = torch.from_numpy(x_np[sl]).to(torch.bfloat16).pin_memory()
    hl = torch.from_numpy(lg_np[sl]).pin_memory()
    dist.barrier()
    torch.cuda.synchronize()
    def e2e_call(dx, dl, dy):
        if graph is None:
            dy.copy_(layer.forward(dx, dl))
            return
        xs.copy_(dx)
        ls.copy_(dl)
        graph.replay()
        dy.copy_(y_static)

    ms_loc, hy = pipelined_e2e(e2e_call, hx, hl, x, logits,
                               torch.empty(tp, D_MODEL, dtype=torch.float32, device="cuda"), args.steps, stream)
    ms_e = torch.tensor([ms_loc], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms_e, op=dist.ReduceOp.MAX)
    assert np.isfinite(hy.numpy()).all()
    assert hotpath.device_status() == 0
    del graph
    nbytes = step_bytes(type_id, T)
    peak, peak_kind = load_peaks()
    # the rank's expert phase streams its experts' bytes once
    local_bytes = per * expert_bytes(type_id)
    exp_ms = phases.get("experts", 0.0)
    if rank == 0:
        line = {
            "metric": METRIC, "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": args.type, "data": "synthetic",
            "config": stack_config(args.type, T, world),
            "entry_point": "freemoe_b200.ep.EPLayer.forward (route, dispatch, experts, combine per step)",
            "exchange": {"p2p": "peer-memory stores fused into the dispatch and partial-sum kernels (CUDA IPC "
                                "mailboxes, no collective in the data path); each step one CUDA graph replay",
                         "rows": "NCCL all-to-all (torch.distributed), one row per token and rank",
                         "pairs": "NCCL all-to-all (torch.distributed), one row per pair"}[args.ep_mode],
            "sharding": f"experts {per}/rank, tokens {tp}/rank",
            "tokens_per_s": T / (ms / 1e3),
            "phase_ms_max_over_ranks": phases,
            "roofline": {"bound": "hbm", "kernel": "one rank's expert phase (tcgen05 decode stage, its "
                                                   f"{per} experts' weights once)",
                         "achieved": local_bytes / (exp_ms / 1e3) / 1e9 if exp_ms else None, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": local_bytes / (exp_ms / 1e3) / 1e9 / peak if exp_ms else None, "traffic": None,
                         "algorithmic_bytes": local_bytes},
            "e2e": {"value": nbytes / (float(ms_e.item()) / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": world * (hx.numel() * 2 + hl.numel() * 4),
                    "d2h_bytes_per_step": world * hy.numel() * 4, "ms_per_step": float(ms_e.item())},
            # per rank and step in mode p2p: route; dispatch keys, grouping, counts, plan,
            # pack + send; wait, expert keys, grouping, B images, gate/up, down, partial
            # return; wait, combine
            "gpu_launches": 7 * args.steps if args.ep_mode == "p2p" else None,
            "clocks": clocks.summary()}
        print(json.dumps(line), flush=True)
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--ep-mode", default="p2p", choices=["p2p", "rows", "pairs"],
                    help="expert-parallel exchange of the layer configurations under torchrun")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--type", default="q4_k", choices=sorted(TYPES))
    ap.add_argument("--tokens", type=int, default=8)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="time budget of the headline's CPU baseline sample")
    ap.add_argument("--no-extras", action="store_true",
                    help="measure the headline only (not the further configurations under 'configs')")
    ap.add_argument("--extra-steps", type=int, default=200, help="timed steps of each further configuration")
    ap.add_argument("--sample", type=int, default=32,
                    help="tokens per step of the reference arm on a layer configuration")
    ap.add_argument("--config", default="stack", choices=["stack", *LAYERS, "gemv", "coldload"],
                    help="stack (default, the headline), a layer configuration, the GEMV shapes, "
                         "or cold expert-record loads")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)  # at least 3 untimed warm-up steps
    args.tokens_set = any(a.startswith("--tokens") for a in sys.argv[1:])
    if args.config == "coldload":
        (run_reference_coldload if args.impl == "reference" else run_coldload)(args)
        return
    if args.config in LAYERS and args.impl == "reference":
        run_reference_layer(args)
        return
    if args.config == "gemv" and args.impl == "ours":
        run_gemv_shapes(args)
        return
    if args.config != "stack" and args.impl == "ours":
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            run_layer_ep(args)
        else:
            run_layer(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif int(os.environ.get("WORLD_SIZE", "1")) > 1:
        run_stack_ep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
