#!/usr/bin/env python
"""Benchmark of the fused-step hot path on B200 (one JSON line on rank 0).

Headline workload (one "step" = one fused chain launch):
    y = relu((x + b) * s) * 0.5 + x,  x f16 [4096, 4096] ~ N(0,1),
    b f16 [4096] ~ N(0, 0.1) per column, s f16 [4096] ~ U[0.5, 1.5]
Secondary (same line, key "attention"): fp_attention prefill
    B=8 H=16 S=2048 D=64 f16, Q/K/V ~ N(0,1) * D^-1/4, scale 1/8.

Multi-GPU (torchrun, one process per GPU): every rank owns its own rows /
batch*heads of a global problem N times the single-GPU one (weak scaling, no
collective on the data path); the time is the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "fp_attention TFLOP/s & chain HBM GB/s per B200, % roofline, 1/2/4/8 GPU"
R, C = 4096, 4096
CHAIN_BYTES = R * C * 2 * 2 + 2 * C * 2  # read x + write y (f16) + b, s
ATT = dict(B=8, H=16, S=2048, D=64)
ATT_FLOP = 4 * ATT["B"] * ATT["H"] * ATT["S"] ** 2 * ATT["D"]
CFG2_BODY = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "mul", "operands": ["t0", "a2"]},
             {"op": "relu", "operands": ["t1"]}, {"op": "scale", "operands": ["t2"], "factor": 0.5},
             {"op": "add", "operands": ["t3", "a0"]}]
NBUF = 4  # rotating input/output sets: 4 x 67 MB > 126 MB L2


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tc": float(d["bf16_tflops"]),
                "tc_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "src": "measured"}
    return {"hbm": 6650.0, "tc": 1590.0, "tc_sustained": 1400.0, "src": "fallback"}


def ncu_traffic():
    p = ROOT / "profiles" / "ncu_traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock, max clock and clock-event reasons through NVML."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period: float = 0.005):
        self.samples = []
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self.t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        while not self._stop.is_set():
            try:
                sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), sm, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self, t0: float, t1: float):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        win = [s for s in self.samples if t0 <= s[0] <= t1] or self.samples[-5:]
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [n for b, n in self.REASONS.items() if bits & b]
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(win)}


# --------------------------------------------------------------- workloads
def chain_inputs(rank: int):
    g = torch.Generator().manual_seed(1000 + rank)
    x = torch.randn(R, C, generator=g).half()
    b = (torch.randn(C, generator=g) * 0.1).half()
    s = (torch.rand(C, generator=g) + 0.5).half()
    return x, b, s


def attention_inputs(rank: int):
    g = torch.Generator().manual_seed(2000 + rank)
    shp = (ATT["B"], ATT["H"], ATT["S"], ATT["D"])
    return tuple((torch.randn(shp, generator=g) * ATT["D"] ** -0.25).half() for _ in range(3))


# -------------------------------------------------------------- CPU legs
def cpu_chain_rate(seconds: float, threads: int):
    """The oracle (numpy f32 restatement of the reference chain kernel) on the host
    cores: bytes of the chain workload processed per second."""
    from oracle import chain as oc

    x, b, s = (t.numpy() for t in chain_inputs(0))
    ops, res = oc.body_to_program(3, CFG2_BODY)
    rows = 256

    def task(r0):
        oc.chain_flat([x[r0:r0 + rows], b, s], ops, res, (rows, C), np.float16)

    passes = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(task, range(0, R, rows)))
            passes += 1
            if time.perf_counter() - t0 >= seconds:
                break
    dt = time.perf_counter() - t0
    return passes * CHAIN_BYTES / dt / 1e9, passes


def cpu_eager_torch_rate(seconds: float, threads: int):
    """Eager PyTorch on the host cores, the same module as the chain workload
    (y = relu((x + b) * s) * 0.5 + x in f16): bytes of the workload per second."""
    torch.set_num_threads(threads)
    x, b, s = chain_inputs(0)
    passes = 0
    t0 = time.perf_counter()
    while True:
        torch.relu((x + b) * s) * 0.5 + x
        passes += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return passes * CHAIN_BYTES / dt / 1e9, passes


def cpu_attention_rate(seconds: float, threads: int):
    """The oracle restatement of fp_attention on B*H slices of the prefill workload."""
    from oracle import attention as oa

    q, k, v = (t.numpy().reshape(-1, ATT["S"], ATT["D"]) for t in attention_inputs(0))
    done = 0
    t0 = time.perf_counter()
    with ThreadPoolExecutor(threads) as ex:
        while True:
            list(ex.map(lambda i: oa.attention_fwd(q[i:i + 1], k[i:i + 1], v[i:i + 1], 0.125),
                        range(done % q.shape[0], done % q.shape[0] + threads)))
            done += threads
            if time.perf_counter() - t0 >= seconds:
                break
    dt = time.perf_counter() - t0
    per_slice = 4 * ATT["S"] ** 2 * ATT["D"]
    return done * per_slice / dt / 1e12, done


# -------------------------------------------------------------- our arm
# ------------------------------------------------------------ rank group
class RankGroup:
    """One process per GPU.  Barrier, max over ranks and a joint pass/fail vote for
    the timed regions (NCCL between GPUs; the same code runs on gloo in CPU tests).
    Every rank calls the same methods in the same order."""

    def __init__(self, rank: int, world: int, device: torch.device):
        self.rank, self.world, self.device = rank, world, device
        self.dist = world > 1

    def barrier(self) -> None:
        if self.dist:
            import torch.distributed as tdist
            tdist.barrier()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)

    def max(self, x: float) -> float:
        if not self.dist:
            return float(x)
        import torch.distributed as tdist
        t = torch.tensor([float(x)], device=self.device, dtype=torch.float64)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        return float(t.item())

    def all_ok(self, ok: bool) -> bool:
        """True only if every rank passed (so all ranks stop together on a failure)."""
        if not self.dist:
            return bool(ok)
        import torch.distributed as tdist
        t = torch.tensor([1 if ok else 0], device=self.device, dtype=torch.int32)
        tdist.all_reduce(t, op=tdist.ReduceOp.MIN)
        return bool(t.item())


def weak_rate(world: int, steps: int, units_per_step: float, ms_max: float) -> float:
    """Whole-job rate (units per second) when each of `world` ranks ran `steps`
    steps of `units_per_step` on its own data and the slowest rank took `ms_max`."""
    return world * steps * units_per_step / (ms_max * 1e-3)


# ----------------------------------------------------- the other configs
def _graph_time_ms(fn, reps: int, group: "RankGroup", stream) -> float:
    """Max over ranks of the device time of `reps` calls of fn replayed from one CUDA graph."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=torch.cuda.Stream(group.device)):
        for _ in range(reps):
            fn()
    g.replay()
    group.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    g.replay()
    e1.record(stream)
    group.barrier()
    ms = group.max(e0.elapsed_time(e1))
    del g
    return ms


def run_configs(args, group: "RankGroup", rank: int, world: int, dev) -> dict:
    """cfg1 (f32 attention demo), cfg4 (long-sequence D=128 attention) and cfg5
    (BERT-base encoder block through the plan executor), each checked before it is
    timed; weak scaling over ranks like the headline."""
    from fusionpass_b200 import fpkern
    from fusionpass_b200.api import compile_model

    from oracle import attention as oa

    stream = torch.cuda.current_stream(dev)
    out = {}

    # cfg1: B1 H4 S128 D64 f32, Q/K/V ~ N(0,1) from seed 0, scale 1/8
    g = torch.Generator().manual_seed(0)
    q1, k1, v1 = (torch.randn(1, 4, 128, 64, generator=g) for _ in range(3))
    qd, kd, vd = (t.to(dev) for t in (q1, k1, v1))
    od = fpkern.attention(qd, kd, vd, 0.125)
    ref = oa.attention_fwd(q1.numpy(), k1.numpy(), v1.numpy(), 0.125)
    err = float(np.abs(od.cpu().numpy() - ref).max())
    if not group.all_ok(err <= 1e-5):
        raise RuntimeError(f"cfg1 attention differs from the oracle (max err {err:.2e})")
    reps = 200
    ms = _graph_time_ms(lambda: fpkern.attention(qd, kd, vd, 0.125, out=od), reps, group, stream)
    flop = 4 * 1 * 4 * 128 * 128 * 64
    out["cfg1_attention_f32"] = {"workload": "fp_attention B1 H4 S128 D64 f32, scale 1/8", "check": f"max err {err:.1e} vs oracle",
                                 "us_per_launch": round(ms / reps * 1e3, 2),
                                 "value": round(weak_rate(world, reps, flop, ms) / 1e12, 3), "unit": "TFLOP/s"}

    # cfg4: B4 H32 S8192 D128 f16, Q/K/V ~ N(0,1), scale 1/sqrt(128)
    if not args.no_long:
        g = torch.Generator(device=dev).manual_seed(4000 + rank)
        shp = (4, 32, 8192, 128)
        q4, k4, v4 = (torch.randn(shp, generator=g, device=dev).half() for _ in range(3))
        sc = 128 ** -0.5
        o4 = fpkern.attention(q4, k4, v4, sc)
        worst = 0.0
        for b, h in ((0, 0), (3, 31)):
            r = torch.softmax((q4[b, h].float() @ k4[b, h].float().T) * sc, -1) @ v4[b, h].float()
            worst = max(worst, float(((o4[b, h].float() - r).abs() / (2e-3 + 1e-2 * r.abs())).max()))
        if not group.all_ok(worst <= 1.0):
            raise RuntimeError(f"cfg4 attention outside the f16 tolerance ({worst:.2f} of it)")
        # 40 launches (~0.15 s of dense tensor work): long enough for the power cap to
        # settle the clocks, so the fraction is against the sustained GEMM peak too
        reps = 40
        pk4 = peaks()
        ms = _graph_time_ms(lambda: fpkern.attention(q4, k4, v4, sc, out=o4), reps, group, stream)
        flop = 4 * 4 * 32 * 8192 ** 2 * 128
        tf = flop / (ms / reps * 1e-3) / 1e12
        out["cfg4_attention_long"] = {
            "workload": "fp_attention B4 H32 S8192 D128 f16, scale 1/sqrt(128)",
            "check": f"2 (b,h) slices vs torch f32: {worst:.2f} of the atol 2e-3 / rtol 1e-2 budget",
            "launches": reps, "ms_per_launch": round(ms / reps, 3),
            "value": round(weak_rate(world, reps, flop, ms) / 1e12, 2), "unit": "TFLOP/s",
            "roofline_frac": round(tf / pk4["tc"], 4),
            "roofline_frac_of_sustained": round(tf / pk4["tc_sustained"], 4),
            # Q, K, V read once and O written once: 4 * 268 MB per launch
            "algorithmic_bytes_per_launch": 4 * 4 * 32 * 8192 * 128 * 2,
            "traffic": ncu_traffic().get("attention_long", {}).get("dram_bytes_per_launch")}
        del q4, k4, v4, o4

    # cfg5: BERT-base block, batch 32 seq 512 hidden 768 heads 12 FFN 3072, f16
    if not args.no_bert:
        sys.path.insert(0, str(ROOT))
        from tests.models import BertBlock, init_bert

        torch.manual_seed(0)
        m = init_bert(BertBlock(32, 512)).half().to(dev).eval()
        g = torch.Generator(device=dev).manual_seed(5000 + rank)
        x = torch.randn(32, 512, 768, generator=g, device=dev).half()
        c = compile_model(m, (x,), fuse=True, extensions=True, strict=False)
        kinds = [st.get("launch", st["kind"]) for st in c.plan["steps"]]
        if not group.all_ok(bool(c.verified)):
            raise RuntimeError(f"cfg5 BERT block failed the equivalence gate: {c.report}")
        reps = 20
        with torch.no_grad():
            ms = _graph_time_ms(lambda: c(x), reps, group, stream)
        tokens = 32 * 512
        out["cfg5_bert_block"] = {
            "workload": "BERT-base encoder block f16, batch 32 seq 512 hidden 768 heads 12 FFN 3072 (random init)",
            "check": "verify_equivalence gate passed (f16 1e-2 / 1e-2, 3 trials)",
            "fused_steps": {"attention": kinds.count("attention"), "flat_chains": kinds.count("flat")},
            "ms_per_block": round(ms / reps, 4), "value": round(weak_rate(world, reps, tokens, ms), 1),
            "unit": "tokens/s",
            "note": "whole block through execute_plan; Linear/LayerNorm run as unfused torch steps"}
    return out


def run_ours(args, rank, world, dev):
    from fusionpass_b200 import fpkern, kernels
    from fusionpass_b200.runtime import execute_plan

    pk = peaks()
    traffic = ncu_traffic()
    group = RankGroup(rank, world, dev)
    barrier, max_over_ranks = group.barrier, group.max

    desc = kernels.chain_descriptor(3, CFG2_BODY, input_bcast=["full", "col", "col"])
    x, b, s = chain_inputs(rank)
    xs = [x.to(dev) for _ in range(NBUF)]
    bd, sd = b.to(dev), s.to(dev)
    ys = [torch.empty(R, C, dtype=torch.float16, device=dev) for _ in range(NBUF)]
    stream = torch.cuda.current_stream(dev)

    def step(i):
        fpkern.chain([xs[i % NBUF], bd, sd], desc, [R, C], torch.float16, out=ys[i % NBUF])

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if not group.all_ok(fpkern.poll_status(dev) == 0):
        raise RuntimeError("chain kernel reported a device-side error during warm-up (on some rank)")
    # parity gate before timing: bit-exact against the oracle on this rank's data
    same = True
    if not args.skip_check:
        from oracle import chain as oc
        ops, res = oc.body_to_program(3, CFG2_BODY)
        ref = oc.chain_flat([x.numpy(), b.numpy(), s.numpy()], ops, res, (R, C), np.float16)
        same = bool(np.array_equal(ys[0].cpu().numpy(), ref))
    if not group.all_ok(same):
        raise RuntimeError("chain output differs from the oracle (on some rank): refusing to time it")

    K = args.steps
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=torch.cuda.Stream(dev)):
        for i in range(K):
            step(i)
    graph.replay()
    torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clk:
        # keep the GPU busy a moment before the timed region so clocks settle
        graph.replay()
        barrier()
        w0 = time.perf_counter()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        barrier()
        w1 = time.perf_counter()
        graph.replay()  # trailing samples under the same load
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms)
    clocks = clk.summary(w0 - 0.05, w1 + 0.05)
    per_launch_ms = ms / K
    chain_gbs = CHAIN_BYTES / (per_launch_ms * 1e-3) / 1e9
    value = weak_rate(world, K, CHAIN_BYTES, ms_max) / 1e9

    # ---- e2e through the public API: pinned host -> device -> execute_plan -> host
    e2e = None
    if not args.no_e2e:
        plan = {"version": 1,
                "inputs": [{"name": "arg0", "shape": [R, C], "dtype": "f16"},
                           {"name": "arg1", "shape": [C], "dtype": "f16"},
                           {"name": "arg2", "shape": [C], "dtype": "f16"}],
                "steps": [{"kind": "triton", "kernel": "fp_chain_0", "launch": "flat",
                           "operands": ["arg0", "arg1", "arg2"], "result": "v0", "shape": [R, C], "dtype": "f16",
                           "attrs": {**kernels.chain_launch_attrs([R, C], rows=False), "desc": desc}}],
                "outputs": ["v0"]}
        hx, hb, hs = (t.pin_memory() for t in (x, b, s))
        ke = max(2, min(K, args.e2e_steps))
        # two streams: step i+1's host -> device copies run while step i computes and
        # copies its result back (the copy engines of the two directions overlap)
        streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
        hys = [torch.empty(R, C, dtype=torch.float16).pin_memory() for _ in streams]

        def e2e_step(i):
            st = streams[i % 2]
            with torch.cuda.stream(st):
                dx = hx.to(dev, non_blocking=True)
                db = hb.to(dev, non_blocking=True)
                ds = hs.to(dev, non_blocking=True)
                y = execute_plan(plan, [dx, db, ds], validate=False)
                hys[i % 2].copy_(y, non_blocking=True)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        same = bool(torch.equal(hys[0], ys[0].cpu()))  # the host result equals the device-resident run's
        if not group.all_ok(same):
            raise RuntimeError("e2e result differs from the device-resident run (on some rank)")
        barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for st in streams:
            st.wait_event(a0)
        for i in range(ke):
            e2e_step(i)
        for st in streams:
            done = torch.cuda.Event()
            done.record(st)
            stream.wait_event(done)
        a1.record(stream)
        barrier()
        ems = max_over_ranks(a0.elapsed_time(a1))
        e2e = {"value": round(weak_rate(world, ke, CHAIN_BYTES, ems) / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": int(hx.numel() * 2 + hb.numel() * 2 + hs.numel() * 2),
               "d2h_bytes_per_step": int(hys[0].numel() * 2), "steps": ke,
               "path": "per step: pinned host -> device copies of x, b, s, execute_plan (libfpkern chain), "
                       "device -> pinned host copy of y; steps alternate over two streams so one step's "
                       "upload overlaps the previous step's download"}

    # ---- secondary: attention prefill
    attention = None
    if not args.no_attention:
        q, k, v = (t.to(dev) for t in attention_inputs(rank))
        o = torch.empty_like(q)
        for _ in range(3):
            fpkern.attention(q, k, v, 0.125, out=o)
        torch.cuda.synchronize()
        if not group.all_ok(fpkern.poll_status(dev) == 0):
            raise RuntimeError("attention kernel reported a device-side error during warm-up (on some rank)")
        ka = args.attn_steps
        ag = torch.cuda.CUDAGraph()
        with torch.cuda.graph(ag, stream=torch.cuda.Stream(dev)):
            for _ in range(ka):
                fpkern.attention(q, k, v, 0.125, out=o)
        ag.replay()
        barrier()
        b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        b0.record(stream)
        ag.replay()
        b1.record(stream)
        barrier()
        ams = b0.elapsed_time(b1)
        ams_max = max_over_ranks(ams)
        tflops = ATT_FLOP / (ams / ka * 1e-3) / 1e12
        attention = {
            "workload": "fp_attention B8 H16 S2048 D64 f16, scale 1/8, non-causal",
            "value": round(weak_rate(world, ka, ATT_FLOP, ams_max) / 1e12, 2), "unit": "TFLOP/s",
            "ms_per_step": round(ams_max / ka, 4), "steps": ka, "gpu_launches": ka,
            "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": pk["tc"], "unit": "TFLOP/s",
                         "frac": round(tflops / pk["tc"], 4),
                         "peak_source": f"{pk['src']} bf16 dense GEMM burst",
                         "frac_of_spec_2250": round(tflops / 2250.0, 4),
                         "traffic": traffic.get("attention_prefill", {}).get("dram_bytes_per_launch")},
        }
        del ag

    del graph
    configs = None if args.no_configs else run_configs(args, group, rank, world, dev)
    cpu = None
    cpu_eager = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        gbs, passes = cpu_chain_rate(args.cpu_seconds, threads)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{passes} full passes of the [4096,4096] chain in 256-row blocks, numpy oracle"}
        eg, ep = cpu_eager_torch_rate(min(args.cpu_seconds, 2.0), threads)
        cpu_eager = {"value": round(eg, 3), "unit": "GB/s", "threads": threads,
                     "sample": f"{ep} passes of the [4096,4096] f16 module in eager PyTorch on the CPU"}
        if attention is not None:
            tf, slices = cpu_attention_rate(args.cpu_seconds, threads)
            attention["cpu_baseline"] = {"value": round(tf, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                         "sample": f"{slices} (b,h) slices of S=2048 D=64, numpy oracle"}

    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(ms_max / K, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "fused chain y = relu((x + b) * s) * 0.5 + x, x f16 [4096,4096], b/s f16 [4096] "
                               "per column (one chain kernel per step)",
                   "per_rank_rows": R, "cols": C, "storage": "f16", "parallelism": f"rows x{world} (weak)",
                   "l2": f"{NBUF} rotating input/output sets ({NBUF * CHAIN_BYTES / 1e6:.0f} MB > 126 MB L2)",
                   "timing": "K launches replayed from one CUDA graph, CUDA events on the launch stream"},
        "roofline": {"bound": "hbm", "achieved": round(chain_gbs, 2), "peak": pk["hbm"], "unit": "GB/s",
                     "frac": round(chain_gbs / pk["hbm"], 4), "peak_source": f"{pk['src']} HBM copy",
                     "frac_of_spec_8000": round(chain_gbs / 8000.0, 4),
                     "traffic": traffic.get("chain_cfg2", {}).get("dram_bytes_per_launch"),
                     "algorithmic_bytes_per_launch": CHAIN_BYTES},
        "clocks": clocks, "gpu_launches": K, "e2e": e2e, "cpu_baseline": cpu, "cpu_eager_torch": cpu_eager, "attention": attention,
        "configs": configs,
        "impl": "ours",
    }
    return line


# -------------------------------------------------------- reference arm
def run_reference(args):
    """The reference path's CPU implementation (its kernels restated in numpy: the
    oracle port) on all host cores, on the same workload, metric and unit."""
    threads = os.cpu_count() or 1
    from oracle import chain as oc

    x, b, s = (t.numpy() for t in chain_inputs(0))
    ops, res = oc.body_to_program(3, CFG2_BODY)
    rows = 256
    sample_rows = 1024  # each step: a bounded 1024-row sample of the [4096,4096] workload

    def task(r0):
        oc.chain_flat([x[r0:r0 + rows], b, s], ops, res, (rows, C), np.float16)

    def one_step(i):
        base = (i * sample_rows) % R
        with ThreadPoolExecutor(threads) as ex:
            list(ex.map(task, range(base, base + sample_rows, rows)))

    for i in range(args.warmup):
        one_step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one_step(i)
    dt = time.perf_counter() - t0
    step_bytes = sample_rows * C * 4 + 2 * C * 2
    gbs = args.steps * step_bytes / dt / 1e9
    sample = f"{sample_rows} of {R} rows per step in {rows}-row blocks on {threads} threads, numpy oracle port"
    return {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "fused chain y = relu((x + b) * s) * 0.5 + x, x f16 [4096,4096], b/s f16 [4096] "
                               "per column", "per_rank_rows": R, "cols": C, "storage": "f16"},
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--attn-steps", type=int, default=50)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-seconds", type=float, default=4.0)
    ap.add_argument("--no-attention", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--skip-check", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the cfg1/cfg4/cfg5 entries")
    ap.add_argument("--no-long", action="store_true", help="skip the cfg4 entry")
    ap.add_argument("--no-bert", action="store_true", help="skip the cfg5 entry")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        print(json.dumps(run_reference(args)), flush=True)
        return 0

    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "impl": "ours", "error": "no CUDA device"}), flush=True)
        return 1
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # stdout carries exactly one JSON line: library output from process-group setup to
    # teardown (the NCCL version banner, for one) goes to stderr
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        if world > 1:
            import datetime

            import torch.distributed as tdist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        try:
            line = run_ours(args, rank, world, dev)
        finally:
            if world > 1:
                import torch.distributed as tdist
                tdist.destroy_process_group()
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
