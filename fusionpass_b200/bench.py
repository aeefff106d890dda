"""``benchmark``: eager vs fused device time, refused for models that failed the gate.

Keeps the interface of the reference ``python/fusionpass/bench.py:43-61``: the
same ``BenchResult`` fields and the same gate order (a speedup is never
reported for a model that has not passed ``verify_equivalence``; CPU inputs are
refused).  Timing is this package's own: each callable runs ``iters`` times
back to back in a few rounds bracketed by CUDA events on the current stream,
and the per-call time is the median over rounds of the round's mean.
``est_bytes_*`` are algorithmic bytes: every step reads each operand once and
writes its result once (the minimum HBM traffic of the plan).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import prod

import torch

from .verify import VerifyReport

_ESZ = {"f16": 2, "f32": 4}


class UnverifiedSpeedupError(RuntimeError):
    """Raised when a speedup is requested for a model that has not passed verification."""


@dataclass(frozen=True)
class BenchResult:
    eager_ms: float
    fused_ms: float
    speedup: float
    iters: int
    eager_launches: int
    fused_launches: int
    est_bytes_unfused: int | None
    est_bytes_fused: int | None
    report: VerifyReport


def plan_bytes(plan: dict) -> int:
    """Algorithmic bytes of a plan: the sum over steps of its operands' and its
    result's sizes (each tensor moved once per step)."""
    size = {t["name"]: prod(t["shape"]) * _ESZ[t["dtype"]] for t in plan["inputs"]}
    total = 0
    for st in plan["steps"]:
        size[st["result"]] = prod(st["shape"]) * _ESZ[st["dtype"]]
        total += sum(size.get(o, 0) for o in st["operands"]) + size[st["result"]]
    return total


def device_ms_per_call(fn, warmup: int, iters: int, rounds: int = 5) -> float:
    """Per-call device time of ``fn`` on the current CUDA stream (median of the
    per-round means of back-to-back calls)."""
    for _ in range(warmup):
        fn()
    stream = torch.cuda.current_stream()
    per_round = max(1, iters // rounds)
    means = []
    for _ in range(rounds):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(per_round):
            fn()
        e1.record(stream)
        e1.synchronize()
        means.append(e0.elapsed_time(e1) / per_round)
    means.sort()
    return means[len(means) // 2]


def benchmark(model, compiled, inputs, *, unfused=None, warmup: int = 25, iters: int = 100) -> BenchResult:
    if not getattr(compiled, "verified", False) or compiled.report is None or not compiled.report.ok:
        raise UnverifiedSpeedupError("refusing to report a speedup: the compiled model has not passed "
                                     "equivalence verification (compile with verify=True)")
    inputs = tuple(inputs)
    if not inputs[0].is_cuda:
        raise RuntimeError("benchmarking requires CUDA tensors")
    with torch.no_grad():
        eager = device_ms_per_call(lambda: model(*inputs), warmup, iters)
        fused = device_ms_per_call(lambda: compiled(*inputs), warmup, iters)
    base = unfused.plan if unfused is not None else None
    return BenchResult(eager_ms=eager, fused_ms=fused, speedup=eager / fused, iters=iters,
                       eager_launches=len(base["steps"]) if base else -1,
                       fused_launches=len(compiled.plan["steps"]),
                       est_bytes_unfused=plan_bytes(base) if base else None,
                       est_bytes_fused=plan_bytes(compiled.plan), report=compiled.report)
