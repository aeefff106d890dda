"""Times the reference's own CPU path for the fused steps: its Triton kernels under
the Triton interpreter (TRITON_INTERPRET=1), driven through its own
``execute_plan -> kernels.launch_step``.  A measurement recipe, not part of the
product and not run by the tests or the bench (it needs the reference checkout).

    python oracle/time_reference_interpreter.py /path/to/reference [--rows 512]

Workloads (the benchmark's configurations, inputs seeded as there):
* the f32 attention demo, B1 H4 S128 D64, scale 1/8 (the reference's
  ``fp_attention`` source, ``python/fusionpass/kernels.py:58-89``);
* the chain y = relu((x + b) * s) * 0.5 + x in f16 at ``--rows`` x 4096 (the
  reference's generated ``fp_chain`` kernel, ``kernels.py:129-211``), b and s
  expanded to full shape because the reference cannot trace broadcast operands.
Prints one JSON object: seconds, the metric's units per second, and the host
threads used (the interpreter runs numpy on one Python thread).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import torch  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("reference", type=Path)
    ap.add_argument("--rows", type=int, default=512)
    a = ap.parse_args(argv)
    sys.path.insert(0, str(a.reference / "python"))
    from fusionpass import kernels as rk  # the reference package
    from fusionpass.runtime import execute_plan

    def plan(inputs, step):
        return {"version": 1, "inputs": inputs, "steps": [step], "outputs": [step["result"]]}

    res = {"threads": 1, "torch_threads": torch.get_num_threads(), "interpreter": "TRITON_INTERPRET=1"}
    with tempfile.TemporaryDirectory() as d:
        # attention demo
        w = rk.KernelModuleWriter()
        w.add_attention_kernel()
        (Path(d) / "attn.py").write_text(w.write())
        mod = rk.load_kernels(Path(d) / "attn.py")
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(1, 4, 128, 64, generator=g) for _ in range(3))
        ins = [{"name": f"arg{i}", "shape": [1, 4, 128, 64], "dtype": "f32"} for i in range(3)]
        step = {"kind": "triton", "kernel": "fp_attention", "launch": "attention",
                "operands": ["arg0", "arg1", "arg2"], "result": "v0", "shape": [1, 4, 128, 64], "dtype": "f32",
                "attrs": rk.attention_launch_attrs(0.125)}
        t0 = time.perf_counter()
        execute_plan(plan(ins, step), [q, k, v], mod)
        dt = time.perf_counter() - t0
        flop = 4 * 1 * 4 * 128 * 128 * 64
        res["attention_f32_B1H4S128D64"] = {"seconds": round(dt, 3), "GFLOP/s": round(flop / dt / 1e9, 4)}

        # the chain workload at a bounded number of rows
        R, C = a.rows, 4096
        g = torch.Generator().manual_seed(0)
        x = torch.randn(R, C, generator=g).half()
        b = (torch.randn(C, generator=g) * 0.1).half().expand(R, C).contiguous()
        s = (torch.rand(C, generator=g) + 0.5).half().expand(R, C).contiguous()
        body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "mul", "operands": ["t0", "a2"]},
                {"op": "relu", "operands": ["t1"]}, {"op": "scale", "operands": ["t2"], "factor": 0.5},
                {"op": "add", "operands": ["t3", "a0"]}]
        w = rk.KernelModuleWriter()
        kname = w.add_chain_kernel(3, body, rows=False)
        (Path(d) / "chain.py").write_text(w.write())
        mod = rk.load_kernels(Path(d) / "chain.py")
        ins = [{"name": f"arg{i}", "shape": [R, C], "dtype": "f16"} for i in range(3)]
        step = {"kind": "triton", "kernel": kname, "launch": "flat", "operands": ["arg0", "arg1", "arg2"],
                "result": "v0", "shape": [R, C], "dtype": "f16", "attrs": rk.chain_launch_attrs([R, C], rows=False)}
        t0 = time.perf_counter()
        execute_plan(plan(ins, step), [x, b, s], mod)
        dt = time.perf_counter() - t0
        nbytes = R * C * 2 * 2 + 2 * C * 2  # the workload's bytes: read x, write y, b and s once
        res[f"chain_f16_{R}x{C}"] = {"seconds": round(dt, 3), "GB/s": round(nbytes / dt / 1e9, 5),
                                     "rows": R, "note": "b, s fed expanded to full shape"}
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
