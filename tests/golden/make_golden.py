"""Generate golden vectors by running the REFERENCE's own kernels on the CPU.

Run once where the reference checkout is available (the tests only read the fixtures):

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

It imports the reference package ``fusionpass`` from ``<reference>/python``, builds
chain kernels with its ``KernelModuleWriter`` (the Python twin of
``lib/Plan/TritonEmitter.cpp``) and the shared ``fp_attention`` source, and runs
them through the reference's own ``runtime.execute_plan`` -> ``kernels.launch_step``
boundary under ``TRITON_INTERPRET=1``.  Inputs are seeded; inputs and outputs
are written as ``.npz`` fixtures next to this script.  The committed fixtures
are what the tests read; the reference is never needed at test time.
"""

from __future__ import annotations

import json
import os
import sys
import tempfile
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
if len(sys.argv) < 2:
    sys.exit("usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF / "python"))

from fusionpass import kernels as rk  # noqa: E402  (reference package)
from fusionpass.runtime import execute_plan  # noqa: E402  (reference package)

_DT = {"f32": torch.float32, "f16": torch.float16}


def _plan(inputs, step):
    return {"version": 1, "inputs": inputs, "steps": [step], "outputs": [step["result"]]}


def run_attention(name, shape, dtype, scale, seed, mult=1.0):
    g = torch.Generator().manual_seed(seed)
    q, k, v = ((torch.randn(shape, generator=g) * mult).to(_DT[dtype]) for _ in range(3))
    w = rk.KernelModuleWriter()
    w.add_attention_kernel()
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "kernels.py"
        p.write_text(w.write())
        mod = rk.load_kernels(p)
        ins = [{"name": f"arg{i}", "shape": list(shape), "dtype": dtype} for i in range(3)]
        step = {"kind": "triton", "kernel": "fp_attention", "launch": "attention",
                "operands": ["arg0", "arg1", "arg2"], "result": "v0", "shape": list(shape),
                "dtype": dtype, "attrs": rk.attention_launch_attrs(scale)}
        out = execute_plan(_plan(ins, step), [q, k, v], mod)
    meta = {"kind": "attention", "dtype": dtype, "scale": float(scale), "shape": list(shape)}
    np.savez_compressed(HERE / f"{name}.npz", q=q.numpy(), k=k.numpy(), v=v.numpy(),
                        out=out.numpy(), meta=json.dumps(meta))
    print(name, tuple(out.shape), dtype)


def run_chain(name, n_args, body, shape, dtype, inputs, launch, small_inputs=None):
    """``inputs`` are full-shape tensors fed to the reference; ``small_inputs`` (optional)
    are the un-expanded broadcast operands stored for the product's broadcast path."""
    w = rk.KernelModuleWriter()
    kname = w.add_chain_kernel(n_args, body, rows=(launch == "rows"))
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "kernels.py"
        p.write_text(w.write())
        mod = rk.load_kernels(p)
        ins = [{"name": f"arg{i}", "shape": list(shape), "dtype": dtype} for i in range(n_args)]
        step = {"kind": "triton", "kernel": kname, "launch": launch,
                "operands": [f"arg{i}" for i in range(n_args)], "result": "v0",
                "shape": list(shape), "dtype": dtype,
                "attrs": rk.chain_launch_attrs(shape, rows=(launch == "rows"))}
        out = execute_plan(_plan(ins, step), list(inputs), mod)
    meta = {"kind": "chain", "launch": launch, "dtype": dtype, "shape": list(shape),
            "n_args": n_args, "body": list(body)}
    arrs = {f"x{i}": t.numpy() for i, t in enumerate(inputs)}
    if small_inputs is not None:
        for i, t in small_inputs.items():
            arrs[f"x{i}_small"] = t.numpy()
    np.savez_compressed(HERE / f"{name}.npz", out=out.numpy(), meta=json.dumps(meta), **arrs)
    print(name, tuple(out.shape), dtype, launch)


def main():
    # ---- attention (reference tests/test_triton.py:401-437, test_edge_cases.py:53-57,149-158)
    run_attention("attn_f32_1x2x20x16", (1, 2, 20, 16), "f32", 0.25, seed=1)
    run_attention("attn_cfg1_f32_1x4x128x64", (1, 4, 128, 64), "f32", 0.125, seed=0)
    for S in (1, 7, 64, 65, 130):
        run_attention(f"attn_f32_S{S}_d16", (1, 2, S, 16), "f32", 0.25, seed=100 + S)
    run_attention("attn_f32_1x1x70x32_x4", (1, 1, 70, 32), "f32", 32 ** -0.5, seed=7, mult=4.0)
    run_attention("attn_f16_1x2x100x64", (1, 2, 100, 64), "f16", 0.125, seed=11)
    run_attention("attn_f16_1x2x130x128", (1, 2, 130, 128), "f16", 128 ** -0.5, seed=12)
    run_attention("attn_f16_1x2x65x16", (1, 2, 65, 16), "f16", 0.25, seed=13)
    run_attention("attn_f16_1x1x7x32", (1, 1, 7, 32), "f16", 32 ** -0.5, seed=14)
    run_attention("attn_f16_2x1x256x64_x2", (2, 1, 256, 64), "f16", 0.125, seed=15, mult=2.0)

    g = torch.Generator().manual_seed(0)
    # ---- flat chains
    body = [{"op": "add", "operands": ["a0", "a1"]},
            {"op": "scale", "operands": ["t0"], "factor": 2.0},
            {"op": "relu", "operands": ["t1"]},
            {"op": "exp", "operands": ["t2"]}]
    a, b = torch.randn(8, 16, generator=g), torch.randn(8, 16, generator=g)
    run_chain("chain_flat_f32_add_scale_relu_exp", 2, body, (8, 16), "f32", [a, b], "flat")

    # cfg2 arithmetic at a small size: y = relu((x + b) * s) * 0.5 + x, b/s per column
    R, C = 64, 256
    x = torch.randn(R, C, generator=g).half()
    bb = (torch.randn(C, generator=g) * 0.1).half()
    ss = (torch.rand(C, generator=g) + 0.5).half()
    body = [{"op": "add", "operands": ["a0", "a1"]},
            {"op": "mul", "operands": ["t0", "a2"]},
            {"op": "relu", "operands": ["t1"]},
            {"op": "scale", "operands": ["t2"], "factor": 0.5},
            {"op": "add", "operands": ["t3", "a0"]}]
    run_chain("chain_flat_f16_cfg2_64x256", 3, body, (R, C), "f16",
              [x, bb.expand(R, C).contiguous(), ss.expand(R, C).contiguous()], "flat",
              small_inputs={1: bb, 2: ss})

    x = torch.randn(5, 7, generator=g)
    run_chain("chain_flat_f32_dedupe_relu_xx", 1,
              [{"op": "mul", "operands": ["a0", "a0"]}, {"op": "relu", "operands": ["t0"]}],
              (5, 7), "f32", [x], "flat")

    ins = [torch.randn(33, 65, generator=g) for _ in range(4)]
    body = [{"op": "add", "operands": ["a2", "a3"]},
            {"op": "add", "operands": ["a0", "a1"]},
            {"op": "mul", "operands": ["t1", "t0"]},
            {"op": "scale", "operands": ["t2"], "factor": 0.25}]
    run_chain("chain_flat_f32_tree_33x65", 4, body, (33, 65), "f32", ins, "flat")

    x = torch.randn(16, 8, generator=g).t().contiguous()
    run_chain("chain_flat_f32_exp_relu_16x8t", 1,
              [{"op": "scale", "operands": ["a0"], "factor": 2.0},
               {"op": "relu", "operands": ["t0"]},
               {"op": "scale", "operands": ["t1"], "factor": 0.1},
               {"op": "exp", "operands": ["t2"]}], (8, 16), "f32", [x], "flat")

    x, y = torch.randn(3, 1001, generator=g).half(), torch.randn(3, 1001, generator=g).half()
    run_chain("chain_flat_f16_ragged_3x1001", 2,
              [{"op": "mul", "operands": ["a0", "a1"]},
               {"op": "scale", "operands": ["t0"], "factor": 1.5},
               {"op": "add", "operands": ["t1", "a1"]}], (3, 1001), "f16", [x, y], "flat")

    # ---- rows chains
    x = torch.randn(6, 100, generator=g)
    run_chain("chain_rows_f32_scale_softmax_relu_6x100", 1,
              [{"op": "scale", "operands": ["a0"], "factor": 0.5},
               {"op": "softmax", "operands": ["t0"]},
               {"op": "relu", "operands": ["t1"]}], (6, 100), "f32", [x], "rows")

    x, bias = torch.randn(16, 128, generator=g), torch.randn(16, 128, generator=g)
    rowchain = [{"op": "scale", "operands": ["a0"], "factor": 0.5},
                {"op": "add", "operands": ["t0", "a1"]},
                {"op": "relu", "operands": ["t1"]},
                {"op": "softmax", "operands": ["t2"]},
                {"op": "scale", "operands": ["t3"], "factor": 2.0}]
    run_chain("chain_rows_f32_rowchain_16x128", 2, rowchain, (16, 128), "f32", [x, bias], "rows")
    x, bias = torch.randn(8, 1000, generator=g).half(), torch.randn(8, 1000, generator=g).half()
    run_chain("chain_rows_f16_rowchain_8x1000", 2, rowchain, (8, 1000), "f16", [x, bias], "rows")

    x = torch.randn(4, 50, generator=g) * 50
    run_chain("chain_rows_f32_large_magnitude_4x50", 1,
              [{"op": "scale", "operands": ["a0"], "factor": 1.0},
               {"op": "softmax", "operands": ["t0"]},
               {"op": "scale", "operands": ["t1"], "factor": 2.0}], (4, 50), "f32", [x], "rows")

    x = torch.randn(4, 8192, generator=g).half()
    run_chain("chain_rows_f16_long_4x8192", 1,
              [{"op": "scale", "operands": ["a0"], "factor": 0.125},
               {"op": "softmax", "operands": ["t0"]}], (4, 8192), "f16", [x], "rows")

    x, y = torch.randn(8, 300, generator=g), torch.randn(8, 300, generator=g)
    run_chain("chain_rows_f32_post_uses_input_8x300", 2,
              [{"op": "softmax", "operands": ["a0"]},
               {"op": "mul", "operands": ["t0", "a1"]},
               {"op": "add", "operands": ["t1", "a0"]}], (8, 300), "f32", [x, y], "rows")


if __name__ == "__main__":
    main()
