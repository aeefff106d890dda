"""``compile_model``: trace -> plan (+ descriptors) -> ``CompiledModel`` -> verify gate.

Same signature and behaviour as the reference ``python/fusionpass/api.py:49-83``,
with the compiler subprocess replaced by the in-process planner twin
(``planner.py``) so no MLIR toolchain is needed.  The workdir receives
``model.mlir`` (the traced fp text), ``plan.json`` and ``kernels.json`` (the
descriptor table that replaces the generated ``kernels.py``).
"""

from __future__ import annotations

import json
import tempfile
from pathlib import Path

import torch

from . import planner
from .runtime import execute_plan, validate_plan
from .verify import EquivalenceError, verify_equivalence


class CompiledModel:
    def __init__(self, plan: dict, captured: list, workdir: Path, mlir_text: str, kernels=None):
        validate_plan(plan)  # fail early on a corrupt plan
        self.plan, self._captured, self.workdir, self.mlir_text, self.kernels = plan, captured, workdir, mlir_text, kernels
        self.report = None      # VerifyReport once verification has run
        self.verified = False   # True only if verification ran and passed

    def __call__(self, *inputs):
        return execute_plan(self.plan, list(inputs) + self._captured, self.kernels, validate=False)


def compile_model(model, example_inputs, *, fuse: bool = False, workdir=None, verify: bool = True,
                  strict: bool = True, atol=None, rtol=None, extensions: bool = False) -> CompiledModel:
    """Compile ``model`` for ``example_inputs``; ``extensions=True`` enables the ops
    beyond the reference subset (broadcast operands, gelu, Linear/LayerNorm/reshape)."""
    example_inputs = tuple(example_inputs)
    g = planner.trace(model, example_inputs, extensions=extensions)
    mlir_text = planner.to_mlir(g)
    workdir = Path(workdir or tempfile.mkdtemp(prefix="fusionpass_"))
    workdir.mkdir(parents=True, exist_ok=True)
    (workdir / "model.mlir").write_text(mlir_text)
    plan, table = planner.compile_graph(g, fuse=fuse, extensions=extensions)
    (workdir / "plan.json").write_text(json.dumps(plan, indent=2))
    (workdir / "kernels.json").write_text(table.to_json())
    has_fused = any(s["kind"] == "triton" for s in plan["steps"])
    captured = g.arg_tensors[g.n_inputs:]
    compiled = CompiledModel(plan, captured, workdir, mlir_text, table if has_fused else None)
    if verify:
        compiled.report = verify_equivalence(model, compiled, example_inputs, atol=atol, rtol=rtol)
        compiled.verified = compiled.report.ok
        if strict and not compiled.report.ok:
            raise EquivalenceError(f"fusion changed results: {compiled.report.reason}")
    return compiled
