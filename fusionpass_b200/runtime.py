"""Plan executor: ``execute_plan`` with the reference signature and semantics.

Reference: ``python/fusionpass/runtime.py:21-60``.  Unfused ``torch`` steps run
as eager PyTorch ops; fused steps (``kind: "triton"``, kept for plan
compatibility) go to ``kernels.launch_step``, i.e. to libfpkern.so on the
current CUDA stream.
"""

from __future__ import annotations

import torch

from .kernels import check_device as _check_device
from .kernels import launch_step, load_kernels
from .validate import validate_plan

_DTYPES = {"f32": torch.float32, "f16": torch.float16}

__all__ = ["execute_plan", "load_kernels", "validate_plan", "_run_torch", "_run_fused", "_check_device",
           "_DTYPES"]


def _run_torch(step: dict, ops: list) -> torch.Tensor:
    op, attrs = step["op"], step["attrs"]
    if op == "add":
        return torch.add(ops[0], ops[1])
    if op == "mul":
        return torch.mul(ops[0], ops[1])
    if op == "scale":
        return ops[0] * attrs["factor"]
    if op == "relu":
        return torch.relu(ops[0])
    if op == "exp":
        return torch.exp(ops[0])
    if op == "softmax":
        return torch.softmax(ops[0], dim=attrs["axis"])
    if op == "matmul":
        return torch.matmul(ops[0], ops[1])
    if op == "transpose":
        return ops[0].transpose(-1, -2)
    # extension steps (planner extensions=True)
    if op == "gelu":
        return torch.nn.functional.gelu(ops[0])
    if op == "linear":
        return torch.nn.functional.linear(ops[0], ops[1], ops[2] if len(ops) == 3 else None)
    if op == "layer_norm":
        w, b = (ops[1], ops[2]) if len(ops) == 3 else (None, None)
        if ops[0].is_cuda and len(attrs["normalized_shape"]) == 1:
            # over the last axis: the libfpkern kernel (None if it does not take the shape)
            from . import fpkern
            y = fpkern.layer_norm(ops[0], w, b, attrs["eps"])
            if y is not None:
                return y
        return torch.nn.functional.layer_norm(ops[0], attrs["normalized_shape"], w, b, attrs["eps"])
    if op == "add_layer_norm":
        # layer_norm of the sum of the first n_addends operands (the add chain that fed it)
        k = attrs["n_addends"]
        w, b = (ops[k], ops[k + 1]) if len(ops) == k + 2 else (None, None)
        if ops[0].is_cuda:
            from . import fpkern
            y = fpkern.add_layer_norm(ops[:k], w, b, attrs["eps"], shape=step.get("shape"))
            if y is not None:
                return y
        x = ops[0]
        for t in ops[1:k]:
            x = x + t
        return torch.nn.functional.layer_norm(x, attrs["normalized_shape"], w, b, attrs["eps"])
    if op == "reshape":
        return ops[0].reshape(attrs["shape"])
    if op == "cat":
        return torch.cat(ops, dim=attrs["dim"])
    if op == "narrow":
        return ops[0].narrow(attrs["dim"], attrs["start"], attrs["length"])
    if op == "permute":
        return ops[0].permute(*attrs["dims"])
    raise ValueError(f"unknown torch op in plan: {op}")


def _run_fused(step: dict, ops: list, kernels) -> torch.Tensor:
    return launch_step(step, ops, kernels)


_run_triton = _run_fused  # the reference's name for the same hook


def execute_plan(plan: dict, args: list, kernels=None, *, validate: bool = True):
    """Run ``plan`` on ``args``; returns the single output (or a tuple)."""
    if validate:
        validate_plan(plan)
    if plan.get("version") != 1:
        raise ValueError(f"unsupported plan version {plan.get('version')}")
    if len(args) != len(plan["inputs"]):
        raise ValueError(f"expected {len(plan['inputs'])} inputs, got {len(args)}")
    env = {}
    for spec, t in zip(plan["inputs"], args):
        # static shapes: the plan and its descriptors are specialised to them
        if list(t.shape) != spec["shape"] or t.dtype != _DTYPES[spec["dtype"]]:
            raise ValueError(f"{spec['name']}: expected {spec['dtype']}{spec['shape']}, "
                             f"got {t.dtype}{list(t.shape)}")
        env[spec["name"]] = t
    for step in plan["steps"]:
        ops = [env[o] for o in step["operands"]]
        kind = step["kind"]
        if kind == "torch":
            env[step["result"]] = _run_torch(step, ops)
        elif kind == "triton":
            env[step["result"]] = _run_fused(step, ops, kernels)
        else:
            raise ValueError(f"unknown step kind {kind}")
    outs = [env[o] for o in plan["outputs"]]
    return outs[0] if len(outs) == 1 else tuple(outs)
