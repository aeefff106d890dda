"""numpy restatement of the reference's generated ``fp_chain_<N>`` kernels.

TEST INFRASTRUCTURE ONLY (the oracle).  Nothing in ``fusionpass_b200`` imports it.

Reference semantics followed here:

* every input is loaded and upcast to float32
  (``lib/Plan/TritonEmitter.cpp:39-40``; twin ``python/fusionpass/kernels.py:167-173``);
* the body ops are evaluated in program order in float32
  (``TritonEmitter.cpp:228-244``; twin ``kernels.py:176-202``):
  ``add`` -> ``a + b``, ``mul`` -> ``a * b``, ``scale`` -> ``a * factor`` (an f32
  attribute, ``FPOps.td:36-40``), ``relu`` -> ``tl.maximum(a, 0.0)``,
  ``exp`` -> ``tl.exp(a)``;
* ``softmax`` (rows launch only, last axis) is the numerically stable form
  ``e = exp(x - max(x)); y = e / sum(e)`` (``TritonEmitter.cpp:237-242``);
* the yielded value is rounded ONCE to the output dtype at the store
  (``TritonEmitter.cpp:245-246``), round-to-nearest-even.

Extension beyond the reference op set (no reference kernel exists, parity is
pinned against eager PyTorch only): ``gelu`` = ``0.5*x*(1+erf(x/sqrt(2)))`` and
broadcast operands (a per-last-dim vector, a per-row column, a scalar), which
the reference frontend rejects (``python/fusionpass/frontend.py:153-154``); for
those the reference arithmetic is the same kernel fed with the operand
expanded to full shape, which is what numpy broadcasting computes here.
"""

from __future__ import annotations

from typing import Any, Mapping, Sequence

import numpy as np

F32 = np.float32
_BINARY = ("add", "mul")
_UNARY = ("scale", "relu", "exp", "softmax", "gelu")

try:  # scipy's float32 erf, used only by the gelu extension op
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover - scipy is present in this image
    _erf = None


def body_to_program(n_args: int, body: Sequence[Mapping[str, Any]], yield_value: str | None = None):
    """Translate a reference chain body into a slot program.

    ``body`` is the format accepted by the reference's Python twin
    ``emit_chain_kernel`` (``python/fusionpass/kernels.py:129-146``): dicts with
    ``op``, ``operands`` (names ``a<i>`` for block args, ``t<k>`` or a custom
    ``out``/``result`` name for earlier results) and ``factor`` for scale.

    Returns ``(ops, result_slot)`` where ``ops`` is a list of
    ``(op, src_a, src_b, imm)`` with slots ``0..n_args-1`` = inputs and
    ``n_args + k`` = result of op ``k``.
    """
    names: dict[str, int] = {f"a{i}": i for i in range(int(n_args))}
    ops = []
    last = n_args - 1 if n_args else None
    for k, op in enumerate(body):
        kind = op["op"]
        if kind not in _BINARY + _UNARY:
            raise ValueError(f"unsupported op in chain: {kind}")
        srcs = [names[x] for x in op.get("operands", ())]
        a = srcs[0]
        b = srcs[1] if kind in _BINARY else -1
        imm = float(np.float32(op.get("factor", 0.0))) if kind == "scale" else 0.0
        ops.append((kind, a, b, imm))
        slot = n_args + k
        names[op.get("out") or op.get("result") or f"t{k}"] = slot
        last = slot
    y = names[yield_value] if yield_value is not None else last
    if y is None:
        raise ValueError("chain has no value to store")
    return ops, y


def _apply(kind: str, a: np.ndarray, b: np.ndarray | None, imm: float) -> np.ndarray:
    if kind == "add":
        return (a + b).astype(F32, copy=False)
    if kind == "mul":
        return (a * b).astype(F32, copy=False)
    if kind == "scale":
        return (a * F32(imm)).astype(F32, copy=False)
    if kind == "relu":
        return np.maximum(a, F32(0.0))
    if kind == "exp":
        return np.exp(a).astype(F32, copy=False)
    if kind == "gelu":
        if _erf is None:
            raise RuntimeError("gelu oracle needs scipy")
        t = (a * F32(0.7071067811865476)).astype(F32)
        e = _erf(t).astype(F32)
        return ((a * F32(0.5)) * (F32(1.0) + e)).astype(F32, copy=False)
    raise ValueError(kind)


def _softmax_last(x: np.ndarray) -> np.ndarray:
    # TritonEmitter.cpp:239-241: where(mask, x, -inf); exp(x - max); / sum
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp((x - m).astype(F32)).astype(F32)
    s = np.sum(e, axis=-1, keepdims=True, dtype=F32)
    return (e / s).astype(F32)


def chain_eval(inputs: Sequence[np.ndarray], ops, result: int, out_shape, out_dtype) -> np.ndarray:
    """Evaluate a slot program over broadcast-compatible inputs; f32 math, one rounding."""
    out_shape = tuple(int(d) for d in out_shape)
    slots: list[np.ndarray] = [np.broadcast_to(np.asarray(x).astype(F32), out_shape) for x in inputs]
    for kind, a, b, imm in ops:
        va = slots[a]
        if kind == "softmax":
            slots.append(_softmax_last(np.asarray(va)))
            continue
        vb = slots[b] if kind in _BINARY else None
        slots.append(np.asarray(_apply(kind, va, vb, imm), dtype=F32))
    y = np.asarray(slots[result], dtype=F32)
    if y.shape != out_shape:
        y = np.broadcast_to(y, out_shape)
    return np.ascontiguousarray(y.astype(out_dtype))


def chain_flat(inputs, ops, result, out_shape, out_dtype):
    """``launch: "flat"`` kernel (no softmax in the body)."""
    if any(op[0] == "softmax" for op in ops):
        raise ValueError("flat chain must not contain softmax")
    return chain_eval(inputs, ops, result, out_shape, out_dtype)


def chain_rows(inputs, ops, result, out_shape, out_dtype):
    """``launch: "rows"`` kernel: exactly one last-axis softmax in the body."""
    if sum(op[0] == "softmax" for op in ops) != 1:
        raise ValueError("rows chain needs exactly one softmax")
    return chain_eval(inputs, ops, result, out_shape, out_dtype)
