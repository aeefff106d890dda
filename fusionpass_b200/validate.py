"""Structural plan checks: a corrupt or stale plan fails before any kernel runs.

Same contract as the reference ``python/fusionpass/validate.py:10-44`` (plan
version 1; list fields; f16/f32 dtypes; known torch ops; fused steps keep
``kind: "triton"`` with ``launch`` in {flat, rows, attention}; attention has 3
operands; no use before definition; no duplicate results; defined outputs),
plus a check of the launch descriptor a fused step may carry in
``attrs["desc"]``.
"""

from __future__ import annotations

DTYPES = {"f16", "f32"}
TORCH_OPS = {"add", "mul", "scale", "relu", "exp", "softmax", "matmul", "transpose"}
# unfused steps the planner emits only with extensions=True (BERT-style blocks)
EXTENSION_TORCH_OPS = {"gelu", "linear", "layer_norm", "add_layer_norm", "reshape", "permute", "cat", "narrow"}
LAUNCHES = {"flat", "rows", "attention"}
_CHAIN_OPS = {"add", "mul", "scale", "relu", "exp", "softmax", "gelu"}


def _check_desc(i: int, st: dict) -> None:
    desc = st.get("attrs", {}).get("desc")
    if desc is None:
        return
    if not isinstance(desc, dict) or desc.get("op") not in ("chain", "attention"):
        raise ValueError(f"step {i}: bad launch descriptor")
    if st["launch"] == "attention":
        if desc["op"] != "attention":
            raise ValueError(f"step {i}: attention step with a {desc['op']} descriptor")
        return
    if desc["op"] != "chain":
        raise ValueError(f"step {i}: chain step with an attention descriptor")
    ops, ins = desc.get("ops"), desc.get("inputs")
    if not isinstance(ops, list) or not ops or not isinstance(ins, list):
        raise ValueError(f"step {i}: chain descriptor needs 'inputs' and 'ops' lists")
    if len(ins) != len(st.get("operands", [])):
        raise ValueError(f"step {i}: descriptor has {len(ins)} inputs, step has {len(st['operands'])} operands")
    n = len(ins)
    softmax = 0
    for k, op in enumerate(ops):
        if op.get("op") not in _CHAIN_OPS:
            raise ValueError(f"step {i}: unsupported chain op {op.get('op')!r}")
        srcs = [op.get("a")] + ([op.get("b")] if op["op"] in ("add", "mul") else [])
        if any(not isinstance(s, int) or not 0 <= s < n + k for s in srcs):
            raise ValueError(f"step {i}: chain op {k} reads an undefined slot")
        softmax += op["op"] == "softmax"
    if not isinstance(desc.get("result"), int) or not 0 <= desc["result"] < n + len(ops):
        raise ValueError(f"step {i}: chain result slot out of range")
    if (st["launch"] == "rows") != (softmax == 1) or softmax > 1:
        raise ValueError(f"step {i}: {st['launch']} launch with {softmax} softmax op(s)")


def validate_plan(plan: dict) -> None:
    """Raise ValueError if ``plan`` is not a well-formed version-1 plan."""
    if plan.get("version") != 1:
        raise ValueError(f"unsupported plan version {plan.get('version')!r}")
    for key in ("inputs", "steps", "outputs"):
        if not isinstance(plan.get(key), list):
            raise ValueError(f"plan['{key}'] must be a list")
    defined = set()
    for spec in plan["inputs"]:
        if spec.get("dtype") not in DTYPES or not isinstance(spec.get("shape"), list):
            raise ValueError(f"bad input spec: {spec}")
        defined.add(spec["name"])
    for i, st in enumerate(plan["steps"]):
        for o in st.get("operands", []):
            if o not in defined:
                raise ValueError(f"step {i}: operand '{o}' used before definition")
        res = st.get("result")
        if not res or res in defined:
            raise ValueError(f"step {i}: missing or duplicate result name '{res}'")
        if st.get("dtype") not in DTYPES:
            raise ValueError(f"step {i}: bad dtype")
        kind = st.get("kind")
        if kind == "torch":
            if st.get("op") not in TORCH_OPS | EXTENSION_TORCH_OPS:
                raise ValueError(f"step {i}: unknown torch op '{st.get('op')}'")
        elif kind == "triton":
            if st.get("launch") not in LAUNCHES or not st.get("kernel"):
                raise ValueError(f"step {i}: bad triton step")
            if st["launch"] == "attention" and len(st["operands"]) != 3:
                raise ValueError(f"step {i}: attention needs exactly 3 operands")
            _check_desc(i, st)
        else:
            raise ValueError(f"step {i}: unknown kind '{kind}'")
        defined.add(res)
    for o in plan["outputs"]:
        if o not in defined:
            raise ValueError(f"output '{o}' is never defined")
