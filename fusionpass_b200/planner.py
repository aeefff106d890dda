"""Python twin of ``fusionpass-compile``: trace -> fp ops -> fusion passes -> plan.

The reference compiler is C++/MLIR 18 (``tools/fusionpass-compile``); this
module reproduces its contract so that plans with launch descriptors can be
produced without MLIR:

* ``trace``: ``torch.fx`` + ``ShapeProp`` over the reference frontend's op
  subset (``python/fusionpass/frontend.py:43-166``): matmul, softmax(dim), relu,
  exp, transpose of the last two dims, tensor add/mul, mul/div by a Python
  number.  ``to_mlir`` prints the same ``fp`` dialect text as the reference.
  With ``extensions=True`` it also accepts what the BERT-style and broadcast
  chain workloads need: operands broadcast along the last dim / per row /
  scalar, ``gelu`` (erf form), ``nn.Linear`` (a ``linear`` torch step + a bias
  ``add``), ``nn.LayerNorm``, ``view``/``reshape``/``permute``/``contiguous``.
* ``fuse_attention``: ``FuseAttentionPattern`` (``lib/Transforms/FuseAttention.cpp:15-49``).
* ``fuse_chains``: ``FuseChainPattern`` (``lib/Transforms/FuseChains.cpp:12-90``).
* ``emit_plan``: ``emitPlan`` (``lib/Plan/PlanEmitter.cpp:59-185``), with each
  fused step carrying its launch descriptor in ``attrs["desc"]``.

Graphs traced with ``extensions=True`` (which the reference cannot trace) get three
more rewrites after chain fusion, none of which touches the reference's rules:
``fold_linear_bias`` (a bias add no chain took goes back into its linear step),
``merge_sibling_linears`` (projections of one input as one GEMM + views) and
``fuse_add_layer_norm`` (an add chain feeding a LayerNorm, as one step); an
attention result that only feeds a heads merge is stored in the merged order.
"""

from __future__ import annotations

import operator
import re
from dataclasses import dataclass, field
from typing import Any

import numpy as np
import torch
import torch.fx as fx
import torch.nn.functional as F
from torch.fx.passes.shape_prop import ShapeProp

from . import kernels as K


class UnsupportedOp(Exception):
    """The traced graph uses something outside the supported subset (never a silent fallback)."""


_DT = {torch.float32: "f32", torch.float16: "f16"}
_MATMUL = {torch.matmul, operator.matmul}
_SOFTMAX = {torch.softmax, F.softmax}
_RELU = {torch.relu, F.relu}
_ADD = {operator.add, torch.add}
_MUL = {operator.mul, torch.mul}
_DIV = {operator.truediv, torch.div}
CHAINABLE = {"add", "mul", "scale", "relu", "exp", "softmax"}
CHAINABLE_EXT = CHAINABLE | {"gelu"}


# ------------------------------------------------------------------- IR ---
@dataclass(eq=False)
class Val:
    shape: tuple
    dtype: str
    producer: "Op | None" = None
    uses: list = field(default_factory=list)  # one entry per operand slot that reads this value
    arg_index: int | None = None


@dataclass(eq=False)
class Op:
    kind: str
    operands: list
    result: Val
    attrs: dict = field(default_factory=dict)
    # fused_chain only: body ops as (kind, refs, attrs); ref = ("a", i) | ("t", j)
    body: list | None = None
    alive: bool = True


@dataclass
class Graph:
    args: list
    ops: list
    output: Val
    arg_tensors: list
    n_inputs: int
    # the function's return (a pseudo-op whose operands are the returned values, so a
    # returned value counts as used), when it returns more than one value
    ret: "Op | None" = None

    def live_ops(self):
        return [o for o in self.ops if o.alive]


def _new_op(kind, operands, shape, dtype, attrs=None, body=None) -> Op:
    op = Op(kind, list(operands), Val(tuple(shape), dtype), dict(attrs or {}), body)
    op.result.producer = op
    for v in op.operands:
        v.uses.append(op)
    return op


# ---------------------------------------------------------------- trace ---
def _fetch_attr(root, target: str):
    obj = root
    for part in target.split("."):
        obj = getattr(obj, part)
    return obj


def _dtype(t) -> str:
    if t not in _DT:
        raise UnsupportedOp(f"unsupported dtype {t}")
    return _DT[t]


def _bcast_ok(small: tuple, big: tuple) -> bool:
    """Broadcasts the chain kernels support: full, per-last-dim vector, per-row column, scalar."""
    n = int(np.prod(small)) if small else 1
    if tuple(small) == tuple(big) or n == 1:
        return True
    if len(small) >= 1 and small[-1] == big[-1] and n == big[-1]:
        return True  # [..., 1, C] / [C]
    if len(small) == len(big) and small[-1] == 1 and tuple(small[:-1]) == tuple(big[:-1]):
        return True  # [..., R, 1]
    return False


def trace(model: torch.nn.Module, example_inputs, *, extensions: bool = False) -> Graph:
    """Trace ``model`` into fp ops (reference ``frontend.trace_to_mlir`` semantics)."""
    gm = fx.symbolic_trace(model)
    ShapeProp(gm).propagate(*example_inputs)
    env: dict[fx.Node, Any] = {}
    args: list[Val] = []
    tensors: list[torch.Tensor] = []
    ph = iter(example_inputs)

    def add_arg(t: torch.Tensor) -> Val:
        v = Val(tuple(t.shape), _dtype(t.dtype), arg_index=len(args))
        if len(t.shape) == 0:
            raise UnsupportedOp("rank-0 tensors are unsupported")
        args.append(v)
        tensors.append(t.detach())
        return v

    for n in gm.graph.nodes:
        if n.op == "placeholder":
            env[n] = add_arg(next(ph))
    n_inputs = len(args)
    for n in gm.graph.nodes:
        if n.op == "get_attr":
            t = _fetch_attr(gm, n.target)
            if not isinstance(t, torch.Tensor):
                raise UnsupportedOp(f"get_attr {n.target} is not a tensor")
            env[n] = add_arg(t)
    module_params: dict[int, Val] = {}

    def param(t: torch.Tensor) -> Val:
        key = id(t)
        if key not in module_params:
            module_params[key] = add_arg(t)
        return module_params[key]

    ops: list[Op] = []
    out_val = None

    def meta(n):
        m = n.meta.get("tensor_meta")
        if m is None or not hasattr(m, "shape"):
            raise UnsupportedOp(f"node {n.name} has no tensor shape info")
        return tuple(int(d) for d in m.shape), _dtype(m.dtype)

    def emit(kind, operands, n, attrs=None):
        shape, dt = meta(n)
        if len(shape) == 0:
            raise UnsupportedOp("rank-0 tensors are unsupported")
        op = _new_op(kind, operands, shape, dt, attrs)
        ops.append(op)
        return op.result

    for n in gm.graph.nodes:
        if n.op in ("placeholder", "get_attr"):
            continue
        if n.op == "output":
            out = n.args[0]
            if not isinstance(out, fx.Node):
                raise UnsupportedOp("exactly one tensor output is supported")
            out_val = env[out]
            continue
        if n.op == "call_module":
            if not extensions:
                raise UnsupportedOp(f"node op call_module ({n.target}) is unsupported (call_module is not inlined)")
            env[n] = _trace_module(gm, n, env, param, ops, meta, emit)
            continue
        if n.op not in ("call_function", "call_method"):
            raise UnsupportedOp(f"node op {n.op} ({n.target}) is unsupported")
        env[n] = _trace_call(n, env, emit, meta, extensions)
    if out_val is None:
        raise UnsupportedOp("graph has no output")
    return Graph(args, ops, out_val, tensors, n_inputs)


def _trace_module(gm, n, env, param, ops, meta, emit):
    mod = _fetch_attr(gm, n.target)
    x = env[n.args[0]]
    if isinstance(mod, torch.nn.Linear):
        shape, dt = meta(n)
        w = param(mod.weight)
        op = _new_op("linear", [x, w], shape, dt)
        ops.append(op)
        if mod.bias is None:
            return op.result
        b = param(mod.bias)
        add = _new_op("add", [op.result, b], shape, dt)
        ops.append(add)
        return add.result
    if isinstance(mod, torch.nn.LayerNorm):
        ins = [x]
        if mod.weight is not None:
            ins += [param(mod.weight), param(mod.bias)]
        return emit("layer_norm", ins, n, {"normalized_shape": list(mod.normalized_shape), "eps": float(mod.eps)})
    if isinstance(mod, torch.nn.GELU):
        if mod.approximate != "none":
            raise UnsupportedOp("only the erf form of GELU is supported")
        return emit("gelu", [x], n)
    if isinstance(mod, torch.nn.ReLU):
        return emit("relu", [x], n)
    if isinstance(mod, (torch.nn.Dropout, torch.nn.Identity)):
        if getattr(mod, "training", False) and isinstance(mod, torch.nn.Dropout) and mod.p > 0:
            raise UnsupportedOp("dropout in training mode is unsupported")
        return x
    raise UnsupportedOp(f"module {type(mod).__name__} is unsupported")


def _norm_axis(dim, rank):
    if dim is None:
        raise UnsupportedOp("softmax requires an explicit dim")
    if not -rank <= dim < rank:
        raise UnsupportedOp(f"softmax dim {dim} out of range")
    return dim % rank


def _trace_call(n, env, emit, meta, extensions):
    tgt, args, kwargs = n.target, n.args, n.kwargs
    is_method = n.op == "call_method"

    def val(x):
        return env[x]

    if (not is_method and tgt in _MATMUL) or (is_method and tgt == "matmul"):
        a, b = args[:2]
        if len(val(a).shape) != len(val(b).shape):
            raise UnsupportedOp("matmul with differing ranks (broadcast) is unsupported")
        return emit("matmul", [val(a), val(b)], n)
    if (not is_method and tgt in _SOFTMAX) or (is_method and tgt == "softmax"):
        x = args[0]
        dim = kwargs.get("dim", args[1] if len(args) > 1 else None)
        if kwargs.get("dtype") is not None:
            raise UnsupportedOp("softmax with dtype= is unsupported")
        return emit("softmax", [val(x)], n, {"axis": _norm_axis(dim, len(val(x).shape))})
    if (not is_method and tgt in _RELU) or (is_method and tgt == "relu"):
        return emit("relu", [val(args[0])], n)
    if (not is_method and tgt is torch.exp) or (is_method and tgt == "exp"):
        return emit("exp", [val(args[0])], n)
    if extensions and ((not is_method and tgt is F.gelu) or (is_method and tgt == "gelu")):
        if kwargs.get("approximate", "none") != "none":
            raise UnsupportedOp("only the erf form of GELU is supported")
        return emit("gelu", [val(args[0])], n)
    if is_method and tgt == "transpose":
        x, d0, d1 = args[:3]
        r = len(val(x).shape)
        if {d0 % r, d1 % r} == {r - 2, r - 1}:
            return emit("transpose", [val(x)], n)
        if not extensions:
            raise UnsupportedOp("only transpose of the last two dims is supported")
        dims = list(range(r))
        dims[d0 % r], dims[d1 % r] = dims[d1 % r], dims[d0 % r]
        return emit("permute", [val(x)], n, {"dims": dims})
    if extensions and is_method and tgt == "permute":
        dims = list(args[1:]) if not isinstance(args[1], (list, tuple)) else list(args[1])
        return emit("permute", [val(args[0])], n, {"dims": [int(d) for d in dims]})
    if extensions and is_method and tgt in ("view", "reshape"):
        shape, _ = meta(n)
        return emit("reshape", [val(args[0])], n, {"shape": list(shape)})
    if extensions and is_method and tgt == "contiguous":
        return val(args[0])

    kind = None
    if not is_method:
        kind = "add" if tgt in _ADD else "mul" if tgt in _MUL else "div" if tgt in _DIV else None
    else:
        kind = {"add": "add", "mul": "mul", "div": "div", "__add__": "add", "__mul__": "mul",
                "__truediv__": "div"}.get(tgt)
    if kind is not None:
        a, b = args[:2]
        a_t, b_t = isinstance(a, fx.Node), isinstance(b, fx.Node)
        if a_t and b_t:
            if kind == "div":
                raise UnsupportedOp("tensor/tensor division is unsupported")
            sa, sb = val(a).shape, val(b).shape
            if sa != sb:
                out_shape, _ = meta(n)
                ok = extensions and (
                    (sa == out_shape and _bcast_ok(sb, out_shape)) or (sb == out_shape and _bcast_ok(sa, out_shape)))
                if not ok:
                    raise UnsupportedOp(f"broadcasting is unsupported: {sa} vs {sb}")
            return emit(kind, [val(a), val(b)], n)
        if kind in ("mul", "div") and (a_t != b_t):
            x, c = (a, b) if a_t else (b, a)
            if kind == "div" and not a_t:
                raise UnsupportedOp("scalar / tensor is unsupported")
            if not isinstance(c, (int, float)):
                raise UnsupportedOp("scale factor must be a Python number")
            factor = float(c) if kind == "mul" else 1.0 / float(c)
            return emit("scale", [val(x)], n, {"factor": float(np.float32(factor))})
        raise UnsupportedOp(f"{kind} with a Python scalar is unsupported (only mul/div by a constant)")
    raise UnsupportedOp(f"unsupported op: {n.op} {tgt}")


# ------------------------------------------------------------ fp text ---
def _ty(v: Val) -> str:
    return "tensor<" + "x".join(str(d) for d in v.shape) + "x" + v.dtype + ">"


def to_mlir(g: Graph, name: str = "main") -> str:
    """The ``fp`` dialect text of an unfused graph (reference ``frontend.py:88-94``)."""
    names = {v: f"%arg{i}" for i, v in enumerate(g.args)}
    lines = []
    for k, op in enumerate(g.ops):
        r = f"%{k}"
        names[op.result] = r
        o = [names[v] for v in op.operands]
        t = _ty(op.result)
        if op.kind == "matmul":
            lines.append(f"{r} = fp.matmul {o[0]}, {o[1]} : ({_ty(op.operands[0])}, {_ty(op.operands[1])}) -> {t}")
        elif op.kind == "softmax":
            lines.append(f"{r} = fp.softmax {o[0]} {{axis = {op.attrs['axis']} : i64}} : {t}")
        elif op.kind == "scale":
            lines.append(f"{r} = fp.scale {o[0]} {{factor = {op.attrs['factor']:.9e} : f32}} : {t}")
        elif op.kind == "transpose":
            lines.append(f"{r} = fp.transpose {o[0]} : {_ty(op.operands[0])} -> {t}")
        elif op.kind in ("add", "mul"):
            lines.append(f"{r} = fp.{op.kind} {o[0]}, {o[1]} : {t}")
        elif op.kind in ("relu", "exp"):
            lines.append(f"{r} = fp.{op.kind} {o[0]} : {t}")
        else:
            lines.append(f"// {r} = {op.kind} (outside the fp dialect)")
    sig = ", ".join(f"%arg{i}: {_ty(v)}" for i, v in enumerate(g.args))
    body = "\n".join("    " + ln for ln in lines)
    outs = g.ret.operands if g.ret is not None else [g.output]
    rty = ", ".join(_ty(v) for v in outs)
    return (f"module {{\n  func.func @{name}({sig}) -> {rty if len(outs) == 1 else '(' + rty + ')'} {{\n{body}\n"
            f"    return {', '.join(names[v] for v in outs)} : {rty}\n  }}\n}}\n")


_TENSOR = re.compile(r"tensor<([0-9x]+)x(f16|f32)>")
_FUNC = re.compile(r"func\.func\s+@(\w+)\s*\((.*?)\)\s*->")
_OPLINE = re.compile(r"^(%[\w.]+)\s*=\s*fp\.(\w+)\s+(.*)$")


def _tensor_type(text: str) -> tuple[tuple, str]:
    m = _TENSOR.search(text)
    if m is None:
        raise UnsupportedOp(f"expected a static f16/f32 tensor type in {text!r}")
    return tuple(int(d) for d in m.group(1).split("x")), m.group(2)


def parse_fp_mlir(text: str) -> dict[str, Graph]:
    """Functions of an ``fp`` dialect module (the textual form ``fusionpass-opt``
    reads: ``fp.add/mul/scale/relu/exp/softmax/transpose/matmul`` and ``return``)
    as unfused graphs, one per ``func.func``.  The reference compiler's passes and
    plan emitter run on this form; here the planner twin runs on it instead."""
    funcs: dict[str, Graph] = {}
    cur = None
    for raw in text.splitlines():
        line = raw.split("//", 1)[0].strip()
        if not line:
            continue
        m = _FUNC.search(line)
        if m is not None:
            args, env = [], {}
            for i, a in enumerate(x for x in m.group(2).split(",") if x.strip()):
                name, ty = a.split(":", 1)
                shape, dt = _tensor_type(ty)
                v = Val(shape, dt, arg_index=i)
                args.append(v)
                env[name.strip()] = v
            cur = (m.group(1), args, env, [])
            continue
        if cur is None:
            continue
        name, args, env, ops = cur
        if line.startswith("return"):
            body, _, _ = line[len("return"):].partition(":")
            outs = [env[x.strip()] for x in body.split(",") if x.strip()]
            g = Graph(args=args, ops=ops, output=outs[0], arg_tensors=[], n_inputs=len(args))
            if len(outs) > 1:
                g.ret = _new_op("return", outs, outs[0].shape, outs[0].dtype)
            funcs[name] = g
            cur = None
            continue
        m = _OPLINE.match(line)
        if m is None:
            continue
        res, kind, rest = m.groups()
        attrs = {}
        am = re.search(r"\{(.*?)\}", rest)
        if am is not None:
            for kv in am.group(1).split(","):
                k, _, v = kv.partition("=")
                v = v.split(":")[0].strip()
                attrs[k.strip()] = float(v) if k.strip() == "factor" else int(v)
            rest = rest[:am.start()] + rest[am.end():]
        head, _, types = rest.partition(" : ")
        operands = [env[x.strip()] for x in head.split(",") if x.strip()]
        shape, dt = _tensor_type(types.split("->")[-1])
        if kind not in ("add", "mul", "scale", "relu", "exp", "softmax", "transpose", "matmul"):
            raise UnsupportedOp(f"fp.{kind} is outside the fp dialect subset")
        op = _new_op(kind, operands, shape, dt, attrs)
        ops.append(op)
        env[res] = op.result
    return funcs


# ------------------------------------------------------------- passes ---
def _replace(g: Graph, old: Op, new: Op, dead: list[Op]) -> None:
    """Put ``new`` at ``old``'s position, redirect uses, drop ``old`` and ``dead``."""
    idx = g.ops.index(old)
    g.ops[idx] = new
    for user in list(old.result.uses):
        user.operands = [new.result if v is old.result else v for v in user.operands]
        new.result.uses.append(user)
    if g.output is old.result:
        g.output = new.result
    for op in [old] + dead:
        op.alive = False
        for v in op.operands:
            while op in v.uses:
                v.uses.remove(op)
    g.ops = [o for o in g.ops if o.alive or o is new]


def fuse_attention(g: Graph) -> int:
    """FuseAttentionPattern: matmul(softmax(scale*...(matmul(Q, transpose(K)))), V)."""
    fused = 0
    for pv in list(g.ops):
        if not pv.alive or pv.kind != "matmul":
            continue
        p, v = pv.operands
        sm = p.producer
        if sm is None or sm.kind != "softmax" or len(p.uses) != 1:
            continue
        if sm.attrs["axis"] != len(sm.result.shape) - 1:
            continue
        scale = 1.0
        cur = sm.operands[0]
        dead = [sm]
        ok = True
        while cur.producer is not None and cur.producer.kind == "scale":
            if len(cur.uses) != 1:
                ok = False
                break
            scale *= float(np.float32(cur.producer.attrs["factor"]))
            dead.append(cur.producer)
            cur = cur.producer.operands[0]
        if not ok:
            continue
        qk = cur.producer
        if qk is None or qk.kind != "matmul" or len(cur.uses) != 1:
            continue
        ktv = qk.operands[1]
        kt = ktv.producer
        if kt is None or kt.kind != "transpose" or len(ktv.uses) != 1:
            continue
        q, k = qk.operands[0], kt.operands[0]
        ty = (q.shape, q.dtype)
        if any((x.shape, x.dtype) != ty for x in (k, v, pv.result)) or len(q.shape) < 3:
            continue
        if q.shape[-1] not in K.HEAD_DIMS:
            continue
        new = _new_op("fused_attention", [q, k, v], pv.result.shape, pv.result.dtype,
                      {"scale": float(np.float32(scale))})
        _replace(g, pv, new, dead + [qk, kt])
        fused += 1
    return fused


def _softmax_count(op: Op) -> int:
    if op.kind == "softmax":
        return 1
    if op.kind == "fused_chain":
        return sum(b[0] == "softmax" for b in op.body)
    return 0


def _chainable(op: Op, ext: bool) -> bool:
    return op.kind == "fused_chain" or op.kind in (CHAINABLE_EXT if ext else CHAINABLE)


def _fusible(op: Op, ext: bool) -> bool:
    if op.kind == "softmax":
        return (op.attrs["axis"] == len(op.result.shape) - 1
                and op.result.shape[-1] <= K.MAX_ROW_SOFTMAX_COLS)
    return _chainable(op, ext)


def _body_of(op: Op, ext_index: dict, base: int, outer_map: dict):
    """Inline ``op`` (plain or fused) as body ops starting at body index ``base``.
    ``outer_map`` maps values defined inside the new body to refs."""
    def ref(v):
        return outer_map[v] if v in outer_map else ("a", ext_index[v])

    if op.kind == "fused_chain":
        inner = [ref(v) for v in op.operands]
        out = []
        for kind, refs, attrs in op.body:
            new_refs = [inner[r[1]] if r[0] == "a" else ("t", base + r[1]) for r in refs]
            out.append((kind, new_refs, dict(attrs)))
        return out, ("t", base + len(op.body) - 1)
    return [(op.kind, [ref(v) for v in op.operands], dict(op.attrs))], ("t", base)


def fuse_chains(g: Graph, *, extensions: bool = False) -> int:
    """FuseChainPattern applied greedily until nothing changes."""
    merges = 0
    changed = True
    while changed:
        changed = False
        for c in list(g.ops):
            if not c.alive or not _chainable(c, extensions) or not _fusible(c, extensions):
                continue
            for pv in list(c.operands):
                p = pv.producer
                if p is None or not p.alive or not _chainable(p, extensions) or not _fusible(p, extensions):
                    continue
                if len(pv.uses) != 1:
                    continue  # a multi-use producer must stay materialised
                if _softmax_count(p) + _softmax_count(c) > 1:
                    continue  # the row kernel supports one reduction
                if p.result.shape != c.result.shape:
                    continue  # a broadcast producer would be recomputed per element
                externals = []
                for x in p.operands + [x for x in c.operands if x is not pv]:
                    if x not in externals:
                        externals.append(x)
                ext_index = {x: i for i, x in enumerate(externals)}
                body_p, p_ref = _body_of(p, ext_index, 0, {})
                body_c, _ = _body_of(c, ext_index, len(body_p), {pv: p_ref})
                new = _new_op("fused_chain", externals, c.result.shape, c.result.dtype, body=body_p + body_c)
                _replace(g, c, new, [p])
                merges += 1
                changed = True
                break
            if changed:
                break
    return merges


def wrap_single_ops(g: Graph) -> None:
    """Nothing to do: like the reference, unfused elementwise ops stay torch steps."""


# --------------------------------------------------------------- plan ---
def _bcast_mode(v: Val, out: tuple) -> str:
    if tuple(v.shape) == tuple(out):
        return "full"
    n = int(np.prod(v.shape))
    if n == 1:
        return "scalar"
    if v.shape[-1] == out[-1] and n == out[-1]:
        return "col"
    return "row"


def _chain_desc(op: Op) -> dict:
    ops = []
    n = len(op.operands)
    for kind, refs, attrs in op.body:
        slots = [r[1] if r[0] == "a" else n + r[1] for r in refs]
        e: dict[str, Any] = {"op": kind, "a": slots[0]}
        if kind in ("add", "mul"):
            e["b"] = slots[1]
        if kind == "scale":
            e["imm"] = float(attrs["factor"])
        ops.append(e)
    rows = any(b[0] == "softmax" for b in op.body)
    return {"op": "chain", "mode": "rows" if rows else "flat",
            "inputs": [{"bcast": _bcast_mode(v, op.result.shape), "dtype": v.dtype} for v in op.operands],
            "ops": ops, "result": n + len(op.body) - 1}


def emit_plan(g: Graph) -> tuple[dict, K.KernelTable]:
    """``emitPlan``: args ``argN``, results ``vN`` in program order, torch / fused steps."""
    names = {v: f"arg{i}" for i, v in enumerate(g.args)}
    inputs = [{"name": f"arg{i}", "shape": list(v.shape), "dtype": v.dtype} for i, v in enumerate(g.args)]
    steps = []
    table = K.KernelTable()
    chains = 0
    for k, op in enumerate(g.live_ops()):
        res = f"v{k}"
        names[op.result] = res
        operands = [names[v] for v in op.operands]
        base = {"operands": operands, "result": res, "shape": list(op.result.shape), "dtype": op.result.dtype}
        if op.kind == "fused_chain":
            kernel = K.chain_kernel_name(chains)
            chains += 1
            desc = _chain_desc(op)
            rows = desc["mode"] == "rows"
            attrs = {**K.chain_launch_attrs(op.result.shape, rows=rows), "desc": desc}
            table[kernel] = desc
            steps.append({"kind": "triton", "kernel": kernel, "launch": "rows" if rows else "flat", **base,
                          "attrs": attrs})
        elif op.kind == "fused_attention":
            desc = K.attention_descriptor(op.result.shape[-1])
            table[K.KERNEL_ATTENTION] = desc
            attrs = {**K.attention_launch_attrs(op.attrs["scale"]), "desc": desc}
            # the result's only consumer swaps heads and sequence ([B, H, S, D] -> [B, S, H, D],
            # as before a merge of the heads): store it in that order, so the permute is a
            # contiguous view and a following reshape copies nothing
            users = op.result.uses
            if (len(users) == 1 and users[0].kind == "permute" and list(users[0].attrs.get("dims", [])) == [0, 2, 1, 3]
                    and len(op.result.shape) == 4 and g.output is not op.result):
                attrs["out_layout"] = [0, 2, 1, 3]
            steps.append({"kind": "triton", "kernel": K.KERNEL_ATTENTION, "launch": "attention", **base,
                          "attrs": attrs})
        else:
            attrs = {}
            if op.kind == "scale":
                attrs["factor"] = float(op.attrs["factor"])
            elif op.kind == "softmax":
                attrs["axis"] = int(op.attrs["axis"])
            elif op.kind in ("reshape", "permute", "layer_norm", "add_layer_norm", "cat", "narrow"):
                attrs = dict(op.attrs)
            steps.append({"kind": "torch", "op": op.kind, **base, "attrs": attrs})
    outs = g.ret.operands if g.ret is not None else [g.output]
    plan = {"version": 1, "inputs": inputs, "steps": steps, "outputs": [names[v] for v in outs]}
    return plan, table


def fold_linear_bias(g: Graph) -> int:
    """Extension graphs: an ``nn.Linear`` is traced as ``linear`` + a bias ``add`` so that
    the add can join a chain (bias + GELU, bias + residual).  A bias add that no chain
    took is folded back into its ``linear`` step (three operands: x, W, b), which runs
    it in the GEMM's epilogue, as eager ``nn.Linear`` does, instead of as a separate pass
    over the output.  Returns the number of folds."""
    folds = 0
    for add in list(g.ops):
        if not add.alive or add.kind != "add" or len(add.operands) != 2:
            continue
        y, b = add.operands
        lin = y.producer
        if lin is None or not lin.alive or lin.kind != "linear" or len(lin.operands) != 2:
            continue
        if len(y.uses) != 1 or g.output is y or (g.ret is not None and y in g.ret.operands):
            continue
        if b.arg_index is None or tuple(b.shape) != (y.shape[-1],) or tuple(add.result.shape) != tuple(y.shape):
            continue
        new = _new_op("linear", [lin.operands[0], lin.operands[1], b], y.shape, y.dtype, lin.attrs)
        _replace(g, add, new, [lin])
        folds += 1
    return folds


def fuse_add_layer_norm(g: Graph) -> int:
    """Extension graphs: a chain of adds (a residual plus a bias) whose only consumer is a
    LayerNorm over the last axis becomes one ``add_layer_norm`` step that sums the chain's
    operands in the chain's order and normalises, so the sum is never written out.  Only
    where the LayerNorm kernel takes the shape (last dim a multiple of 8, at most 2048,
    one dtype); returns the number of fusions."""
    fused = 0
    for ln in list(g.ops):
        if not ln.alive or ln.kind != "layer_norm" or len(ln.operands) not in (1, 3):
            continue
        x = ln.operands[0]
        ch = x.producer
        cols = x.shape[-1] if x.shape else 0
        if (ch is None or not ch.alive or ch.kind != "fused_chain" or len(x.uses) != 1 or g.output is x
                or list(ln.attrs.get("normalized_shape", [])) != [cols] or cols % 8 or cols > 2048 or cols == 0):
            continue
        if g.ret is not None and x in g.ret.operands:
            continue
        order = []
        ok = all(kind == "add" for kind, _, _ in ch.body)
        for k, (_, refs, _) in enumerate(ch.body if ok else []):
            temps = [r for r in refs if r[0] == "t"]
            args = [r[1] for r in refs if r[0] == "a"]
            if (k == 0 and temps) or (k > 0 and temps != [("t", k - 1)]):
                ok = False
                break
            order += args
        ext = ch.operands
        if (not ok or sorted(order) != list(range(len(ext))) or len(ext) > 4
                or any(v.dtype != x.dtype or _bcast_mode(v, x.shape) not in ("full", "col") for v in ext)
                or any(v.dtype != x.dtype for v in ln.operands[1:])):
            continue
        new = _new_op("add_layer_norm", [ext[i] for i in order] + list(ln.operands[1:]), ln.result.shape,
                      ln.result.dtype, {**ln.attrs, "n_addends": len(order)})
        _replace(g, ln, new, [ch])
        fused += 1
    return fused


def merge_sibling_linears(g: Graph) -> int:
    """Extension graphs: ``linear`` steps (with their biases) that read the same input —
    the q / k / v projections of an attention block — become one GEMM over the
    concatenated weights and biases (``cat`` steps, a few MB per call) followed by one
    ``narrow`` view per original output, so the projections run as one wider GEMM and the
    attention reads its operands straight out of its result.  Returns the number of
    linear steps merged away."""
    merged = 0
    groups: dict[int, list[Op]] = {}
    for op in g.ops:
        if op.alive and op.kind == "linear" and len(op.operands) == 3:
            w, b = op.operands[1], op.operands[2]
            if w.arg_index is not None and b.arg_index is not None and len(w.shape) == 2:
                groups.setdefault(id(op.operands[0]), []).append(op)
    for sibs in groups.values():
        if len(sibs) < 2 or len({(o.result.dtype, o.operands[1].shape[1]) for o in sibs}) != 1:
            continue
        x = sibs[0].operands[0]
        dt = sibs[0].result.dtype
        outs = [o.operands[1].shape[0] for o in sibs]
        total = sum(outs)
        lead = tuple(sibs[0].result.shape[:-1])
        cat_w = _new_op("cat", [o.operands[1] for o in sibs], (total, sibs[0].operands[1].shape[1]), dt, {"dim": 0})
        cat_b = _new_op("cat", [o.operands[2] for o in sibs], (total,), dt, {"dim": 0})
        lin = _new_op("linear", [x, cat_w.result, cat_b.result], lead + (total,), dt)
        at = g.ops.index(sibs[0])
        g.ops[at:at] = [cat_w, cat_b, lin]
        start = 0
        for o, n in zip(sibs, outs):
            view = _new_op("narrow", [lin.result], o.result.shape, dt, {"dim": -1, "start": start, "length": n})
            _replace(g, o, view, [])
            start += n
        merged += len(sibs) - 1
    return merged


def compile_graph(g: Graph, *, fuse: bool, extensions: bool = False) -> tuple[dict, K.KernelTable]:
    if fuse:
        fuse_attention(g)  # attention first so its scale/softmax are absorbed before chain fusion
        fuse_chains(g, extensions=extensions)
        if extensions:
            fold_linear_bias(g)
            merge_sibling_linears(g)
            fuse_add_layer_norm(g)
    return emit_plan(g)
