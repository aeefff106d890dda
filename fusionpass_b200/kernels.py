"""Fused-step launch boundary: descriptors + libfpkern instead of generated Triton.

Mirrors the reference module ``python/fusionpass/kernels.py``:

* the plan/launch constants and attribute helpers (``kernels.py:33-40,97-126``)
  are kept so existing plans (``launch`` in {flat, rows, attention}, the
  ``block``/``block_n``/``num_warps`` attrs) stay valid;
* ``DescriptorWriter`` replaces ``KernelModuleWriter`` (``kernels.py:214-254``):
  it takes the same chain-body format and returns the same kernel names
  (``fp_chain_<N>``, ``fp_attention``) but records a launch descriptor (op list,
  operand dtypes and broadcast modes) instead of Triton source;
* ``launch_step`` (``kernels.py:336-368``) keeps its signature, argument meaning
  and errors (``RuntimeError`` without kernels, ``ValueError`` for an unknown
  launch) and enqueues the step in ``libfpkern.so`` on the current CUDA stream.

There is no Triton import, no CPU path and no second backend.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Mapping, Sequence

# --- plan / launch constants (same values as the reference plan emitter) ---
FLAT_BLOCK = 1024
ATTENTION_BLOCK_M = 64
ATTENTION_BLOCK_N = 64
ATTENTION_NUM_WARPS = 4
ATTENTION_NUM_STAGES = 2
MAX_ROW_SOFTMAX_COLS = 8192
HEAD_DIMS = (16, 32, 64, 128)
KERNEL_ATTENTION = "fp_attention"

CHAINABLE = ("add", "mul", "scale", "relu", "exp", "softmax")
# chain ops this backend adds beyond the reference dialect (for bias + GELU chains)
EXTENSION_OPS = ("gelu",)
_BINARY = ("add", "mul")
LAUNCHES = ("flat", "rows", "attention")


def chain_kernel_name(index: int) -> str:
    return f"fp_chain_{int(index)}"


def next_pow2(n: int) -> int:
    """Smallest power of two ``>= n`` (``n >= 1``), like ``llvm::PowerOf2Ceil``."""
    n = int(n)
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def chain_launch_attrs(shape: Sequence[int], *, rows: bool) -> dict[str, int]:
    """``plan.json`` attrs of a fused-chain step (reference ``PlanEmitter.cpp:126-133``)."""
    if rows:
        block_n = next_pow2(int(shape[-1]))
        return {"block_n": block_n, "num_warps": 4 if block_n <= 2048 else 8}
    return {"block": FLAT_BLOCK}


def attention_launch_attrs(scale: float) -> dict[str, Any]:
    """``plan.json`` attrs of the attention step (reference ``PlanEmitter.cpp:140-145``)."""
    return {
        "scale": float(scale),
        "block_m": ATTENTION_BLOCK_M,
        "block_n": ATTENTION_BLOCK_N,
        "num_warps": ATTENTION_NUM_WARPS,
        "num_stages": ATTENTION_NUM_STAGES,
    }


def chain_descriptor(n_args: int, body: Sequence[Mapping[str, Any]], *, rows: bool | None = None,
                     yield_value: str | None = None, input_bcast: Sequence[str] | None = None,
                     input_dtypes: Sequence[str] | None = None) -> dict[str, Any]:
    """Descriptor of one fused chain from a reference-format body.

    ``body``: dicts ``{"op", "operands", "factor"}`` in program order; operand
    names are ``a<i>`` for block arguments and ``t<k>`` (or a custom
    ``out``/``result``) for earlier results, as in the reference's
    ``emit_chain_kernel`` (``kernels.py:139-146``).
    """
    n_args = int(n_args)
    if rows is None:
        rows = any(op.get("op") == "softmax" for op in body)
    names = {f"a{i}": i for i in range(n_args)}
    ops = []
    last = n_args - 1 if n_args else None
    n_softmax = 0
    for k, op in enumerate(body):
        kind = op["op"]
        if kind not in CHAINABLE + EXTENSION_OPS:
            raise ValueError(f"unsupported op in chain: {kind}")
        try:
            srcs = [names[x] for x in op.get("operands", ())]
        except KeyError as e:
            raise ValueError(f"chain op {k} uses undefined value {e.args[0]!r}") from None
        if len(srcs) != (2 if kind in _BINARY else 1):
            raise ValueError(f"chain op {k} ({kind}) has {len(srcs)} operands")
        entry: dict[str, Any] = {"op": kind, "a": srcs[0]}
        if kind in _BINARY:
            entry["b"] = srcs[1]
        if kind == "scale":
            entry["imm"] = float(op["factor"])
        if kind == "softmax":
            n_softmax += 1
        ops.append(entry)
        slot = n_args + k
        names[op.get("out") or op.get("result") or f"t{k}"] = slot
        last = slot
    if rows and n_softmax != 1:
        raise ValueError("a rows chain needs exactly one softmax")
    if not rows and n_softmax:
        raise ValueError("a flat chain cannot contain softmax")
    result = names[yield_value] if yield_value is not None else last
    if result is None:
        raise ValueError("chain kernel has no value to store")
    bc = list(input_bcast) if input_bcast is not None else ["full"] * n_args
    dts = list(input_dtypes) if input_dtypes is not None else [None] * n_args
    return {
        "op": "chain",
        "mode": "rows" if rows else "flat",
        "inputs": [{"bcast": b, **({"dtype": d} if d else {})} for b, d in zip(bc, dts)],
        "ops": ops,
        "result": result,
    }


def attention_descriptor(head_dim: int | None = None) -> dict[str, Any]:
    d: dict[str, Any] = {"op": "attention"}
    if head_dim is not None:
        d["head_dim"] = int(head_dim)
    return d


class KernelTable(dict):
    """kernel name -> descriptor; plays the role of the reference's loaded
    ``kernels.py`` module in ``execute_plan(plan, args, kernels)``."""

    def to_json(self) -> str:
        return json.dumps({"version": 1, "kernels": dict(self)}, indent=2)


class DescriptorWriter:
    """Twin of the reference ``KernelModuleWriter`` that records descriptors."""

    def __init__(self) -> None:
        self.chain_count = 0
        self.has_attention = False
        self.table = KernelTable()

    def add_chain_kernel(self, n_args: int, body: Sequence[Mapping[str, Any]], *, rows: bool | None = None,
                         yield_value: str | None = None, input_bcast: Sequence[str] | None = None) -> str:
        name = chain_kernel_name(self.chain_count)
        self.chain_count += 1
        self.table[name] = chain_descriptor(n_args, body, rows=rows, yield_value=yield_value,
                                            input_bcast=input_bcast)
        return name

    def add_attention_kernel(self) -> str:
        self.has_attention = True
        self.table[KERNEL_ATTENTION] = attention_descriptor()
        return KERNEL_ATTENTION

    def write(self) -> KernelTable:
        return KernelTable(self.table)

    def write_path(self, path) -> Path:
        path = Path(path)
        path.write_text(self.table.to_json(), encoding="utf-8")
        return path


def load_kernels(path) -> KernelTable:
    """Load a ``kernels.json`` descriptor table written by ``DescriptorWriter``."""
    data = json.loads(Path(path).read_text(encoding="utf-8"))
    if data.get("version") != 1 or not isinstance(data.get("kernels"), dict):
        raise ValueError(f"{path}: not a fusionpass descriptor table")
    return KernelTable(data["kernels"])


def check_device(t) -> None:
    """Fused steps need CUDA tensors: libfpkern has no CPU path."""
    if getattr(t, "device", None) is None or t.device.type != "cuda":
        raise RuntimeError(
            "fused steps run only in libfpkern.so on a CUDA device (sm_100); "
            f"got a tensor on {getattr(t, 'device', None)}. There is no CPU or Triton fallback.")


def _torch_dtype(dtype: str):
    import torch

    if dtype == "f32":
        return torch.float32
    if dtype == "f16":
        return torch.float16
    raise ValueError(f"unsupported dtype {dtype!r}")


def _step_desc(step: Mapping[str, Any], kernels) -> Mapping[str, Any]:
    desc = step.get("attrs", {}).get("desc")
    if desc is not None:
        return desc
    if kernels is None:
        raise RuntimeError("plan has triton steps but no kernels module was provided")
    try:
        return kernels[step["kernel"]]
    except (KeyError, TypeError):
        raise RuntimeError(f"no descriptor for kernel {step.get('kernel')!r}") from None


def launch_flat(desc, ops: Sequence[Any], out, flags: int = 0):
    from . import fpkern

    return fpkern.chain(ops, desc, list(out.shape), out.dtype, out=out, flags=flags, mode="flat")


def launch_rows(desc, ops: Sequence[Any], out, flags: int = 0):
    from . import fpkern

    if int(out.shape[-1]) > 16384:
        raise ValueError(f"rows chain with {int(out.shape[-1])} columns exceeds the on-chip row limit")
    return fpkern.chain(ops, desc, list(out.shape), out.dtype, out=out, flags=flags, mode="rows")


def launch_attention(q, k, v, out, *, scale: float, flags: int = 0, **_ignored):
    """Launch attrs ``block_m/block_n/num_warps/num_stages`` of the reference plan are
    accepted and ignored: the sm_100a kernel picks its own tiling."""
    from . import fpkern

    return fpkern.attention(q, k, v, scale, out=out, flags=flags)


def launch_step(step: dict, ops: Sequence[Any], kernels):
    """Launch one fused (``kind == "triton"``) plan step in libfpkern.so."""
    import torch

    desc = _step_desc(step, kernels)
    launch = step["launch"]
    if launch not in LAUNCHES:
        raise ValueError(f"unknown launch kind {launch}")
    check_device(ops[0])
    a = step["attrs"]
    layout = a.get("out_layout") if launch == "attention" else None
    if layout is not None:
        # stored as the permutation `layout` of the step's shape (a self-inverse swap of
        # two axes): the result is a strided view of that buffer, which the attention
        # kernel writes through its output strides
        perm = [int(i) for i in layout]
        if sorted(perm) != list(range(len(step["shape"]))) or [perm[i] for i in perm] != list(range(len(perm))):
            raise ValueError(f"out_layout {layout} is not a self-inverse permutation of the result's axes")
        buf = torch.empty([step["shape"][i] for i in perm], dtype=_torch_dtype(step["dtype"]), device=ops[0].device)
        out = buf.permute(*perm)
    else:
        out = torch.empty(step["shape"], dtype=_torch_dtype(step["dtype"]), device=ops[0].device)
    if launch == "flat":
        launch_flat(desc, ops, out)
    elif launch == "rows":
        launch_rows(desc, ops, out)
    else:
        if len(ops) != 3:
            raise ValueError("attention needs exactly 3 operands")
        q, k, v = ops  # strided [B, H, S, D] views go straight to the strided TMA maps
        launch_attention(q, k, v, out, scale=a["scale"])
    return out
