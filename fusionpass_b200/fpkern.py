"""Tensor-level calls into libfpkern: descriptors in, kernels enqueued on torch's stream.

Descriptor format (what a plan step carries in ``attrs["desc"]``)::

    chain:     {"op": "chain", "mode": "flat" | "rows",
                "inputs": [{"dtype": "f16", "bcast": "full" | "col" | "row" | "scalar"}, ...],
                "ops": [{"op": "add", "a": 0, "b": 1}, {"op": "scale", "a": 2, "imm": 0.5}, ...],
                "result": <slot>}
    attention: {"op": "attention", "scale": <float>, "head_dim": <16|32|64|128>}

Slots ``0..n_inputs-1`` are the step's operands in order; slot ``n_inputs + k`` is
the result of op ``k``.  All math is f32 with one rounding at the store.
PyTorch supplies device memory and the current CUDA stream only; every fused
step runs in ``libfpkern.so`` and there is no CPU path.  Launches go through the
torch C++ extension ``fusionpass_b200._fpkern`` (``csrc/torch_ext.cpp``), which
builds the C descriptors and takes torch's current stream; the ctypes binding in
``_lib`` serves the ahead-of-time chain compile, the status word and the tests of
the raw C ABI.
"""

from __future__ import annotations

import ctypes
from typing import Any, Mapping, Sequence

import torch

from . import _lib

_TORCH_DT = {torch.float32: _lib.FPK_F32, torch.float16: _lib.FPK_F16}
_NAME_DT = {"f32": _lib.FPK_F32, "f16": _lib.FPK_F16}
_DT_NAME = {torch.float32: "f32", torch.float16: "f16"}

_ext_mod = None


def extension():
    """The torch C++ extension; raises (never falls back) when it is not built."""
    global _ext_mod
    if _ext_mod is None:
        _lib.load()  # the extension links libfpkern.so: report a missing library first
        try:
            from . import _fpkern
        except ImportError as e:
            raise RuntimeError("the torch extension fusionpass_b200._fpkern is not built; build it with "
                               "`python -m fusionpass_b200.build` (there is no CPU or Triton fallback for "
                               f"fused steps): {e}") from None
        _ext_mod = _fpkern
    return _ext_mod


def _stream_handle(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(t: torch.Tensor, what: str) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise RuntimeError(f"{what}: fused steps run only in libfpkern.so on a CUDA device "
                           f"(got {getattr(t, 'device', type(t))}); there is no CPU path")


def _bcast_of(t: torch.Tensor, rows: int, cols: int, declared: str | None) -> str:
    n = t.numel()
    if declared is not None:
        want = {"full": rows * cols, "col": cols, "row": rows, "scalar": 1}[declared]
        if n != want:
            raise ValueError(f"operand with {n} elements does not match broadcast '{declared}' "
                             f"of a [{rows}, {cols}] chain")
        return declared
    if n == rows * cols:
        return "full"
    if n == 1:
        return "scalar"
    if n == cols and n == rows:
        # square output: the operand's shape decides, as torch broadcasting places it --
        # [..., 1] is one value per row, [cols] or [1, cols] one value per column
        if t.dim() >= 2 and t.shape[-1] == 1:
            return "row"
        if t.dim() == 1 or (t.shape[-1] == cols and t.shape[-2] == 1):
            return "col"
        raise ValueError(f"operand of shape {tuple(t.shape)} is ambiguous on a [{rows}, {cols}] chain: "
                         "declare its broadcast in the descriptor's 'inputs'")
    if n == cols:
        return "col"
    if n == rows:
        return "row"
    raise ValueError(f"operand with {n} elements cannot broadcast onto [{rows}, {cols}]")


def build_chain_desc(desc: Mapping[str, Any], rows: int, cols: int, in_dtypes: Sequence[int],
                     bcasts: Sequence[str], out_dtype: int, flags: int = 0,
                     mode: str | None = None) -> _lib.ChainDesc:
    """Fill the C descriptor for one chain launch (validated again by the library).
    ``mode`` ("flat" / "rows") overrides the descriptor's own."""
    ops = desc["ops"]
    n_in = len(in_dtypes)
    if not 1 <= n_in <= _lib.FPK_CHAIN_MAX_INPUTS:
        raise ValueError(f"chain needs 1..{_lib.FPK_CHAIN_MAX_INPUTS} inputs, got {n_in}")
    if not 1 <= len(ops) <= _lib.FPK_CHAIN_MAX_OPS:
        raise ValueError(f"chain needs 1..{_lib.FPK_CHAIN_MAX_OPS} ops, got {len(ops)}")
    d = _lib.ChainDesc()
    d.size = ctypes.sizeof(_lib.ChainDesc)
    d.version = _lib.FPK_ABI_VERSION
    d.mode = _lib.FPK_CHAIN_ROWS if (mode or desc.get("mode")) == "rows" else _lib.FPK_CHAIN_FLAT
    d.out_dtype = out_dtype
    d.rows = rows
    d.cols = cols
    d.n_inputs = n_in
    d.n_ops = len(ops)
    d.result = int(desc["result"])
    d.flags = flags
    for i in range(n_in):
        d.in_dtype[i] = in_dtypes[i]
        d.in_bcast[i] = _lib.BCAST[bcasts[i]]
    for k, op in enumerate(ops):
        name = op["op"]
        if name not in _lib.OPCODES:
            raise ValueError(f"unsupported op in chain: {name}")
        d.ops[k].opcode = _lib.OPCODES[name]
        d.ops[k].src_a = int(op["a"])
        d.ops[k].src_b = int(op.get("b", -1))
        d.ops[k].imm = float(op.get("imm", 0.0))
    return d


def chain(inputs: Sequence[torch.Tensor], desc: Mapping[str, Any], out_shape, out_dtype: torch.dtype,
          out: torch.Tensor | None = None, flags: int = 0, mode: str | None = None) -> torch.Tensor:
    """Run one fused chain; ``out_shape`` is the step's result shape ([..., cols]).
    ``mode`` ("flat" / "rows", the plan step's launch) overrides the descriptor's."""
    ext = extension()
    out_shape = [int(s) for s in out_shape]
    if not inputs:
        raise ValueError("chain needs at least one input")
    for t in inputs:
        require_cuda(t, "chain")
    dev = inputs[0].device
    for t in inputs:
        if t.dtype not in _TORCH_DT:
            raise ValueError(f"unsupported dtype {t.dtype}")
        if t.device != dev:
            raise ValueError("all chain operands must be on one device")
    if out is None:
        out = torch.empty(out_shape, dtype=out_dtype, device=dev)
    elif not out.is_contiguous() or list(out.shape) != out_shape or out.dtype != out_dtype:
        raise ValueError("out must be a contiguous tensor of the step's shape and dtype")
    ext.chain([t.contiguous() for t in inputs], out, desc, flags, mode)
    return out


def precompile_chain(desc: Mapping[str, Any], cols: int, in_dtypes: Sequence[torch.dtype], bcasts: Sequence[str],
                     out_dtype: torch.dtype, flags: int = 0) -> bool:
    """Compile and cache the run-time specialised kernel of a flat chain before its
    first launch (the first ``chain`` call with this op list, operand dtypes and
    broadcast modes would do the same).  Needs no GPU.  Returns False when the
    chain runs on the prebuilt kernels instead (rows mode, ``cols % 8 != 0``,
    ``FPK_FLAG_NO_JIT``, or no run-time compiler in the process)."""
    lib = _lib.load()
    c = build_chain_desc(desc, 1, int(cols), [_TORCH_DT[dt] for dt in in_dtypes], list(bcasts),
                         _TORCH_DT[out_dtype], flags)
    rc = lib.fpk_chain_precompile(ctypes.byref(c))
    if rc == _lib.FPK_ERR_UNSUPPORTED:
        return False
    _lib.check(rc, "fpk_chain_precompile")
    return True


def chain_jit_launches() -> int:
    """Flat chains launched so far through run-time compiled kernels (diagnostic)."""
    return int(_lib.load().fpk_chain_jit_launches())


def _bhsd(t: torch.Tensor):
    """(B, H, S, D, strides[b, h, s]) of a [..., S, D] tensor with a unit D stride."""
    if t.dim() < 3:
        raise ValueError("attention tensors must have rank >= 3 ([batch..., S, D])")
    if t.stride(-1) != 1:
        t = t.contiguous()
    S, D = t.shape[-2], t.shape[-1]
    if t.dim() == 3:
        B, H = 1, t.shape[0]
        st = (t.shape[0] * t.stride(0), t.stride(0), t.stride(1))
    else:
        lead = t.shape[:-3]
        B = 1
        for s in lead:
            B *= s
        H = t.shape[-3]
        # leading dims must flatten to one stride
        if t.dim() > 4:
            exp = t.stride(-4)
            for i in range(t.dim() - 5, -1, -1):
                exp *= t.shape[i + 1]
                if t.stride(i) != exp:
                    t = t.contiguous()
                    break
        b_stride = t.stride(-4) if t.dim() >= 4 else H * t.stride(-3)
        st = (b_stride, t.stride(-3), t.stride(-2))
    return t, B, H, S, D, st


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
              out: torch.Tensor | None = None, flags: int = 0) -> torch.Tensor:
    """``softmax(scale * q @ k^T) @ v`` over ``[..., S, D]`` (self-attention shapes)."""
    ext = extension()
    for t in (q, k, v):
        require_cuda(t, "attention")
    if not (q.shape == k.shape == v.shape) or not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k, v must share one shape and dtype (FusedAttentionOp contract)")
    if q.dtype not in _TORCH_DT:
        raise ValueError(f"unsupported dtype {q.dtype}")
    q, k, v = (_bhsd(t)[0] for t in (q, k, v))  # strided views pass as they are; others are copied
    if out is None:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    elif out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("out must match q's shape and dtype")
    elif _bhsd(out)[0].data_ptr() != out.data_ptr():
        raise ValueError("out must have a unit stride in its last dim and flattenable batch dims")
    ext.attention(q, k, v, out, {"scale": float(scale)}, flags)
    return out


def layer_norm(x: torch.Tensor, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float,
               out: torch.Tensor | None = None) -> torch.Tensor | None:
    """LayerNorm over the last axis of a CUDA tensor in libfpkern.so (f16 / f32, last dim a
    multiple of 8 and at most 2048, weight and bias of x's dtype or both None).  Returns
    None when the kernel does not take the shape; the caller then runs torch's."""
    ext = extension()
    require_cuda(x, "layer_norm")
    if x.dtype not in _TORCH_DT or x.dim() < 1:
        return None
    if (weight is None) != (bias is None):
        return None
    if weight is not None and (weight.dtype != x.dtype or bias.dtype != x.dtype):
        return None
    cols = x.shape[-1]
    if cols % 8 or cols > _lib.FPK_LN_MAX_COLS or cols == 0:
        return None
    x = x.contiguous()
    if out is None:
        out = torch.empty_like(x)
    w = weight.contiguous() if weight is not None else None
    b = bias.contiguous() if bias is not None else None
    return out if ext.layer_norm(x, w, b, out, float(eps)) else None


def add_layer_norm(addends, weight: torch.Tensor | None, bias: torch.Tensor | None, eps: float,
                   out: torch.Tensor | None = None, shape=None) -> torch.Tensor | None:
    """LayerNorm over the last axis of ``addends[0] + addends[1] + ...`` (1 to 4 CUDA
    tensors of the result's shape or vectors of its last dim, summed in f32 in order) in
    libfpkern.so; None when the kernel does not take the shapes or dtypes.  ``shape`` is
    the result's shape (default: that of the addend with the most elements)."""
    ext = extension()
    addends = list(addends)
    if not 1 <= len(addends) <= 4:
        return None
    if shape is None:
        shape = max(addends, key=lambda t: t.numel()).shape
    shape = tuple(int(d) for d in shape)
    if not shape:
        return None
    dt = addends[0].dtype
    for t in addends:
        require_cuda(t, "add_layer_norm")
        if t.dtype != dt or (tuple(t.shape) != tuple(shape) and t.numel() != shape[-1]):
            return None
    if dt not in _TORCH_DT or (weight is None) != (bias is None):
        return None
    if weight is not None and (weight.dtype != dt or bias.dtype != dt):
        return None
    cols = shape[-1]
    if cols % 8 or cols > _lib.FPK_LN_MAX_COLS or cols == 0:
        return None
    addends = [t.contiguous() for t in addends]
    if out is None:
        out = torch.empty(shape, dtype=dt, device=addends[0].device)
    w = weight.contiguous() if weight is not None else None
    b = bias.contiguous() if bias is not None else None
    return out if ext.add_layer_norm(addends, w, b, out, float(eps)) else None


def poll_status(device: torch.device | int | None = None) -> int:
    """Synchronise the current stream and return/clear the device status word."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index or 0))
    return int(lib.fpk_poll_status(dev.index, _stream_handle(dev)))
