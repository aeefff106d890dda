"""ctypes binding of ``libfpkern.so`` (the C ABI declared in ``include/fpkern.h``).

The library is loaded from the package directory (or ``$FUSIONPASS_FPKERN_LIB``).
There is no fallback: if the library cannot be loaded, every fused step raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PKG = Path(__file__).resolve().parent

# ---- constants mirrored from include/fpkern.h --------------------------------
FPK_ABI_VERSION = 1
FPK_OK = 0
FPK_ERR_INVALID = -1
FPK_ERR_UNSUPPORTED = -2
FPK_ERR_ALIGN = -3
FPK_ERR_CUDA = -4
FPK_ERR_DEVICE = -5
FPK_ERR_TIMEOUT = -6

FPK_F32 = 0
FPK_F16 = 1

FPK_FLAG_TEST_TIMEOUT = 0x1
FPK_FLAG_NO_STAGING = 0x2
FPK_FLAG_NO_JIT = 0x4

FPK_CHAIN_MAX_INPUTS = 8
FPK_CHAIN_MAX_OPS = 32
FPK_CHAIN_MAX_ROW_COLS = 16384

OPCODES = {"add": 1, "mul": 2, "scale": 3, "relu": 4, "exp": 5, "softmax": 6, "gelu": 7}
BCAST = {"full": 0, "col": 1, "row": 2, "scalar": 3}
FPK_CHAIN_FLAT = 0
FPK_CHAIN_ROWS = 1

EXPORTS = (
    "fpk_version",
    "fpk_status_string",
    "fpk_device_check",
    "fpk_attn_desc_init",
    "fpk_attention_fwd",
    "fpk_chain_fwd",
    "fpk_chain_precompile",
    "fpk_chain_jit_launches",
    "fpk_layer_norm_fwd",
    "fpk_add_layer_norm_fwd",
    "fpk_poll_status",
)
FPK_LN_MAX_COLS = 2048


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("size", ctypes.c_uint32),
        ("version", ctypes.c_uint32),
        ("dtype", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("seq_len", ctypes.c_int64),
        ("scale", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("q_strides", ctypes.c_int64 * 3),
        ("k_strides", ctypes.c_int64 * 3),
        ("v_strides", ctypes.c_int64 * 3),
        ("o_strides", ctypes.c_int64 * 3),
    ]


class ChainOp(ctypes.Structure):
    _fields_ = [
        ("opcode", ctypes.c_int32),
        ("src_a", ctypes.c_int32),
        ("src_b", ctypes.c_int32),
        ("imm", ctypes.c_float),
    ]


class ChainDesc(ctypes.Structure):
    _fields_ = [
        ("size", ctypes.c_uint32),
        ("version", ctypes.c_uint32),
        ("mode", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("n_inputs", ctypes.c_int32),
        ("n_ops", ctypes.c_int32),
        ("result", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("in_dtype", ctypes.c_int32 * FPK_CHAIN_MAX_INPUTS),
        ("in_bcast", ctypes.c_int32 * FPK_CHAIN_MAX_INPUTS),
        ("ops", ChainOp * FPK_CHAIN_MAX_OPS),
    ]


class LnDesc(ctypes.Structure):
    _fields_ = [
        ("size", ctypes.c_uint32),
        ("version", ctypes.c_uint32),
        ("dtype", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("eps", ctypes.c_float),
        ("flags", ctypes.c_uint32),
    ]


class FpkernError(RuntimeError):
    """A libfpkern entry point returned a negative status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} (status {status})")


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    env = os.environ.get("FUSIONPASS_FPKERN_LIB")
    return Path(env) if env else PKG / "libfpkern.so"


def load() -> ctypes.CDLL:
    """Load libfpkern.so once; raise (never fall back) if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.exists():
            raise RuntimeError(
                f"libfpkern.so not found at {path}; build it with `python -m fusionpass_b200.build` "
                "(there is no CPU or Triton fallback for fused steps)")
        lib = ctypes.CDLL(str(path))
        lib.fpk_version.restype = ctypes.c_int
        lib.fpk_status_string.restype = ctypes.c_char_p
        lib.fpk_status_string.argtypes = [ctypes.c_int]
        lib.fpk_device_check.restype = ctypes.c_int
        lib.fpk_device_check.argtypes = [ctypes.c_int]
        lib.fpk_attn_desc_init.restype = ctypes.c_int
        lib.fpk_attn_desc_init.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_int, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_float]
        lib.fpk_attention_fwd.restype = ctypes.c_int
        lib.fpk_attention_fwd.argtypes = [ctypes.POINTER(AttnDesc), ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.fpk_chain_fwd.restype = ctypes.c_int
        lib.fpk_chain_fwd.argtypes = [ctypes.POINTER(ChainDesc), ctypes.POINTER(ctypes.c_void_p),
                                      ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        lib.fpk_chain_precompile.restype = ctypes.c_int
        lib.fpk_chain_precompile.argtypes = [ctypes.POINTER(ChainDesc)]
        lib.fpk_chain_jit_launches.restype = ctypes.c_int64
        lib.fpk_chain_jit_launches.argtypes = []
        lib.fpk_add_layer_norm_fwd.restype = ctypes.c_int
        lib.fpk_add_layer_norm_fwd.argtypes = [ctypes.POINTER(LnDesc), ctypes.POINTER(ctypes.c_void_p),
                                               ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.fpk_layer_norm_fwd.restype = ctypes.c_int
        lib.fpk_layer_norm_fwd.argtypes = [ctypes.POINTER(LnDesc), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_void_p, ctypes.c_void_p]
        lib.fpk_poll_status.restype = ctypes.c_int
        lib.fpk_poll_status.argtypes = [ctypes.c_int, ctypes.c_void_p]
        if lib.fpk_version() != FPK_ABI_VERSION:
            raise RuntimeError(f"libfpkern ABI {lib.fpk_version()} != expected {FPK_ABI_VERSION}")
        _lib = lib
        return lib


def status_string(status: int) -> str:
    try:
        return load().fpk_status_string(int(status)).decode()
    except RuntimeError:
        return f"status {status}"


def check(status: int, what: str) -> None:
    if status != FPK_OK:
        raise FpkernError(status, what)
