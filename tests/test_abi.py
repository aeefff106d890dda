"""The C ABI library loads and exports every entry point include/fpkern.h declares,
and the ctypes mirrors have the C layout (checked against gcc).  No GPU needed."""

import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from fusionpass_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fpkern.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(fpk_[a-z_]+)\s*\(", text)))


def test_header_declares_the_bound_entry_points():
    assert _declared() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name
    nm = shutil.which("nm")
    if nm:
        out = subprocess.run([nm, "-D", "--defined-only", str(_lib.library_path())],
                             capture_output=True, text=True).stdout
        exported = set(re.findall(r" T (fpk_\w+)", out))
        assert set(_declared()) <= exported


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.fpk_version() == _lib.FPK_ABI_VERSION == 1
    for code in (0, -1, -2, -3, -4, -5, -6):
        assert _lib.status_string(code)
    assert "timed out" in _lib.status_string(_lib.FPK_ERR_TIMEOUT)


def test_bad_descriptors_rejected_before_any_device_work():
    lib = _lib.load()
    d = _lib.ChainDesc()
    d.size = 1  # wrong size
    ptrs = (ctypes.c_void_p * 1)(None)
    assert lib.fpk_chain_fwd(ctypes.byref(d), ptrs, 1, None, None) == _lib.FPK_ERR_INVALID
    a = _lib.AttnDesc()
    a.size = ctypes.sizeof(_lib.AttnDesc)
    a.version = 99
    assert lib.fpk_attention_fwd(ctypes.byref(a), None, None, None, None, None) == _lib.FPK_ERR_INVALID


def test_attn_desc_init_fills_contiguous_strides():
    lib = _lib.load()
    d = _lib.AttnDesc()
    assert lib.fpk_attn_desc_init(ctypes.byref(d), _lib.FPK_F16, 2, 3, 100, 64, 0.125) == 0
    assert d.size == ctypes.sizeof(_lib.AttnDesc) and d.version == 1
    assert list(d.q_strides) == [3 * 100 * 64, 100 * 64, 64]


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_ctypes_layout_matches_c(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(f"""
#include <stdio.h>
#include <stddef.h>
#include "{HEADER}"
int main(void) {{
  printf("%zu %zu %zu %zu %zu %zu %zu\\n", sizeof(fpk_attn_desc), offsetof(fpk_attn_desc, q_strides),
         offsetof(fpk_attn_desc, o_strides), sizeof(fpk_chain_desc), offsetof(fpk_chain_desc, in_dtype),
         offsetof(fpk_chain_desc, ops), sizeof(fpk_chain_op));
  return 0;
}}
""")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    got = list(map(int, subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()))
    want = [ctypes.sizeof(_lib.AttnDesc), _lib.AttnDesc.q_strides.offset, _lib.AttnDesc.o_strides.offset,
            ctypes.sizeof(_lib.ChainDesc), _lib.ChainDesc.in_dtype.offset, _lib.ChainDesc.ops.offset,
            ctypes.sizeof(_lib.ChainOp)]
    assert got == want


def test_torch_extension_loads_and_refuses_cpu_tensors():
    """fusionpass_b200._fpkern (the binding the plan runtime launches through) is
    built in-tree, links this libfpkern.so and raises for CPU tensors."""
    import torch

    from fusionpass_b200 import fpkern

    ext = fpkern.extension()
    assert ext.version() == _lib.FPK_ABI_VERSION
    assert Path(ext.__file__).parent == Path(_lib.library_path()).parent
    desc = {"ops": [{"op": "relu", "a": 0}], "result": 1}
    with pytest.raises(RuntimeError, match="CUDA"):
        ext.chain([torch.randn(4, 4)], torch.empty(4, 4), desc)
    with pytest.raises(RuntimeError, match="CUDA"):
        q = torch.randn(1, 1, 8, 16)
        ext.attention(q, q, q, torch.empty_like(q), {"scale": 0.25})
