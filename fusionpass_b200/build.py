"""Build ``libfpkern.so`` in-tree with nvcc for sm_100a (B200).

    python -m fusionpass_b200.build          # incremental
    python -m fusionpass_b200.build --force  # rebuild everything

Objects go to ``fusionpass_b200/_build/``; the shared library is written next to
this file so that it travels with the source tree.  The CUDA runtime is linked
statically and the driver's tensor-map encoder is looked up at run time, so the
library needs nothing but the NVIDIA driver on the target machine.

The torch C++ extension ``fusionpass_b200._fpkern`` (``csrc/torch_ext.cpp``, the
binding the plan runtime launches through) is compiled with the host compiler
against the installed torch and linked to ``libfpkern.so`` (found next to it
through the run path ``$ORIGIN``), also in-tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libfpkern.so"
SOURCES = ["fpkern.cu", "chain.cu", "chain_jit.cu", "attention_f32.cu", "attention_tc.cu", "layer_norm.cu"]
HEADERS = ["common.cuh", "internal.h", "tmem_ops.cuh", "chain_ops.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
                     f"-I{ROOT / 'include'}", f"-I{BUILD}"]


def nvcc() -> str:
    exe = shutil.which("nvcc")
    if exe is None:
        cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
        if cand.exists():
            exe = str(cand)
    if exe is None:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return exe


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _compile(src: str, force: bool) -> tuple[str, int, str]:
    obj = BUILD / (Path(src).stem + ".o")
    deps = [CSRC / src] + [CSRC / h for h in HEADERS] + [ROOT / "include" / "fpkern.h"]
    if not force and not _stale(obj, deps):
        return src, 0, "up to date"
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
    p = subprocess.run(cmd, capture_output=True, text=True)
    (BUILD / (Path(src).stem + ".log")).write_text(p.stdout + p.stderr)
    return src, p.returncode, p.stderr[-4000:]


def _embed_ops_source() -> None:
    """Write chain_ops.cuh as a C++ raw-string literal for the run-time compiled
    chain kernels (chain_jit.cu), so they use the interpreter's op definitions."""
    text = (CSRC / "chain_ops.cuh").read_text(encoding="utf-8")
    if ')FPKOPS"' in text:
        raise RuntimeError("chain_ops.cuh contains the raw-string delimiter")
    inc = BUILD / "chain_ops_src.inc"
    body = 'R"FPKOPS(' + text + ')FPKOPS"\n'
    if not inc.exists() or inc.read_text(encoding="utf-8") != body:
        inc.write_text(body, encoding="utf-8")


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    _embed_ops_source()
    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), SOURCES))
    for src, rc, log in results:
        if rc != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{log}")
        if verbose:
            print(f"[fpkern] {src}: ok")
    objs = [BUILD / (Path(s).stem + ".o") for s in SOURCES]
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        print(f"[fpkern] {LIB}")
    return LIB


def extension_path() -> Path:
    return PKG / ("_fpkern" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/torch_ext.cpp into the importable module fusionpass_b200._fpkern."""
    import torch
    from torch.utils import cpp_extension as ce

    out = extension_path()
    src = CSRC / "torch_ext.cpp"
    deps = [src, ROOT / "include" / "fpkern.h", LIB]
    if not force and not _stale(out, deps):
        return out
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    cxx = os.environ.get("CXX", "g++")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-w",
           "-DTORCH_EXTENSION_NAME=_fpkern", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{sysconfig.get_paths()['include']}",
           f"-I{cuda_home / 'include'}", f"-I{ROOT / 'include'}",
           str(src), "-o", str(out.with_suffix(".tmp")),
           *[f"-L{p}" for p in ce.library_paths()], f"-L{PKG}",
           "-lfpkern", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           "-Wl,-rpath,$ORIGIN"]
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError(f"building the torch extension failed:\n{p.stderr[-4000:]}")
    os.replace(out.with_suffix(".tmp"), out)
    if verbose:
        print(f"[fpkern] {out}")
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    build(force=a.force, verbose=True)
    build_extension(force=a.force, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
