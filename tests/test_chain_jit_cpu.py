"""Run-time specialised flat chains: the generated CUDA compiles (NVRTC, sm_100a)
for random programs and the eligibility rules hold.  No GPU is needed to compile."""

import numpy as np
import pytest
import torch

from fusionpass_b200 import _lib, fpkern, kernels

OPS = ["add", "mul", "scale", "relu", "exp", "gelu"]
DT = [torch.float16, torch.float32]


def random_chain(rng, n_in):
    names = [f"a{i}" for i in range(n_in)]
    body = []
    for k in range(int(rng.integers(1, 9))):
        op = OPS[int(rng.integers(len(OPS)))]
        if op in ("add", "mul"):
            body.append({"op": op, "operands": [names[int(rng.integers(len(names)))],
                                                names[int(rng.integers(len(names)))]]})
        elif op == "scale":
            body.append({"op": op, "operands": [names[int(rng.integers(len(names)))]],
                         "factor": float(rng.uniform(-3, 3))})
        else:
            body.append({"op": op, "operands": [names[int(rng.integers(len(names)))]]})
        names.append(f"t{k}")
    return body


def _has_nvrtc():
    body = [{"op": "relu", "operands": ["a0"]}]
    d = kernels.chain_descriptor(1, body)
    return fpkern.precompile_chain(d, 8, [torch.float16], ["full"], torch.float16)


@pytest.fixture(scope="module")
def nvrtc_ok():
    try:
        _lib.load()
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"libfpkern.so not built: {e}")
    if not _has_nvrtc():
        pytest.skip("no run-time compiler (libnvrtc.so.12) in this process")


def test_random_programs_compile(nvrtc_ok):
    rng = np.random.default_rng(7)
    for _ in range(12):
        n_in = int(rng.integers(1, 5))
        body = random_chain(rng, n_in)
        bc = ["full"] + [["full", "col", "row", "scalar"][int(rng.integers(4))] for _ in range(n_in - 1)]
        d = kernels.chain_descriptor(n_in, body, input_bcast=bc)
        dts = [DT[int(rng.integers(2))] for _ in range(n_in)]
        assert fpkern.precompile_chain(d, 8 * int(rng.integers(1, 600)), dts, bc, DT[int(rng.integers(2))])


def test_not_taken_cases(nvrtc_ok):
    body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "relu", "operands": ["t0"]}]
    d = kernels.chain_descriptor(2, body, input_bcast=["full", "col"])
    args = ([torch.float16, torch.float16], ["full", "col"], torch.float16)
    assert fpkern.precompile_chain(d, 64, *args)
    assert not fpkern.precompile_chain(d, 60, *args)  # cols % 8 != 0
    assert not fpkern.precompile_chain(d, 64, *args, flags=_lib.FPK_FLAG_NO_JIT)
    assert not fpkern.precompile_chain(d, 64, *args, flags=_lib.FPK_FLAG_TEST_TIMEOUT)
    rows = kernels.chain_descriptor(1, [{"op": "softmax", "operands": ["a0"]}])
    assert fpkern.precompile_chain(rows, 64, [torch.float16], ["full"], torch.float16)
    assert fpkern.precompile_chain(rows, 16384, [torch.float16], ["full"], torch.float16)
    assert not fpkern.precompile_chain(rows, 16392, [torch.float16], ["full"], torch.float16)  # > 16384 columns
    assert not fpkern.precompile_chain(rows, 100, [torch.float16], ["full"], torch.float16)  # cols % 8 != 0


def random_rows_chain(rng, n_in):
    """pre-softmax ops, one softmax, post-softmax ops (which may read any earlier value)."""
    names = [f"a{i}" for i in range(n_in)]
    body = []

    def pick():
        return names[int(rng.integers(len(names)))]

    def elementwise(k):
        op = ["add", "mul", "scale", "relu", "exp", "gelu"][int(rng.integers(6))]
        if op in ("add", "mul"):
            return {"op": op, "operands": [pick(), pick()]}
        if op == "scale":
            return {"op": op, "operands": [pick()], "factor": float(rng.uniform(-1.5, 1.5))}
        return {"op": op, "operands": [pick()]}

    k = 0
    for _ in range(int(rng.integers(0, 3))):
        body.append(elementwise(k))
        names.append(f"t{k}")
        k += 1
    body.append({"op": "softmax", "operands": [pick()]})
    names.append(f"t{k}")
    k += 1
    for _ in range(int(rng.integers(0, 3))):
        body.append(elementwise(k))
        names.append(f"t{k}")
        k += 1
    return body


def test_random_rows_programs_compile(nvrtc_ok):
    rng = np.random.default_rng(11)
    for cols in (8, 40, 128, 1000, 1024, 2048, 4096, 8192, 16384):
        n_in = int(rng.integers(1, 4))
        body = random_rows_chain(rng, n_in)
        bc = ["full"] + [["full", "col", "row", "scalar"][int(rng.integers(4))] for _ in range(n_in - 1)]
        d = kernels.chain_descriptor(n_in, body, input_bcast=bc)
        dts = [DT[int(rng.integers(2))] for _ in range(n_in)]
        assert fpkern.precompile_chain(d, cols, dts, bc, DT[int(rng.integers(2))])


def test_invalid_descriptor_is_rejected(nvrtc_ok):
    d = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    bad = {**d, "result": 7}  # slot that does not exist
    with pytest.raises(_lib.FpkernError):
        fpkern.precompile_chain(bad, 8, [torch.float16], ["full"], torch.float16)
