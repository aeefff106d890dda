"""GPU: run-time compiled flat chains are bit-identical to the interpreter kernels
and to the oracle, and they really run (launch counter)."""

import numpy as np
import pytest
import torch

import oracle
from fusionpass_b200 import _lib, fpkern, kernels
from tests.test_chain_jit_cpu import random_chain, random_rows_chain

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert fpkern.poll_status() == 0, "a kernel recorded a device-side error"


def _bits(t):
    """Bit pattern with every NaN mapped to one canonical value."""
    t = t.detach()
    if t.dtype == torch.float16:
        return torch.where(torch.isnan(t), torch.full_like(t, float("nan")), t).view(torch.int16).cpu()
    return torch.where(torch.isnan(t), torch.full_like(t, float("nan")), t).view(torch.int32).cpu()


def _operand(shape_kind, R, C, dt, g):
    n = {"full": (R, C), "col": (C,), "row": (R, 1), "scalar": (1,)}[shape_kind]
    return (torch.randn(n, generator=g) * 2).to(dt).cuda()


@pytest.mark.parametrize("seed", range(6))
# (R, C): one vector; short rows several per CTA (40, 64, 16 columns); 97 and 201 vectors per row
# (a CTA block of 97, two blocks of 101 with the last thread idle); a full-size row
@pytest.mark.parametrize("R,C", [(1, 8), (37, 40), (1000, 64), (4097, 16), (19, 776), (33, 1608), (2048, 4096)])
def test_random_programs_jit_equals_interpreter(seed, R, C):
    rng = np.random.default_rng(100 + seed)
    g = torch.Generator().manual_seed(seed)
    n_in = int(rng.integers(1, 5))
    body = random_chain(rng, n_in)
    bc = ["full"] + [["full", "col", "row", "scalar"][int(rng.integers(4))] for _ in range(n_in - 1)]
    dts = [[torch.float16, torch.float32][int(rng.integers(2))] for _ in range(n_in)]
    out_dt = [torch.float16, torch.float32][int(rng.integers(2))]
    desc = kernels.chain_descriptor(n_in, body, input_bcast=bc)
    ins = [_operand(k, R, C, dt, g) for k, dt in zip(bc, dts)]
    n0 = fpkern.chain_jit_launches()
    y_jit = fpkern.chain(ins, desc, [R, C], out_dt)
    assert fpkern.chain_jit_launches() == n0 + 1, "the run-time compiled kernel did not run"
    y_tiled = fpkern.chain(ins, desc, [R, C], out_dt, flags=_lib.FPK_FLAG_NO_JIT)
    y_gen = fpkern.chain(ins, desc, [R, C], out_dt, flags=_lib.FPK_FLAG_NO_STAGING)
    assert fpkern.chain_jit_launches() == n0 + 1
    assert torch.equal(_bits(y_jit), _bits(y_tiled))
    assert torch.equal(_bits(y_jit), _bits(y_gen))


def test_special_values_bit_exact_vs_oracle():
    """inf, -inf, NaN, -0.0, denormal f16 through relu / scale / add / mul."""
    vals = torch.tensor([float("inf"), float("-inf"), float("nan"), -0.0, 0.0, 6e-8, -6e-8, 65504.0, -65504.0,
                         1.0, -1.0, 3.5], dtype=torch.float16)
    R, C = 24, 64
    x = vals[torch.arange(R * C) % len(vals)].reshape(R, C)
    y = vals[(torch.arange(R * C) * 7 + 3) % len(vals)].reshape(R, C)
    body = [{"op": "relu", "operands": ["a0"]}, {"op": "scale", "operands": ["t0"], "factor": -1.5},
            {"op": "add", "operands": ["t1", "a1"]}, {"op": "mul", "operands": ["t2", "a0"]}]
    desc = kernels.chain_descriptor(2, body)
    n0 = fpkern.chain_jit_launches()
    out = fpkern.chain([x.cuda(), y.cuda()], desc, [R, C], torch.float32)
    assert fpkern.chain_jit_launches() == n0 + 1
    ops, res = oracle.body_to_program(2, body)
    ref = oracle.chain_flat([x.numpy(), y.numpy()], ops, res, (R, C), np.float32)
    o = out.cpu().numpy()
    assert np.array_equal(np.isnan(o), np.isnan(ref))
    np.testing.assert_array_equal(np.where(np.isnan(o), 0, o).view(np.int32), np.where(np.isnan(ref), 0, ref).view(np.int32))


def test_jit_inside_cuda_graph_after_warmup():
    R, C = 512, 1024
    g = torch.Generator().manual_seed(3)
    x = torch.randn(R, C, generator=g).half().cuda()
    b = torch.randn(C, generator=g).half().cuda()
    body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "gelu", "operands": ["t0"]}]
    desc = kernels.chain_descriptor(2, body, input_bcast=["full", "col"])
    out = torch.empty(R, C, dtype=torch.float16, device="cuda")
    fpkern.chain([x, b], desc, [R, C], torch.float16, out=out)  # compiles and loads
    ref = out.clone()
    out.zero_()
    torch.cuda.synchronize()
    n0 = fpkern.chain_jit_launches()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fpkern.chain([x, b], desc, [R, C], torch.float16, out=out)
    graph.replay()
    torch.cuda.synchronize()
    assert fpkern.chain_jit_launches() == n0 + 1
    assert torch.equal(out, ref)
    del graph


def test_first_use_under_capture_runs_the_interpreter():
    """A chain first seen while a stream is capturing is served by the prebuilt
    kernels (no module load inside a capture); the result is the same."""
    R, C = 64, 256
    g = torch.Generator().manual_seed(4)
    x = torch.randn(R, C, generator=g).half().cuda()
    body = [{"op": "scale", "operands": ["a0"], "factor": 0.731}, {"op": "exp", "operands": ["t0"]},
            {"op": "mul", "operands": ["t1", "a0"]}]
    desc = kernels.chain_descriptor(1, body)
    out = torch.empty(R, C, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fpkern.chain([x], desc, [R, C], torch.float32, out=out)
    graph.replay()
    torch.cuda.synchronize()
    ref = fpkern.chain([x], desc, [R, C], torch.float32, flags=_lib.FPK_FLAG_NO_JIT)
    assert torch.equal(_bits(out), _bits(ref))
    del graph


def _allclose(a, b, dt):
    a, b = a.float().cpu().numpy(), b.float().cpu().numpy()
    if dt == torch.float16:
        np.testing.assert_allclose(a, b, rtol=1e-2, atol=2e-3, equal_nan=True)
    else:
        np.testing.assert_allclose(a, b, rtol=2e-5, atol=1e-6, equal_nan=True)


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("R,C", [(1, 8), (37, 40), (300, 128), (64, 1000), (33, 1024), (17, 4096), (5, 16384)])
def test_random_rows_programs_jit_vs_interpreter(seed, R, C):
    """Rows mode: the compiled kernel reduces in another order than the interpreter, so the
    two agree within rounding (and both within tolerance of the oracle elsewhere)."""
    rng = np.random.default_rng(200 + seed)
    g = torch.Generator().manual_seed(seed)
    n_in = int(rng.integers(1, 4))
    body = random_rows_chain(rng, n_in)
    bc = ["full"] + [["full", "col", "row", "scalar"][int(rng.integers(4))] for _ in range(n_in - 1)]
    dts = [[torch.float16, torch.float32][int(rng.integers(2))] for _ in range(n_in)]
    out_dt = [torch.float16, torch.float32][int(rng.integers(2))]
    desc = kernels.chain_descriptor(n_in, body, input_bcast=bc)
    ins = [_operand(k, R, C, dt, g) for k, dt in zip(bc, dts)]
    n0 = fpkern.chain_jit_launches()
    y_jit = fpkern.chain(ins, desc, [R, C], out_dt)
    assert fpkern.chain_jit_launches() == n0 + 1, "the run-time compiled rows kernel did not run"
    y_int = fpkern.chain(ins, desc, [R, C], out_dt, flags=_lib.FPK_FLAG_NO_JIT)
    assert fpkern.chain_jit_launches() == n0 + 1
    _allclose(y_jit, y_int, out_dt)


@pytest.mark.parametrize("C", [8, 128, 1000, 4096, 16384])
def test_rows_softmax_jit_vs_oracle(C):
    R = 24
    g = torch.Generator().manual_seed(C)
    x = (torch.randn(R, C, generator=g) * 4).float()
    b = torch.randn(C, generator=g).float()
    body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "softmax", "operands": ["t0"]},
            {"op": "mul", "operands": ["t1", "a0"]}]
    desc = kernels.chain_descriptor(2, body, input_bcast=["full", "col"])
    n0 = fpkern.chain_jit_launches()
    out = fpkern.chain([x.cuda(), b.cuda()], desc, [R, C], torch.float32)
    assert fpkern.chain_jit_launches() == n0 + 1
    ops, res = oracle.body_to_program(2, body)
    ref = oracle.chain_rows([x.numpy(), np.broadcast_to(b.numpy(), (R, C))], ops, res, (R, C), np.float32)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


def test_rows_all_masked_like_values():
    """A row of -inf scores gives NaN like the reference (exp(-inf - -inf)); others are fine."""
    R, C = 4, 64
    x = torch.randn(R, C)
    x[1] = float("-inf")
    desc = kernels.chain_descriptor(1, [{"op": "softmax", "operands": ["a0"]}])
    out = fpkern.chain([x.cuda()], desc, [R, C], torch.float32).cpu()
    ref = fpkern.chain([x.cuda()], desc, [R, C], torch.float32, flags=_lib.FPK_FLAG_NO_JIT).cpu()
    assert torch.isnan(out[1]).all() and torch.isnan(ref[1]).all()
    torch.testing.assert_close(out[[0, 2, 3]], torch.softmax(x[[0, 2, 3]], -1), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("mode", ["flat", "rows"])
def test_max_size_chain_jit_vs_interpreter(mode):
    """8 operands (all broadcast modes, both dtypes) and 32 ops, the descriptor limits."""
    rng = np.random.default_rng(31)
    g = torch.Generator().manual_seed(31)
    R, C = 96, 1024
    n_in = _lib.FPK_CHAIN_MAX_INPUTS
    bc = ["full", "col", "row", "scalar", "full", "col", "full", "row"]
    dts = [torch.float16, torch.float32] * 4
    names = [f"a{i}" for i in range(n_in)]
    body = []
    n_ops = _lib.FPK_CHAIN_MAX_OPS
    for k in range(n_ops):
        if mode == "rows" and k == 20:
            body.append({"op": "softmax", "operands": [names[-1]]})
        elif k % 4 == 3:
            body.append({"op": "scale", "operands": [names[-1]], "factor": 0.5})
        else:
            op = ["add", "mul", "relu"][k % 3]
            a, b = names[-1], names[int(rng.integers(n_in))]
            body.append({"op": op, "operands": [a, b] if op != "relu" else [a]})
        names.append(f"t{k}")
    desc = kernels.chain_descriptor(n_in, body, input_bcast=bc)
    ins = [_operand(k, R, C, dt, g) * 0.5 for k, dt in zip(bc, dts)]
    n0 = fpkern.chain_jit_launches()
    y_jit = fpkern.chain(ins, desc, [R, C], torch.float32)
    assert fpkern.chain_jit_launches() == n0 + 1
    y_int = fpkern.chain(ins, desc, [R, C], torch.float32, flags=_lib.FPK_FLAG_NO_JIT)
    if mode == "flat":
        assert torch.equal(_bits(y_jit), _bits(y_int))
    else:
        _allclose(y_jit, y_int, torch.float32)
