"""GPU: LayerNorm over the last axis in libfpkern.so (the `layer_norm` torch steps of
extension plans) against torch's layer_norm computed in f32: within the f16 budget
(atol 2e-3, rtol 1e-2) for f16 and within 1e-5 / 1e-5 for f32; shapes the kernel does
not take come back as None; the plan runtime runs the kernel."""

import ctypes

import pytest
import torch

from fusionpass_b200 import _lib, fpkern, runtime

pytestmark = pytest.mark.gpu


def _ref(x, w, b, eps):
    return torch.nn.functional.layer_norm(x.float(), (x.shape[-1],), None if w is None else w.float(),
                                          None if b is None else b.float(), eps)


# (shape, dtype, affine): the BERT block's rows; 97 and 96 vectors per row; one vector; the
# widest row (2048); several leading dims; no affine parameters
CASES = [((16384, 768), torch.float16, True), ((5, 776), torch.float16, True), ((3, 8), torch.float32, True),
         ((4, 2048), torch.float16, True), ((2, 3, 64), torch.float32, False), ((33, 1000), torch.float32, True),
         ((7, 512), torch.float16, False)]


@pytest.mark.parametrize("shape,dt,affine", CASES)
def test_layer_norm_matches_torch_f32(shape, dt, affine):
    g = torch.Generator(device="cuda").manual_seed(sum(shape))
    x = (torch.randn(shape, generator=g, device="cuda") * 3 + 1).to(dt)
    w = (torch.randn(shape[-1], generator=g, device="cuda") * 0.5 + 1).to(dt) if affine else None
    b = (torch.randn(shape[-1], generator=g, device="cuda") * 0.1).to(dt) if affine else None
    y = fpkern.layer_norm(x, w, b, 1e-5)
    assert y is not None and y.shape == x.shape and y.dtype == dt
    ref = _ref(x, w, b, 1e-5)
    atol, rtol = (2e-3, 1e-2) if dt == torch.float16 else (1e-5, 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=atol, rtol=rtol)
    assert fpkern.poll_status() == 0


def test_shapes_the_kernel_does_not_take():
    x = torch.randn(4, 20, device="cuda").half()  # 20 % 8 != 0
    assert fpkern.layer_norm(x, None, None, 1e-5) is None
    x = torch.randn(2, 2056, device="cuda").half()  # above 2048 columns
    assert fpkern.layer_norm(x, None, None, 1e-5) is None
    x = torch.randn(2, 64, device="cuda").half()
    assert fpkern.layer_norm(x, torch.ones(64, device="cuda"), torch.zeros(64, device="cuda"), 1e-5) is None  # f32 params


def test_constant_rows_and_large_offsets():
    """A constant row has zero variance: y = b exactly (0 * rstd * w + b); rows far from
    zero keep their spread (two-pass variance, no E[x^2] - mean^2 cancellation)."""
    x = torch.full((3, 256), 7.0, device="cuda")
    w, b = torch.full((256,), 2.0, device="cuda"), torch.full((256,), 0.25, device="cuda")
    y = fpkern.layer_norm(x, w, b, 1e-5)
    assert torch.equal(y, torch.full_like(x, 0.25))
    g = torch.Generator(device="cuda").manual_seed(1)
    x = 1e4 + torch.randn(64, 512, generator=g, device="cuda")
    torch.testing.assert_close(fpkern.layer_norm(x, None, None, 1e-5), _ref(x, None, None, 1e-5), atol=5e-3, rtol=1e-3)


def test_plan_runtime_runs_the_kernel(monkeypatch):
    calls = []
    real = fpkern.layer_norm

    def spy(*a, **k):
        y = real(*a, **k)
        calls.append(y is not None)
        return y

    monkeypatch.setattr(fpkern, "layer_norm", spy)
    x = torch.randn(8, 768, device="cuda").half()
    w, b = torch.randn(768, device="cuda").half(), torch.randn(768, device="cuda").half()
    y = runtime._run_torch({"op": "layer_norm", "attrs": {"normalized_shape": [768], "eps": 1e-12}}, [x, w, b])
    assert calls == [True]
    torch.testing.assert_close(y.float(), _ref(x, w, b, 1e-12), atol=2e-3, rtol=1e-2)


def test_c_abi_rejects_malformed_descriptors():
    lib = _lib.load()
    x = torch.randn(4, 64, device="cuda")
    d = _lib.LnDesc(size=ctypes.sizeof(_lib.LnDesc), version=_lib.FPK_ABI_VERSION, dtype=_lib.FPK_F32, rows=4,
                    cols=64, eps=1e-5)
    ptr = ctypes.c_void_p(x.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.fpk_layer_norm_fwd(ctypes.byref(d), ptr, ptr, None, ptr, stream) == _lib.FPK_ERR_INVALID  # w without b
    d.eps = -1.0
    assert lib.fpk_layer_norm_fwd(ctypes.byref(d), ptr, None, None, ptr, stream) == _lib.FPK_ERR_INVALID
    d.eps, d.cols, d.rows = 1e-5, 60, 4
    assert lib.fpk_layer_norm_fwd(ctypes.byref(d), ptr, None, None, ptr, stream) == _lib.FPK_ERR_UNSUPPORTED


@pytest.mark.parametrize("shape,dt,kinds", [((16384, 768), torch.float16, ("full", "col", "full")),
                                            ((9, 1000), torch.float32, ("full", "full")),
                                            ((5, 2, 64), torch.float16, ("col", "full", "full", "col")),
                                            ((3, 8), torch.float32, ("full",))])
def test_add_layer_norm_matches_torch_f32(shape, dt, kinds):
    """LayerNorm of the in-order sum of full-shape and per-column addends."""
    g = torch.Generator(device="cuda").manual_seed(len(kinds) + shape[-1])
    adds = [(torch.randn(shape if k == "full" else shape[-1:], generator=g, device="cuda")).to(dt) for k in kinds]
    w = (torch.randn(shape[-1], generator=g, device="cuda") * 0.5 + 1).to(dt)
    b = (torch.randn(shape[-1], generator=g, device="cuda") * 0.1).to(dt)
    y = fpkern.add_layer_norm(adds, w, b, 1e-5)
    assert y is not None and tuple(y.shape) == tuple(shape)
    s = adds[0].float()
    for t in adds[1:]:
        s = s + t.float()
    ref = _ref(s, w, b, 1e-5)
    atol, rtol = (2e-3, 1e-2) if dt == torch.float16 else (1e-5, 1e-5)
    torch.testing.assert_close(y.float(), ref, atol=atol, rtol=rtol)
    assert fpkern.poll_status() == 0


def test_add_layer_norm_plan_step_runs_the_kernel(monkeypatch):
    calls = []
    real = fpkern.add_layer_norm

    def spy(*a, **k):
        y = real(*a, **k)
        calls.append(y is not None)
        return y

    monkeypatch.setattr(fpkern, "add_layer_norm", spy)
    a, c = torch.randn(8, 768, device="cuda").half(), torch.randn(8, 768, device="cuda").half()
    bias, w, b = (torch.randn(768, device="cuda").half() for _ in range(3))
    step = {"op": "add_layer_norm", "attrs": {"normalized_shape": [768], "eps": 1e-12, "n_addends": 3}}
    y = runtime._run_torch(step, [a, bias, c, w, b])
    assert calls == [True]
    torch.testing.assert_close(y.float(), _ref(a.float() + bias.float() + c.float(), w, b, 1e-12), atol=2e-3, rtol=1e-2)


def test_add_layer_norm_single_row_takes_the_step_shape():
    """A [1, 1, cols] result whose first addend is a per-column vector keeps the step's shape."""
    g = torch.Generator(device="cuda").manual_seed(2)
    bias, x = torch.randn(64, generator=g, device="cuda").half(), torch.randn(1, 1, 64, generator=g, device="cuda").half()
    step = {"op": "add_layer_norm", "shape": [1, 1, 64], "attrs": {"normalized_shape": [64], "eps": 1e-5, "n_addends": 2}}
    y = runtime._run_torch(step, [bias, x])
    assert tuple(y.shape) == (1, 1, 64)
    torch.testing.assert_close(y.float(), _ref(bias.float() + x.float(), None, None, 1e-5), atol=2e-3, rtol=1e-2)
