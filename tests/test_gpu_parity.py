"""GPU parity: libfpkern kernels vs the reference's own outputs and the oracle.

Tolerances against the reference's own kernel outputs (the parity contract):
  f32: |err| <= 1e-5 + 1e-5*|ref|       f16: |err| <= 2e-3 + 1e-2*|ref|
Chains made only of add/mul/scale/relu are compared bit for bit (the oracle and
the kernel both do f32 round-to-nearest ops in program order with one final
rounding).
"""

import numpy as np
import pytest
import torch

import oracle
from fusionpass_b200 import _lib, fpkern, kernels
from fusionpass_b200.runtime import execute_plan
from tests import _golden

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """Every kernel of every test must leave the device status word clean."""
    yield
    if "timeout" not in request.node.name:
        assert fpkern.poll_status() == 0, "a kernel recorded a device-side error"

TOL = {"f32": (1e-5, 1e-5), "f16": (2e-3, 1e-2)}
_DT = {"f32": torch.float32, "f16": torch.float16}


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _close(out, ref, dtype, what=""):
    atol, rtol = TOL[dtype]
    o = out.detach().float().cpu().numpy() if torch.is_tensor(out) else out.astype(np.float32)
    r = ref.astype(np.float32)
    err = np.abs(o - r)
    bad = err > atol + rtol * np.abs(r)
    assert not bad.any(), f"{what}: {bad.sum()} / {bad.size} beyond tol, max err {err.max():.3e}"


@pytest.mark.parametrize("name", _golden.names("attn"))
def test_attention_matches_reference_fixture(name):
    meta, a = _golden.load(name)
    q, k, v = (_cuda(a[x]) for x in "qkv")
    out = fpkern.attention(q, k, v, meta["scale"])
    torch.cuda.synchronize()
    assert fpkern.poll_status() == 0
    _close(out, a["out"], meta["dtype"], name)


@pytest.mark.parametrize("name", _golden.names("chain"))
def test_chain_matches_reference_fixture(name):
    meta, a = _golden.load(name)
    n = meta["n_args"]
    desc = kernels.chain_descriptor(n, meta["body"], rows=meta["launch"] == "rows")
    shape = meta["shape"]
    plan = {"version": 1,
            "inputs": [{"name": f"arg{i}", "shape": shape, "dtype": meta["dtype"]} for i in range(n)],
            "steps": [{"kind": "triton", "kernel": "fp_chain_0", "launch": meta["launch"],
                       "operands": [f"arg{i}" for i in range(n)], "result": "v0", "shape": shape,
                       "dtype": meta["dtype"],
                       "attrs": {**kernels.chain_launch_attrs(shape, rows=meta["launch"] == "rows"),
                                 "desc": desc}}],
            "outputs": ["v0"]}
    out = execute_plan(plan, [_cuda(a[f"x{i}"]) for i in range(n)])
    torch.cuda.synchronize()
    ops = {o["op"] for o in meta["body"]}
    if ops <= {"add", "mul", "scale", "relu"}:
        np.testing.assert_array_equal(out.cpu().numpy(), a["out"])
    else:
        _close(out, a["out"], meta["dtype"], name)


def test_cfg2_broadcast_operands_bit_exact():
    meta, a = _golden.load("chain_flat_f16_cfg2_64x256")
    desc = kernels.chain_descriptor(3, meta["body"], input_bcast=["full", "col", "col"])
    out = fpkern.chain([_cuda(a["x0"]), _cuda(a["x1_small"]), _cuda(a["x2_small"])], desc,
                       meta["shape"], torch.float16)
    np.testing.assert_array_equal(out.cpu().numpy(), a["out"])


CFG2_BODY = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "mul", "operands": ["t0", "a2"]},
             {"op": "relu", "operands": ["t1"]}, {"op": "scale", "operands": ["t2"], "factor": 0.5},
             {"op": "add", "operands": ["t3", "a0"]}]


def _cfg2_inputs(R, C, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(R, C, generator=g).half()
    b = (torch.randn(C, generator=g) * 0.1).half()
    s = (torch.rand(C, generator=g) + 0.5).half()
    return x, b, s


@pytest.mark.parametrize("R,C", [(4096, 4096), (1, 8), (3, 12), (257, 4100), (7, 3), (33, 8192), (19, 5000),
                                 (1000, 16), (5, 768), (64, 3072), (3, 8200)])
@pytest.mark.parametrize("path", ["jit", "tiled", "general"])
def test_cfg2_chain_vs_oracle_bit_exact(R, C, path):
    """All three flat-chain tiers: run-time compiled (cols % 8 == 0), the row-tiled
    interpreter and the general interpreter."""
    x, b, s = _cfg2_inputs(R, C)
    desc = kernels.chain_descriptor(3, CFG2_BODY, input_bcast=["full", "col", "col"])
    flags = {"jit": 0, "tiled": _lib.FPK_FLAG_NO_JIT, "general": _lib.FPK_FLAG_NO_STAGING}[path]
    out = fpkern.chain([x.cuda(), b.cuda(), s.cuda()], desc, [R, C], torch.float16, flags=flags)
    ops, res = oracle.body_to_program(3, CFG2_BODY)
    ref = oracle.chain_flat([x.numpy(), b.numpy(), s.numpy()], ops, res, (R, C), np.float16)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_chain_misaligned_and_row_broadcast_and_scalar():
    g = torch.Generator().manual_seed(3)
    R, C = 33, 130
    base = torch.randn(R * C + 1, generator=g)
    x = base[1:].view(R, C)            # 4-byte aligned only: element-load path
    rowv = torch.randn(R, 1, generator=g)
    sc = torch.randn(1, generator=g)
    body = [{"op": "mul", "operands": ["a0", "a1"]}, {"op": "add", "operands": ["t0", "a2"]},
            {"op": "exp", "operands": ["t1"]}]
    desc = kernels.chain_descriptor(3, body, input_bcast=["full", "row", "scalar"])
    xc = x.cuda()
    assert xc.data_ptr() % 16 == 0  # .cuda() copies into a fresh allocation
    xm = torch.empty(R * C + 1, device="cuda")[1:].view(R, C)
    xm.copy_(xc)
    out = fpkern.chain([xm, rowv.cuda(), sc.cuda()], desc, [R, C], torch.float32)
    ops, res = oracle.body_to_program(3, body)
    ref = oracle.chain_flat([x.numpy(), rowv.numpy(), sc.numpy()], ops, res, (R, C), np.float32)
    _close(out, ref, "f32", "misaligned/row/scalar")


@pytest.mark.parametrize("dt", [torch.float16, torch.float32])
@pytest.mark.parametrize("R,C", [(130, 96), (17, 4096), (9, 6000)])
def test_tiled_chain_operand_orders_and_dtypes(dt, R, C):
    """Column operands before full ones, a full operand used twice, f32 and f16:
    the row-tiled kernel reorders operands internally; results must not change."""
    g = torch.Generator().manual_seed(R + C)
    b = torch.randn(C, generator=g).to(dt)
    x = torch.randn(R, C, generator=g).to(dt)
    y = torch.randn(R, C, generator=g).to(dt)
    body = [{"op": "mul", "operands": ["a1", "a0"]}, {"op": "add", "operands": ["t0", "a2"]},
            {"op": "scale", "operands": ["t1"], "factor": -0.75}, {"op": "add", "operands": ["t2", "a1"]},
            {"op": "exp", "operands": ["t3"]}]
    desc = kernels.chain_descriptor(3, body, input_bcast=["col", "full", "full"])
    out = fpkern.chain([b.cuda(), x.cuda(), y.cuda()], desc, [R, C], dt)
    ops, res = oracle.body_to_program(3, body)
    ref = oracle.chain_flat([b.numpy(), x.numpy(), y.numpy()], ops, res, (R, C), x.numpy().dtype)
    _close(out, ref, "f32" if dt == torch.float32 else "f16", f"tiled {dt} {R}x{C}")


def test_chain_tree_needs_spill_registers():
    g = torch.Generator().manual_seed(5)
    ins = [torch.randn(64, 96, generator=g) for _ in range(4)]
    # ((a+b) * (c+d)) + (a*c): several values live at once
    body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "add", "operands": ["a2", "a3"]},
            {"op": "mul", "operands": ["t0", "t1"]}, {"op": "mul", "operands": ["a0", "a2"]},
            {"op": "add", "operands": ["t2", "t3"]}, {"op": "relu", "operands": ["t4"]}]
    desc = kernels.chain_descriptor(4, body)
    out = fpkern.chain([t.cuda() for t in ins], desc, [64, 96], torch.float32)
    ops, res = oracle.body_to_program(4, body)
    ref = oracle.chain_flat([t.numpy() for t in ins], ops, res, (64, 96), np.float32)
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("cols", [1, 5, 100, 128, 129, 1000, 1024, 1025, 4096, 8192, 16384])
def test_rows_softmax_chain_vs_oracle(cols):
    g = torch.Generator().manual_seed(cols)
    R = 37
    x = torch.randn(R, cols, generator=g) * 3
    y = torch.randn(R, cols, generator=g)
    body = [{"op": "scale", "operands": ["a0"], "factor": 0.5}, {"op": "softmax", "operands": ["t0"]},
            {"op": "mul", "operands": ["t1", "a1"]}, {"op": "relu", "operands": ["t2"]}]
    desc = kernels.chain_descriptor(2, body)
    for dt, tol in ((torch.float32, "f32"), (torch.float16, "f16")):
        xs, ys = x.to(dt), y.to(dt)
        out = fpkern.chain([xs.cuda(), ys.cuda()], desc, [R, cols], dt)
        ops, res = oracle.body_to_program(2, body)
        ref = oracle.chain_rows([xs.numpy(), ys.numpy()], ops, res, (R, cols), xs.numpy().dtype)
        _close(out, ref, tol, f"rows cols={cols} {dt}")


def test_gelu_extension_vs_eager():
    g = torch.Generator().manual_seed(9)
    x = torch.randn(512, 3072, generator=g).half().cuda()
    bias = (torch.randn(3072, generator=g) * 0.02).half().cuda()
    desc = kernels.chain_descriptor(2, [{"op": "add", "operands": ["a0", "a1"]},
                                        {"op": "gelu", "operands": ["t0"]}], input_bcast=["full", "col"])
    out = fpkern.chain([x, bias], desc, [512, 3072], torch.float16)
    ref = torch.nn.functional.gelu(x.float() + bias.float()).half()
    _close(out, ref.cpu().numpy(), "f16", "bias+gelu")


def _attn_torch_f32(q, k, v, scale):
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    return torch.matmul(torch.softmax(s, dim=-1), v.float())


@pytest.mark.parametrize("shape", [(1, 1, 1, 64), (2, 3, 300, 64), (1, 2, 513, 128), (1, 4, 255, 32),
                                   (2, 2, 129, 16), (1, 1, 2048, 128), (3, 1, 384, 64)])
def test_attention_f16_vs_torch_f32(shape):
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator().manual_seed(sum(shape))
    q, k, v = (torch.randn(shape, generator=g).half().cuda() for _ in range(3))
    scale = shape[-1] ** -0.5
    out = fpkern.attention(q, k, v, scale)
    ref = _attn_torch_f32(q, k, v, scale)
    assert fpkern.poll_status() == 0
    _close(out, ref.cpu().numpy(), "f16", f"attention {shape}")


# more (b*h, 256-row block) items than SMs, so every CTA of the persistent f16 kernel walks
# several and issues the next item's first Q K^T during the current one: items alternating
# between two tiles and one ((16, 16, 300, 64), (8, 16, 384, 32)), single-tile items of one
# key tile ((64, 16, 100, 64)), a second tile of one row ((40, 8, 129, 64)), D = 16
@pytest.mark.parametrize("shape", [(16, 16, 300, 64), (8, 16, 384, 32), (64, 16, 100, 64), (40, 8, 129, 64),
                                   (20, 16, 200, 16)])
def test_attention_f16_items_per_cta_vs_torch_f32(shape):
    g = torch.Generator().manual_seed(sum(shape) + 7)
    q, k, v = (torch.randn(shape, generator=g).half().cuda() for _ in range(3))
    scale = shape[-1] ** -0.5
    out = fpkern.attention(q, k, v, scale)
    _close(out, _attn_torch_f32(q, k, v, scale).cpu().numpy(), "f16", f"attention {shape}")


def test_attention_waits_for_the_kernel_that_wrote_its_inputs():
    """The persistent f16 kernel is a programmatic dependent launch: a torch kernel that
    rewrites Q in place right before it (and one that reads O right after) must be ordered
    with it.  Five rounds with different Q, each checked against torch f32."""
    B, H, S, D = 4, 16, 1024, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").half() for _ in range(2))
    qs = [torch.randn(B, H, S, D, generator=g, device="cuda").half() for _ in range(5)]
    q = torch.empty_like(qs[0])
    outs = []
    for qi in qs:
        q.copy_(qi)
        o = fpkern.attention(q, k, v, 0.125)
        outs.append(o.float() * 1.0)  # a plain kernel reading O right after
    for qi, o in zip(qs, outs):
        _close(o, _attn_torch_f32(qi, k, v, 0.125).cpu().numpy(), "f16", "attention after a producer")


def _split_batch(H, S, n_sms):
    """Smallest batch whose (b*h, 256-row block) items leave a last round of at most half
    the SMs: the persistent f16 kernel then runs that round's blocks as single 128-row
    tiles (only when every block holds two tiles: S % 256 == 0 or > 128)."""
    m = (S + 255) // 256
    for B in range(1, 64):
        blocks = B * H * m
        r = blocks % n_sms
        if blocks > n_sms and 0 < r and 2 * r <= n_sms:
            return B, r
    raise AssertionError("no batch size splits the last round")


@pytest.mark.parametrize("H,S,D", [(12, 512, 64), (16, 400, 64), (16, 512, 16), (32, 1024, 32)])
def test_attention_last_round_split_vs_torch_and_oracle(H, S, D):
    """Shapes whose last round of work items runs as single-tile items: every row against
    torch f32, and the last (b, h) slice (all of its blocks in the split round) and the
    first against the oracle."""
    n_sms = torch.cuda.get_device_properties(0).multi_processor_count
    B, r = _split_batch(H, S, n_sms)
    g = torch.Generator().manual_seed(H + S + D)
    q, k, v = ((torch.randn(B, H, S, D, generator=g) * D ** -0.25).half() for _ in range(3))
    scale = D ** -0.5
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = fpkern.attention(qc, kc, vc, scale)
    _close(out, _attn_torch_f32(qc, kc, vc, scale).cpu().numpy(), "f16", f"split B{B} H{H} S{S} D{D} ({r} blocks)")
    o = out.cpu().numpy().reshape(B * H, S, D)
    qs, ks, vs = (t.numpy().reshape(B * H, S, D) for t in (q, k, v))
    for bh in (0, B * H - 1):
        ref = oracle.attention_fwd(qs[bh:bh + 1], ks[bh:bh + 1], vs[bh:bh + 1], scale)
        _close(o[bh:bh + 1], ref, "f16", f"split slice {bh}")


@pytest.mark.parametrize("scale", [-0.3, 0.0, 2.0])
def test_attention_f16_unusual_scales(scale):
    g = torch.Generator().manual_seed(11)
    q, k, v = (torch.randn(1, 2, 200, 64, generator=g).half().cuda() for _ in range(3))
    out = fpkern.attention(q, k, v, scale)
    ref = _attn_torch_f32(q, k, v, scale)
    _close(out, ref.cpu().numpy(), "f16", f"scale {scale}")


# small grids run 16-row query tiles with their key tiles split over 4 thread groups per CTA
# ((1, 2, 300, 64), (1, 2, 512, 16)), 2 groups ((2, 1, 77, 128), (1, 3, 65, 16): the second group
# holds one key, (1, 4, 128, 64), (1, 1, 1000, 128)) or one ((1, 1, 1, 32)); (4, 8, 320, 32) has
# >= 148 64-row tiles and runs 64-row ones
@pytest.mark.parametrize("shape", [(1, 2, 300, 64), (2, 1, 77, 128), (1, 3, 65, 16), (1, 1, 1, 32),
                                   (1, 4, 128, 64), (4, 8, 320, 32), (1, 2, 512, 16), (1, 1, 1000, 128)])
def test_attention_f32_vs_oracle(shape):
    g = torch.Generator().manual_seed(sum(shape) + 1)
    q, k, v = (torch.randn(shape, generator=g) for _ in range(3))
    scale = shape[-1] ** -0.5
    out = fpkern.attention(q.cuda(), k.cuda(), v.cuda(), scale)
    ref = oracle.attention_fwd(q.numpy(), k.numpy(), v.numpy(), scale)
    _close(out, ref, "f32", f"f32 attention {shape}")


def test_attention_f32_scalar_load_path_vs_oracle():
    """K and V 4-byte but not 16-byte aligned (views one element into their buffers): the
    kernel falls back from 16-byte to scalar tile loads; same results."""
    shape = (1, 3, 200, 64)
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(shape, generator=g) for _ in range(3))
    bufs = [torch.empty(k.numel() + 1, device="cuda") for _ in range(2)]
    kd, vd = (b[1:].view(shape) for b in bufs)
    kd.copy_(k)
    vd.copy_(v)
    assert kd.data_ptr() % 16 and vd.data_ptr() % 16
    out = fpkern.attention(q.cuda(), kd, vd, 0.125)
    _close(out, oracle.attention_fwd(q.numpy(), k.numpy(), v.numpy(), 0.125), "f32", "f32 attention, scalar loads")


def test_attention_prefill_config_slices_vs_oracle():
    """B8 H16 S2048 D64 f16 (Q/K/V ~ N(0,1) * D^-1/4, scale 1/8): whole-tensor check
    against a torch f32 reference plus three B*H slices against the oracle."""
    B, H, S, D = 8, 16, 2048, 64
    g = torch.Generator().manual_seed(0)
    q, k, v = ((torch.randn(B, H, S, D, generator=g) * D ** -0.25).half() for _ in range(3))
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = fpkern.attention(qc, kc, vc, 0.125)
    _close(out, _attn_torch_f32(qc, kc, vc, 0.125).cpu().numpy(), "f16", "cfg3 full")
    o = out.cpu().numpy().reshape(B * H, S, D)
    for bh in (0, 63, 127):
        ref = oracle.attention_fwd(q.numpy().reshape(B * H, S, D)[bh:bh + 1], k.numpy().reshape(B * H, S, D)[bh:bh + 1],
                                   v.numpy().reshape(B * H, S, D)[bh:bh + 1], 0.125)
        _close(o[bh:bh + 1], ref, "f16", f"cfg3 slice {bh}")


def _budget(out, ref, dtype="f16"):
    atol, rtol = TOL[dtype]
    o = out.detach().float().cpu().numpy() if torch.is_tensor(out) else out.astype(np.float32)
    r = ref.astype(np.float32)
    return float((np.abs(o - r) / (atol + rtol * np.abs(r))).max())


def test_attention_long_config_slices_vs_oracle(capsys):
    """B4 H32 S8192 D128 f16 (Q/K/V ~ N(0,1) from the device generator, seed 0, scale
    1/sqrt(128)), the long-sequence workload at full size: every (b,h) slice against a
    torch f32 reference and three slices (first, middle, last) against the oracle,
    which walks the reference's 64 x 64 tiles.  Prints the worst fraction of the
    atol 2e-3 / rtol 1e-2 budget."""
    B, H, S, D = 4, 32, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").half() for _ in range(3))
    sc = D ** -0.5
    out = fpkern.attention(q, k, v, sc)
    torch.cuda.synchronize()
    assert fpkern.poll_status() == 0
    worst_torch = 0.0
    q3, k3, v3, o3 = (t.reshape(B * H, S, D) for t in (q, k, v, out))
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for i in range(0, B * H, 2):
            ref = _attn_torch_f32(q3[i:i + 2], k3[i:i + 2], v3[i:i + 2], sc)
            worst_torch = max(worst_torch, _budget(o3[i:i + 2], ref.cpu().numpy()))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    worst_oracle = 0.0
    for bh in (0, 63, 127):
        qs, ks, vs = (t[bh:bh + 1].cpu().numpy() for t in (q3, k3, v3))
        ref = oracle.attention_fwd(qs, ks, vs, sc)
        worst_oracle = max(worst_oracle, _budget(o3[bh:bh + 1], ref))
    with capsys.disabled():
        print(f"\n[cfg4 B4 H32 S8192 D128] worst fraction of the f16 budget: torch f32 {worst_torch:.3f}, "
              f"oracle slices 0/63/127 {worst_oracle:.3f}")
    assert worst_torch <= 1.0 and worst_oracle <= 1.0


def test_strided_attention_bshd_layout():
    """q/k/v as [B, S, H, D] memory viewed as [B, H, S, D]: no copy, strided TMA maps."""
    g = torch.Generator().manual_seed(21)
    B, S, H, D = 2, 300, 3, 64
    q, k, v = (torch.randn(B, S, H, D, generator=g).half().cuda().transpose(1, 2) for _ in range(3))
    out = torch.empty(B, S, H, D, dtype=torch.float16, device="cuda").transpose(1, 2)
    fpkern.attention(q, k, v, 0.125, out=out)
    ref = _attn_torch_f32(q, k, v, 0.125)
    _close(out, ref.cpu().numpy(), "f16", "strided")


def test_empty_inputs_launch_nothing():
    desc = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    out = fpkern.chain([torch.empty(0, 16, device="cuda")], desc, [0, 16], torch.float32)
    assert out.shape == (0, 16)


def test_bounded_wait_timeout_is_reported_not_hung():
    """The test flag withholds one producer signal; the bounded wait runs out after
    ~5 ms, the kernel records FPK_ERR_TIMEOUT and returns, and the context stays usable."""
    x = torch.randn(1 << 20, device="cuda")
    desc = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    assert fpkern.poll_status() == 0
    fpkern.chain([x], desc, [1024, 1024], torch.float32, flags=_lib.FPK_FLAG_TEST_TIMEOUT)
    assert fpkern.poll_status() == _lib.FPK_ERR_TIMEOUT
    q = torch.randn(1, 1, 256, 64, device="cuda").half()
    fpkern.attention(q, q, q, 0.125, flags=_lib.FPK_FLAG_TEST_TIMEOUT)
    assert fpkern.poll_status() == _lib.FPK_ERR_TIMEOUT
    y = fpkern.chain([x], desc, [1024, 1024], torch.float32)  # context still healthy
    assert fpkern.poll_status() == 0
    assert torch.equal(y.view(-1), torch.relu(x))


def test_fused_step_on_cpu_raises():
    desc = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    with pytest.raises(RuntimeError, match="CUDA"):
        fpkern.chain([torch.randn(4, 4)], desc, [4, 4], torch.float32)
