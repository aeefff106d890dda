"""End to end on the GPU: compile_model(fuse=True) -> plan with descriptors ->
libfpkern, gated by verify_equivalence against eager PyTorch (reference
tests/test_fusion_e2e.py, test_edge_cases.py, test_verify_bench.py)."""

import copy

import pytest
import torch

from fusionpass_b200 import compile_model, fpkern
from fusionpass_b200.bench import UnverifiedSpeedupError, benchmark
from fusionpass_b200.verify import EquivalenceError, assert_equivalent, verify_equivalence
from tests.models import Attn, BertBlock, BroadcastChain, Chain, RowChain, SoftmaxChain, init_bert

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(autouse=True)
def _device_status_clean():
    yield
    assert fpkern.poll_status() == 0


def kinds(c):
    return [s.get("launch", s.get("op")) for s in c.plan["steps"]]


@pytest.mark.parametrize("S", [1, 7, 64, 65, 130])
def test_attention_sequence_lengths(S):
    xs = [torch.randn(1, 2, S, 16, device=DEV) for _ in range(3)]
    c = compile_model(Attn(), xs, fuse=True)
    assert kinds(c) == ["attention"] and c.verified


def test_fused_equals_eager_and_unfused():
    m = Chain().to(DEV).eval()
    x = torch.randn(8, 16, device=DEV)
    c = compile_model(m, (x,), fuse=True)
    assert kinds(c) == ["flat"]
    torch.testing.assert_close(c(x), m(x), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(compile_model(m, (x,), fuse=False)(x), c(x))


def test_softmax_and_row_chains():
    x = torch.randn(6, 100, device=DEV)
    c = compile_model(SoftmaxChain(), (x,), fuse=True)
    assert kinds(c) == ["rows"]
    torch.testing.assert_close(c(x), SoftmaxChain()(x), atol=1e-5, rtol=1e-5)
    xs = (torch.randn(64, 128, device=DEV), torch.randn(64, 128, device=DEV))
    assert compile_model(RowChain(), xs, fuse=True).verified


def test_large_magnitude_softmax_is_stable():
    class M(torch.nn.Module):
        def forward(self, x):
            return torch.softmax(x * 1.0, dim=-1) * 2.0

    x = torch.randn(4, 50, device=DEV) * 50
    c = compile_model(M(), (x,), fuse=True)
    torch.testing.assert_close(c(x), M()(x), atol=1e-4, rtol=1e-4)


def test_noncontiguous_input_handled():
    class M(torch.nn.Module):
        def forward(self, x):
            return torch.exp(torch.relu(x * 2.0) * 0.1)

    x = torch.randn(16, 8, device=DEV).t()
    c = compile_model(M(), (x.contiguous(),), fuse=True)
    torch.testing.assert_close(c(x), M()(x), atol=1e-5, rtol=1e-5)


def test_wrong_shape_at_call_time():
    class M(torch.nn.Module):
        def forward(self, x):
            return torch.relu(x * 2.0)

    c = compile_model(M(), (torch.randn(4, 4, device=DEV),), fuse=True)
    with pytest.raises(ValueError):
        c(torch.randn(4, 5, device=DEV))


def test_fp16_attention_and_chain():
    """Mirrors the reference's fp16 test.  The eager-f16 gate is not used for the
    attention here: eager f16 rounds the S x S scores to f16 before the softmax,
    and at the gate's x4 trial that alone moves the output by ~9e-2, beyond the
    1e-2 f16 tolerance, for any kernel that keeps the scores in f32 (the
    reference Triton kernel does too).  The fused output is checked against an
    f32 computation instead."""
    xs = [torch.randn(2, 4, 100, 64, device=DEV, dtype=torch.float16) for _ in range(3)]
    c = compile_model(Attn(0.125), xs, fuse=True, verify=False)
    assert kinds(c) == ["attention"]
    ref = Attn(0.125)(*[x.float() for x in xs])
    torch.testing.assert_close(c(*xs).float(), ref, atol=2e-3, rtol=1e-2)

    class C(torch.nn.Module):
        def forward(self, x):
            return torch.relu(x * 1.5) * 0.5

    assert kinds(compile_model(C(), (torch.randn(64, 256, device=DEV, dtype=torch.float16),), fuse=True)) == ["flat"]


def test_broadcast_chain_workload_compiles_and_verifies():
    R, C = 512, 4096
    x = torch.randn(R, C, device=DEV).half()
    b = (torch.randn(C, device=DEV) * 0.1).half()
    s = (torch.rand(C, device=DEV) + 0.5).half()
    c = compile_model(BroadcastChain(), (x, b, s), fuse=True, extensions=True)
    assert kinds(c) == ["flat"] and c.verified


def test_bert_block_compiles_and_verifies():
    m = init_bert(BertBlock(2, 128)).half().to(DEV).eval()
    x = torch.randn(2, 128, 768, device=DEV).half()
    c = compile_model(m, (x,), fuse=True, extensions=True)
    # fused: attention, the bias + GELU chain, and two residual + bias adds with their LayerNorms
    assert kinds(c).count("attention") == 1 and kinds(c).count("flat") == 1
    assert kinds(c).count("add_layer_norm") == 2
    assert c.verified, c.report


@pytest.mark.parametrize("batch,seq", [(1, 1), (1, 24), (3, 200)])
def test_bert_block_small_and_ragged_sizes_verify(batch, seq):
    """The whole rewritten plan (merged projections read as views, attention stored in the
    heads-merge order, add + LayerNorm, the GELU chain) at one token, a sequence shorter than
    one key tile and a ragged one, through the equivalence gate."""
    m = init_bert(BertBlock(batch, seq)).half().to(DEV).eval()
    x = torch.randn(batch, seq, 768, device=DEV).half()
    c = compile_model(m, (x,), fuse=True, extensions=True)
    assert kinds(c).count("add_layer_norm") == 2
    assert c.verified, c.report


def test_gate_catches_miscompile():
    xs = [torch.randn(1, 2, 20, 16, device=DEV) for _ in range(3)]
    c = compile_model(Attn(), xs, fuse=True)
    bad = copy.deepcopy(c.plan)
    for s in bad["steps"]:
        if s.get("launch") == "attention":
            s["attrs"]["scale"] *= 1.5
    c.plan = bad
    rep = verify_equivalence(Attn(), c, xs)
    assert rep.ok is False and "exceed" in rep.reason
    with pytest.raises(EquivalenceError):
        assert_equivalent(Attn(), c, xs)


def test_benchmark_only_after_verification():
    xs = [torch.randn(1, 2, 128, 64, device=DEV) for _ in range(3)]
    unverified = compile_model(Attn(0.125), xs, fuse=True, verify=False)
    with pytest.raises(UnverifiedSpeedupError):
        benchmark(Attn(0.125), unverified, xs)
    c = compile_model(Attn(0.125), xs, fuse=True)
    r = benchmark(Attn(0.125), c, xs, warmup=3, iters=10, unfused=compile_model(Attn(0.125), xs, verify=False))
    assert r.fused_ms > 0 and r.fused_launches == 1 and r.eager_launches == 5
