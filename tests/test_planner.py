"""The planner twin reproduces the reference compiler's fusion decisions and plan
format (lib/Transforms/FuseAttention.cpp, FuseChains.cpp, lib/Plan/PlanEmitter.cpp;
reference tests test_fusion.py, test_edge_cases.py, test/fusion/*.mlir).  CPU only:
plans are built and validated, fused steps are not executed here."""

import pytest
import torch
from torch import nn

from fusionpass_b200 import compile_model, planner
from fusionpass_b200.planner import UnsupportedOp
from fusionpass_b200.validate import validate_plan
from tests.models import Attn, BertBlock, BroadcastChain, Chain, RowChain, SoftmaxChain


def launches(plan):
    return [s.get("launch") or s.get("op") for s in plan["steps"]]


def plan_of(model, xs, fuse=True, extensions=False):
    g = planner.trace(model, xs, extensions=extensions)
    plan, table = planner.compile_graph(g, fuse=fuse, extensions=extensions)
    validate_plan(plan)
    return plan, table


@pytest.mark.parametrize("S", [1, 7, 64, 65, 130])
def test_attention_fused_single_step(S):
    xs = [torch.randn(1, 2, S, 16) for _ in range(3)]
    plan, table = plan_of(Attn(), xs)
    assert launches(plan) == ["attention"]
    st = plan["steps"][0]
    assert st["kernel"] == "fp_attention" and st["operands"] == ["arg0", "arg1", "arg2"]
    assert st["attrs"]["scale"] == pytest.approx(0.25)
    assert st["attrs"]["block_m"] == 64 and st["attrs"]["desc"]["op"] == "attention"
    assert "fp_attention" in table


def test_scales_fold_multiplicatively():
    class TwoScales(nn.Module):
        def forward(self, q, k, v):
            s = (torch.matmul(q, k.transpose(-2, -1)) * 0.5) * 0.5
            return torch.matmul(torch.softmax(s, dim=-1), v)

    plan, _ = plan_of(TwoScales(), [torch.randn(2, 4, 32, 64).half() for _ in range(3)])
    assert launches(plan) == ["attention"] and plan["steps"][0]["attrs"]["scale"] == pytest.approx(0.25)


def test_unsupported_head_dim_not_fused():
    plan, _ = plan_of(Attn(), [torch.randn(1, 2, 8, 24) for _ in range(3)])
    assert "attention" not in launches(plan)


def test_cross_attention_shapes_not_fused():
    q, k, v = torch.randn(1, 2, 8, 16), torch.randn(1, 2, 12, 16), torch.randn(1, 2, 12, 16)
    plan, _ = plan_of(Attn(), [q, k, v])
    assert "attention" not in launches(plan)


def test_multiuse_probabilities_not_fused():
    class Twice(nn.Module):
        def forward(self, q, k, v):
            p = torch.softmax(torch.matmul(q, k.transpose(-2, -1)), dim=-1)
            return torch.matmul(p, v) + torch.matmul(p, v)

    plan, _ = plan_of(Twice(), [torch.randn(1, 2, 16, 16) for _ in range(3)])
    assert "attention" not in launches(plan)


def test_chain_fused_single_flat_kernel():
    plan, table = plan_of(Chain(), [torch.randn(8, 16)])
    assert launches(plan) == ["flat"]
    st = plan["steps"][0]
    assert st["kernel"] == "fp_chain_0" and st["attrs"]["block"] == 1024
    assert [o["op"] for o in st["attrs"]["desc"]["ops"]] == ["scale", "add", "relu", "scale", "exp"]
    assert table["fp_chain_0"] == st["attrs"]["desc"]


def test_softmax_chain_rows_kernel_attrs():
    plan, _ = plan_of(SoftmaxChain(), [torch.randn(6, 100)])
    assert launches(plan) == ["rows"]
    assert plan["steps"][0]["attrs"]["block_n"] == 128 and plan["steps"][0]["attrs"]["num_warps"] == 4


def test_multiuse_producer_not_fused():
    """Like test/fusion/fuse_chains.mlir @multiuse: relu feeds exp and a matmul,
    so neither exp nor the matmul may absorb it."""
    class M(nn.Module):
        def forward(self, x):
            r = torch.relu(x)
            return torch.matmul(torch.exp(r), r)

    plan, _ = plan_of(M(), [torch.randn(4, 4)])
    assert launches(plan) == ["relu", "exp", "matmul"]


def test_multiuse_absorbed_when_all_uses_merge():
    """Once both consumers sit in one chain the deduplicated producer has one use,
    so the greedy rewrite fuses it as well (FuseChains.cpp:59,64-67)."""
    class M(nn.Module):
        def forward(self, x):
            r = torch.relu(x)
            return torch.exp(r) + r * 3.0

    plan, _ = plan_of(M(), [torch.randn(4, 4)])
    assert launches(plan) == ["flat"] and plan["steps"][0]["operands"] == ["arg0"]


def test_non_last_axis_softmax_not_fused():
    class M(nn.Module):
        def forward(self, x):
            return torch.relu(torch.softmax(x * 0.5, dim=0))

    plan, _ = plan_of(M(), [torch.randn(6, 32)])
    assert "rows" not in launches(plan)


def test_two_softmaxes_never_share_a_chain():
    class M(nn.Module):
        def forward(self, x):
            return torch.softmax(torch.softmax(x, dim=-1), dim=-1)

    plan, _ = plan_of(M(), [torch.randn(4, 8)])
    assert launches(plan) == ["softmax", "softmax"]


def test_softmax_row_cap():
    plan, _ = plan_of(SoftmaxChain(), [torch.randn(2, 8193)])
    assert "rows" not in launches(plan)


def test_duplicate_operand_deduplicated():
    class M(nn.Module):
        def forward(self, x):
            return torch.relu(x * x)

    plan, _ = plan_of(M(), [torch.randn(5, 7)])
    assert launches(plan) == ["flat"] and plan["steps"][0]["operands"] == ["arg0"]


def test_rowchain_demo_and_unfused_plan_names():
    plan, _ = plan_of(RowChain(), [torch.randn(4, 64), torch.randn(4, 64)])
    assert launches(plan) == ["rows"]
    plan, _ = plan_of(RowChain(), [torch.randn(4, 64), torch.randn(4, 64)], fuse=False)
    assert [s["result"] for s in plan["steps"]] == ["v0", "v1", "v2", "v3", "v4"]
    assert all(s["kind"] == "torch" for s in plan["steps"])


def test_broadcast_raises_without_extensions():
    with pytest.raises(UnsupportedOp):
        plan_of(BroadcastChain(), [torch.randn(4, 8), torch.randn(8), torch.randn(8)])


def test_broadcast_chain_with_extensions():
    plan, _ = plan_of(BroadcastChain(), [torch.randn(64, 32).half(), torch.randn(32).half(), torch.randn(32).half()],
                      extensions=True)
    assert launches(plan) == ["flat"]
    d = plan["steps"][0]["attrs"]["desc"]
    assert [i["bcast"] for i in d["inputs"]] == ["full", "col", "col"]
    assert [o["op"] for o in d["ops"]] == ["add", "mul", "relu", "scale", "add"]


def test_bert_block_plan_shape():
    m = BertBlock(2, 64).half().eval()
    plan, table = plan_of(m, [torch.randn(2, 64, 768).half()], extensions=True)
    kinds = launches(plan)
    assert kinds.count("attention") == 1
    chains = [s for s in plan["steps"] if s.get("launch") == "flat"]
    ops = sorted(tuple(o["op"] for o in s["attrs"]["desc"]["ops"]) for s in chains)
    # the two residual + bias chains feed LayerNorms: fused into add_layer_norm steps
    assert ops == [("add", "gelu")]
    lns = [s for s in plan["steps"] if s.get("op") == "add_layer_norm"]
    assert len(lns) == 2 and kinds.count("layer_norm") == 0
    assert all(s["attrs"]["n_addends"] == 3 and len(s["operands"]) == 5 for s in lns)
    # the q / k / v biases have no chain to join: folded back into their linear steps, and the
    # three projections of x merged into one GEMM over the concatenated weights and biases
    linears = [s for s in plan["steps"] if s.get("op") == "linear"]
    assert len(linears) == 4 and [len(s["operands"]) for s in linears] == [3, 2, 2, 2]
    assert linears[0]["shape"][-1] == 3 * 768
    cats = [s for s in plan["steps"] if s.get("op") == "cat"]
    assert [c["shape"] for c in cats] == [[3 * 768, 768], [3 * 768]]
    narrows = [s["attrs"] for s in plan["steps"] if s.get("op") == "narrow"]
    assert [(a["start"], a["length"]) for a in narrows] == [(0, 768), (768, 768), (1536, 768)]
    assert not any(s.get("op") == "add" for s in plan["steps"])
    # the attention result feeds the heads merge: stored as [B, S, H, D]
    att = [s for s in plan["steps"] if s.get("launch") == "attention"][0]
    assert att["attrs"]["out_layout"] == [0, 2, 1, 3]
    validate_plan(plan)


def test_linear_bias_fold_keeps_chained_biases():
    class M(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a, self.b = torch.nn.Linear(16, 16), torch.nn.Linear(16, 16)
            self.ln = torch.nn.LayerNorm(16)

        def forward(self, x):
            return self.ln(self.b(torch.nn.functional.gelu(self.a(x))))

    g = planner.trace(M().eval(), (torch.randn(4, 16),), extensions=True)
    plan, _ = planner.compile_graph(g, fuse=True, extensions=True)
    linears = [s for s in plan["steps"] if s.get("op") == "linear"]
    chains = [s for s in plan["steps"] if s.get("launch") == "flat"]
    # a's bias joins the GELU chain; b's bias add is folded into its linear
    assert [len(s["operands"]) for s in linears] == [2, 3]
    assert [tuple(o["op"] for o in s["attrs"]["desc"]["ops"]) for s in chains] == [("add", "gelu")]
    assert not any(s.get("op") == "add" for s in plan["steps"])


def test_unfused_compile_verifies_on_cpu(tmp_path):
    c = compile_model(Chain(), [torch.randn(8, 16)], fuse=False, workdir=tmp_path)
    assert c.verified and c.report.trials == 3
    assert (tmp_path / "plan.json").exists() and (tmp_path / "model.mlir").exists()
    assert "fp.scale" in c.mlir_text and "func.func @main" in c.mlir_text


def test_mlir_text_matches_reference_format():
    g = planner.trace(Attn(), [torch.randn(2, 4, 32, 64) for _ in range(3)])
    text = planner.to_mlir(g)
    assert "fp.transpose %arg1 : tensor<2x4x32x64xf32> -> tensor<2x4x64x32xf32>" in text
    assert "fp.scale" in text and "{factor = 2.500000000e-01 : f32}" in text
    assert "fp.softmax %2 {axis = 3 : i64}" in text


def test_add_layer_norm_step_semantics_on_cpu():
    """The torch form of an add_layer_norm step (used where the kernel does not take the
    shape): the operands summed in order, then layer_norm."""
    from fusionpass_b200 import runtime
    g = torch.Generator().manual_seed(0)
    a, c = torch.randn(4, 16, generator=g), torch.randn(4, 16, generator=g)
    bias, w, b = torch.randn(16, generator=g), torch.randn(16, generator=g), torch.randn(16, generator=g)
    step = {"op": "add_layer_norm", "attrs": {"normalized_shape": [16], "eps": 1e-5, "n_addends": 3}}
    y = runtime._run_torch(step, [a, bias, c, w, b])
    ref = torch.nn.functional.layer_norm((a + bias) + c, (16,), w, b, 1e-5)
    assert torch.equal(y, ref)


def test_add_layer_norm_fusion_conditions():
    class M(nn.Module):
        def __init__(self, cols):
            super().__init__()
            self.lin, self.ln = nn.Linear(cols, cols), nn.LayerNorm(cols)

        def forward(self, x):
            return self.ln(x + self.lin(x))

    for cols, fused in ((64, True), (20, False), (4096, False)):  # 20 % 8 != 0; above 2048 columns
        g = planner.trace(M(cols).eval(), (torch.randn(3, cols),), extensions=True)
        plan, _ = planner.compile_graph(g, fuse=True, extensions=True)
        kinds = [s.get("op") or s.get("launch") for s in plan["steps"]]
        assert ("add_layer_norm" in kinds) == fused, (cols, kinds)
        assert ("layer_norm" in kinds) != fused
