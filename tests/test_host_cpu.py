"""Host-side logic on the CPU: plan validation, the plan executor's torch steps and
errors, descriptors, the verify gate and the benchmark gate.  Mirrors the
reference's tests/test_runtime.py, test_plan_validation.py, test_triton.py
(launch-attr and writer contracts) and test_verify_bench.py (compiler-free parts)."""

import copy

import pytest
import torch

import oracle
from fusionpass_b200 import kernels
from fusionpass_b200.bench import UnverifiedSpeedupError, benchmark, plan_bytes
from fusionpass_b200.runtime import execute_plan
from fusionpass_b200.validate import validate_plan
from fusionpass_b200.verify import EquivalenceError, assert_equivalent, default_tolerances, verify_equivalence


def _torch_step(op, operands, result, shape, dtype="f32", attrs=None):
    return {"kind": "torch", "op": op, "operands": operands, "result": result, "shape": shape,
            "dtype": dtype, "attrs": {} if attrs is None else attrs}


GOOD = {"version": 1, "inputs": [{"name": "arg0", "shape": [2, 2], "dtype": "f32"}],
        "steps": [_torch_step("relu", ["arg0"], "v0", [2, 2])], "outputs": ["v0"]}


# ---------------------------------------------------------------- runtime
def test_execute_elementwise_ops():
    a = torch.tensor([[-1.0, 2.0], [0.5, -3.0]])
    b = torch.tensor([[1.0, 1.0], [2.0, 2.0]])
    plan = {"version": 1,
            "inputs": [{"name": "arg0", "shape": [2, 2], "dtype": "f32"},
                       {"name": "arg1", "shape": [2, 2], "dtype": "f32"}],
            "steps": [_torch_step("add", ["arg0", "arg1"], "v0", [2, 2]),
                      _torch_step("mul", ["v0", "arg1"], "v1", [2, 2]),
                      _torch_step("scale", ["v1"], "v2", [2, 2], attrs={"factor": 0.5}),
                      _torch_step("relu", ["v2"], "v3", [2, 2]),
                      _torch_step("exp", ["v3"], "v4", [2, 2])],
            "outputs": ["v4"]}
    torch.testing.assert_close(execute_plan(plan, [a, b]), torch.exp(torch.relu((a + b) * b * 0.5)))


def test_execute_unfused_attention_plan():
    q, k, v = (torch.randn(1, 2, 8, 16) for _ in range(3))
    ins = [{"name": f"arg{i}", "shape": [1, 2, 8, 16], "dtype": "f32"} for i in range(3)]
    plan = {"version": 1, "inputs": ins,
            "steps": [_torch_step("transpose", ["arg1"], "v0", [1, 2, 16, 8]),
                      _torch_step("matmul", ["arg0", "v0"], "v1", [1, 2, 8, 8]),
                      _torch_step("scale", ["v1"], "v2", [1, 2, 8, 8], attrs={"factor": 0.25}),
                      _torch_step("softmax", ["v2"], "v3", [1, 2, 8, 8], attrs={"axis": 3}),
                      _torch_step("matmul", ["v3", "arg2"], "v4", [1, 2, 8, 16])],
            "outputs": ["v4"]}
    eager = torch.matmul(torch.softmax(torch.matmul(q, k.transpose(-2, -1)) * 0.25, dim=-1), v)
    torch.testing.assert_close(execute_plan(plan, [q, k, v]), eager)


def test_plan_version_mismatch():
    p = copy.deepcopy(GOOD)
    p["version"] = 99
    with pytest.raises(ValueError, match="unsupported plan version"):
        execute_plan(p, [torch.randn(2, 2)])


def test_wrong_input_count_shape_dtype():
    with pytest.raises(ValueError, match="expected 1 inputs"):
        execute_plan(GOOD, [])
    with pytest.raises(ValueError, match="arg0"):
        execute_plan(GOOD, [torch.randn(3, 3)])
    with pytest.raises(ValueError, match="arg0"):
        execute_plan(GOOD, [torch.randn(2, 2, dtype=torch.float16)])


def test_unknown_torch_op_and_step_kind():
    p = copy.deepcopy(GOOD)
    p["steps"][0]["op"] = "tanh"
    with pytest.raises(ValueError, match="unknown torch op"):
        execute_plan(p, [torch.randn(2, 2)])
    p = copy.deepcopy(GOOD)
    p["steps"][0]["kind"] = "cuda"
    with pytest.raises(ValueError, match="unknown kind"):
        execute_plan(p, [torch.randn(2, 2)])


def _fused_plan(launch="flat", desc=True):
    step = {"kind": "triton", "kernel": "fp_chain_0", "launch": launch, "operands": ["arg0"], "result": "v0",
            "shape": [2, 2], "dtype": "f32", "attrs": {"block": 1024}}
    if desc:
        step["attrs"]["desc"] = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    return {"version": 1, "inputs": [{"name": "arg0", "shape": [2, 2], "dtype": "f32"}], "steps": [step],
            "outputs": ["v0"]}


def test_fused_step_without_kernels_raises():
    with pytest.raises(RuntimeError, match="no kernels module"):
        execute_plan(_fused_plan(desc=False), [torch.randn(2, 2)], kernels=None)


def test_unknown_launch_kind_raises():
    with pytest.raises(ValueError, match="unknown launch kind"):
        execute_plan(_fused_plan(launch="bogus"), [torch.randn(2, 2)], validate=False)


def test_fused_step_on_cpu_has_no_fallback():
    with pytest.raises(RuntimeError, match="no CPU"):
        execute_plan(_fused_plan(), [torch.randn(2, 2)])


def test_malformed_fused_step_rejected():
    p = copy.deepcopy(GOOD)
    p["steps"][0] = {"kind": "triton", "op": "relu", "operands": ["arg0"], "result": "v0", "shape": [2, 2],
                     "dtype": "f32", "attrs": {}}
    with pytest.raises(ValueError, match="bad triton step"):
        execute_plan(p, [torch.randn(2, 2)])


# ------------------------------------------------------------- validation
@pytest.mark.parametrize("mutate", [
    lambda p: p.update(version=2),
    lambda p: p["steps"][0].update(operands=["nope"]),
    lambda p: p["steps"][0].update(op="tanh"),
    lambda p: p["steps"][0].update(kind="cuda"),
    lambda p: p["steps"][0].update(result="arg0"),
    lambda p: p.update(outputs=["v9"]),
])
def test_bad_plans_rejected(mutate):
    p = copy.deepcopy(GOOD)
    mutate(p)
    with pytest.raises(ValueError):
        validate_plan(p)


def test_list_fields_and_input_specs():
    for key in ("inputs", "steps", "outputs"):
        p = copy.deepcopy(GOOD)
        p[key] = "nope"
        with pytest.raises(ValueError, match=key):
            validate_plan(p)
    p = copy.deepcopy(GOOD)
    p["inputs"][0]["dtype"] = "bf16"
    with pytest.raises(ValueError, match="bad input spec"):
        validate_plan(p)


def test_attention_arity_and_descriptor_checks():
    p = {"version": 1, "inputs": [{"name": f"arg{i}", "shape": [1, 2, 8, 16], "dtype": "f32"} for i in range(3)],
         "steps": [{"kind": "triton", "kernel": "fp_attention", "launch": "attention",
                    "operands": ["arg0", "arg1", "arg2"], "result": "v0", "shape": [1, 2, 8, 16], "dtype": "f32",
                    "attrs": {**kernels.attention_launch_attrs(0.125), "desc": kernels.attention_descriptor()}}],
         "outputs": ["v0"]}
    validate_plan(p)
    bad = copy.deepcopy(p)
    bad["steps"][0]["attrs"]["desc"] = kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a0"]}])
    with pytest.raises(ValueError, match="descriptor"):
        validate_plan(bad)
    p["steps"][0]["operands"] = ["arg0", "arg1"]
    with pytest.raises(ValueError, match="exactly 3 operands"):
        validate_plan(p)


def test_chain_descriptor_checks():
    p = _fused_plan()
    validate_plan(p)
    bad = copy.deepcopy(p)
    bad["steps"][0]["attrs"]["desc"]["ops"][0]["a"] = 5
    with pytest.raises(ValueError, match="undefined slot"):
        validate_plan(bad)
    bad = copy.deepcopy(p)
    bad["steps"][0]["launch"] = "rows"
    with pytest.raises(ValueError, match="softmax"):
        validate_plan(bad)


def test_plan_bytes_are_algorithmic():
    fused = {"version": 1, "inputs": [{"name": f"arg{i}", "shape": [1, 2, 1024, 64], "dtype": "f16"}
                                      for i in range(3)],
             "steps": [{"kind": "triton", "kernel": "fp_attention", "launch": "attention",
                        "operands": ["arg0", "arg1", "arg2"], "result": "v0", "shape": [1, 2, 1024, 64],
                        "dtype": "f16", "attrs": kernels.attention_launch_attrs(0.125)}],
             "outputs": ["v0"]}
    assert plan_bytes(fused) == 4 * 262144  # q, k, v read once, out written once


# ------------------------------------------------------------ descriptors
def test_launch_attr_contract():
    assert kernels.chain_launch_attrs([8, 16], rows=False) == {"block": 1024}
    assert kernels.chain_launch_attrs([6, 100], rows=True) == {"block_n": 128, "num_warps": 4}
    assert kernels.chain_launch_attrs([4, 3000], rows=True)["num_warps"] == 8
    assert kernels.next_pow2(100) == 128 and kernels.next_pow2(1) == 1
    a = kernels.attention_launch_attrs(0.25)
    assert a["scale"] == pytest.approx(0.25) and a["block_m"] == 64 and a["block_n"] == 64


def test_descriptor_writer_names_and_json_roundtrip(tmp_path):
    w = kernels.DescriptorWriter()
    body = [{"op": "add", "operands": ["a0", "a1"]}, {"op": "scale", "operands": ["t0"], "factor": 2.0},
            {"op": "relu", "operands": ["t1"]}, {"op": "exp", "operands": ["t2"]}]
    assert w.add_chain_kernel(2, body) == "fp_chain_0"
    assert w.add_chain_kernel(1, [{"op": "softmax", "operands": ["a0"]}]) == "fp_chain_1"
    assert w.add_attention_kernel() == kernels.KERNEL_ATTENTION == "fp_attention"
    t = kernels.load_kernels(w.write_path(tmp_path / "kernels.json"))
    assert t["fp_chain_0"]["mode"] == "flat" and t["fp_chain_1"]["mode"] == "rows"
    assert t["fp_chain_0"]["ops"][1] == {"op": "scale", "a": 2, "imm": 2.0}
    assert t == w.write()


def test_descriptor_slots_agree_with_oracle_program():
    from tests import _golden
    for name in _golden.names("chain"):
        meta, _ = _golden.load(name)
        d = kernels.chain_descriptor(meta["n_args"], meta["body"])
        ops, res = oracle.body_to_program(meta["n_args"], meta["body"])
        assert d["result"] == res
        assert [(o["op"], o["a"], o.get("b", -1)) for o in d["ops"]] == [(o[0], o[1], o[2]) for o in ops]


def test_descriptor_rejects_bad_bodies():
    with pytest.raises(ValueError, match="unsupported op"):
        kernels.chain_descriptor(1, [{"op": "tanh", "operands": ["a0"]}])
    with pytest.raises(ValueError, match="undefined"):
        kernels.chain_descriptor(1, [{"op": "relu", "operands": ["a3"]}])
    with pytest.raises(ValueError, match="exactly one softmax"):
        kernels.chain_descriptor(1, [{"op": "softmax", "operands": ["a0"]}, {"op": "softmax", "operands": ["t0"]}])


# ------------------------------------------------------------ verify gate
def test_default_tolerances():
    assert default_tolerances(torch.float16, False) == (1e-2, 1e-2)
    assert default_tolerances(torch.float32, True) == (5e-3, 5e-3)
    assert default_tolerances(torch.float32, False) == (1e-4, 1e-4)


class _Dummy:
    def __init__(self, fn, plan=GOOD):
        self.plan, self._fn = plan, fn

    def __call__(self, *xs):
        return self._fn(*xs)


def test_verify_equivalence_matches_and_mismatches():
    m = torch.nn.ReLU()
    x = torch.randn(4, 4)
    rep = verify_equivalence(m, _Dummy(torch.relu), (x,), extra_trials=2)
    assert rep.ok and rep.trials == 3 and rep.reason == ""
    assert_equivalent(m, _Dummy(torch.relu), (x,), extra_trials=0)
    rep = verify_equivalence(m, _Dummy(lambda t: torch.relu(t) + 1.0), (x,), extra_trials=0)
    assert rep.ok is False and "exceed" in rep.reason
    with pytest.raises(EquivalenceError):
        assert_equivalent(m, _Dummy(lambda t: torch.relu(t) + 1.0), (x,), extra_trials=0)


def test_verify_nan_pattern_must_match():
    m = torch.nn.Identity()
    x = torch.tensor([1.0, float("nan")])
    rep = verify_equivalence(m, _Dummy(lambda t: torch.nan_to_num(t)), (x,), extra_trials=0)
    assert not rep.ok and "NaN" in rep.reason


def test_benchmark_refuses_unverified():
    class D:
        verified = False
        report = None
        plan = {"steps": []}

    with pytest.raises(UnverifiedSpeedupError):
        benchmark(torch.nn.ReLU(), D(), (torch.randn(2, 2),))
