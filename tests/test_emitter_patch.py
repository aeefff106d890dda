"""The descriptor emitter: planner twin vs the plans the C++ patch must produce.

integration/PlanEmitter.descriptors.patch adds descriptor emission to the
reference's C++ plan emitter (lib/Plan/PlanEmitter.cpp:120-149); it cannot be
built here (no LLVM/MLIR 18).  These tests pin the rules it implements:

* the planner twin, run on the reference's fusion lit inputs (re-printed in
  tests/golden/emitter_inputs.mlir by tests/golden/make_emitter_golden.py),
  produces exactly the committed plans, descriptors included;
* those plans show what the lit tests' FileCheck lines require of the passes;
* the patch emits the descriptor keys the plans use, at both fused-op branches;
* with a reference checkout named by $FUSIONPASS_REFERENCE, the original lit
  files give the same plans and the patch applies cleanly.
"""

import json
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from fusionpass_b200 import planner

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
PATCH = ROOT / "integration" / "PlanEmitter.descriptors.patch"


def _plans_from(text: str) -> dict:
    out = {}
    for fn, g in planner.parse_fp_mlir(text).items():
        out[fn.replace("__", ".")] = planner.compile_graph(g, fuse=True)[0]
    return out


@pytest.fixture(scope="module")
def golden():
    return json.loads((GOLDEN / "emitter_plans.json").read_text())


@pytest.fixture(scope="module")
def plans():
    return _plans_from((GOLDEN / "emitter_inputs.mlir").read_text())


def test_planner_reproduces_the_committed_plans(plans, golden):
    assert set(plans) == set(golden)
    for name in golden:
        assert json.loads(json.dumps(plans[name])) == golden[name], name


def _fused(plan):
    return [s for s in plan["steps"] if s["kind"] == "triton"]


def test_plans_meet_the_lit_expectations(golden):
    chain = _fused(golden["fuse_chains.chain"])
    assert len(chain) == 1 and chain[0]["launch"] == "flat"
    assert [o["op"] for o in chain[0]["attrs"]["desc"]["ops"]] == ["add", "scale", "relu", "exp"]
    assert chain[0]["attrs"]["desc"]["ops"][1]["imm"] == 2.0
    assert _fused(golden["fuse_chains.multiuse"]) == []  # a multi-use producer stays materialised
    sm = _fused(golden["fuse_chains.softmax_chain"])
    assert len(sm) == 1 and sm[0]["launch"] == "rows" and sm[0]["attrs"]["desc"]["mode"] == "rows"
    assert sm[0]["attrs"]["block_n"] == 64 and sm[0]["attrs"]["num_warps"] == 4
    assert _fused(golden["fuse_chains.softmax_axis0"]) == []  # softmax over axis 0 is not fusible
    for key in ("fuse_chains.dedupe", "dedupe_mul.dedupe"):
        d = _fused(golden[key])
        assert len(d) == 1 and d[0]["operands"] == ["arg0"]  # the duplicated operand enters once
        assert d[0]["attrs"]["desc"]["ops"][0] == {"op": "mul", "a": 0, "b": 0}
    att = _fused(golden["fuse_attention.attn"])
    assert len(att) == 1 and att[0]["launch"] == "attention" and att[0]["attrs"]["scale"] == 0.25
    assert att[0]["attrs"]["desc"] == {"op": "attention", "head_dim": 64}
    assert _fused(golden["fuse_attention.attn_multiuse"]) == []  # P is returned, so it stays
    assert golden["fuse_attention.attn_multiuse"]["outputs"] == ["v3", "v2"]
    assert _fused(golden["two_softmax.two_sm"]) == []  # one softmax per chain
    assert [s["launch"] for s in _fused(golden["no_fuse_head_dim.attn_d24"])] == ["rows"]  # D=24: no attention


def test_patch_emits_the_descriptor_keys_at_both_branches(golden):
    text = PATCH.read_text()
    added = "\n".join(ln[1:] for ln in text.splitlines() if ln.startswith("+") and not ln.startswith("+++"))
    keys = set()
    for plan in golden.values():
        for s in _fused(plan):
            d = s["attrs"]["desc"]
            keys |= set(d)
            for sub in d.get("inputs", []) + d.get("ops", []):
                keys |= set(sub)
    for k in sorted(keys):
        assert f'"{k}"' in added, f"the patch never emits descriptor key {k!r}"
    assert "emitChainDescriptor(fc)" in added and "emitAttentionDescriptor(fa)" in added
    assert re.search(r'a\["desc"\]', added)
    assert "+++ b/lib/Plan/PlanEmitter.cpp" in text and "DescriptorEmitter.cpp" in text


REF = os.environ.get("FUSIONPASS_REFERENCE")


@pytest.mark.skipif(not REF, reason="set FUSIONPASS_REFERENCE to a reference checkout")
def test_original_lit_files_give_the_same_plans(golden):
    got = {}
    for name in ("fuse_chains", "fuse_attention", "dedupe_mul", "two_softmax", "no_fuse_head_dim"):
        text = (Path(REF) / "test" / "fusion" / f"{name}.mlir").read_text()
        for fn, g in planner.parse_fp_mlir(text).items():
            got[f"{name}.{fn}"] = planner.compile_graph(g, fuse=True)[0]
    assert json.loads(json.dumps(got)) == golden


@pytest.mark.skipif(not REF or shutil.which("patch") is None, reason="needs a reference checkout and patch(1)")
def test_patch_applies_to_the_reference(tmp_path):
    for sub in ("lib", "include"):
        shutil.copytree(Path(REF) / sub, tmp_path / sub)
    r = subprocess.run(["patch", "-p1", "--dry-run", "-d", str(tmp_path)], stdin=PATCH.open(), capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stdout + r.stderr
