"""Multi-rank logic of bench.py on CPU: two gloo ranks over 127.0.0.1.

The GPU run uses the same RankGroup over NCCL, one process per GPU.  The
partition is strong scaling: each rank owns a contiguous share of the global
problem's independent units (chain rows, attention (batch, head) slices); the
data path has no collective, and the outputs are collected afterwards with
all_gather_into_tensor.
"""

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
WORKER = ROOT / "tests" / "_rank_worker.py"


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def two_ranks(tmp_path_factory):
    d = tmp_path_factory.mktemp("ranks")
    port = _free_port()
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    procs = [subprocess.Popen([sys.executable, str(WORKER), str(r), "2", str(port), str(d / f"r{r}.json")],
                              env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
             for r in range(2)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            pytest.fail("gloo ranks did not finish")
        outs.append(out.decode(errors="replace"))
    for r, p in enumerate(procs):
        assert p.returncode == 0, f"rank {r} failed:\n{outs[r][-3000:]}"
    return [json.loads((d / f"r{r}.json").read_text()) for r in range(2)]


def test_max_over_ranks_is_the_slowest_rank(two_ranks):
    assert [r["ms_max"] for r in two_ranks] == [15.0, 15.0]


def test_pass_fail_vote_is_joint(two_ranks):
    assert all(r["all_pass"] for r in two_ranks)
    assert not any(r["one_fails"] for r in two_ranks)


def test_strong_scaling_rate_counts_the_global_problem_once(two_ranks):
    # 100 steps x 1e6 units of the whole (split) problem in 15 ms (the slowest rank)
    for r in two_ranks:
        assert r["rate"] == pytest.approx(100 * 1.0e6 / 15e-3)


def test_shards_tile_the_global_problem(two_ranks):
    a, b = two_ranks
    assert a["rows"] == [0, 32] and b["rows"] == [32, 64]
    assert a["slices"] == [0, 3] and b["slices"] == [3, 6]


def test_gathered_outputs_equal_the_single_rank_outputs(two_ranks):
    for r in two_ranks:
        assert r["chain_shape"] == [64, 256] and r["chain_equal"]
        assert r["attn_shape"] == [6, 40, 16] and r["attn_equal"]


@pytest.mark.parametrize("n,world", [(4096, 1), (4096, 8), (128, 8), (128, 3), (5, 8), (32, 4)])
def test_shard_range_is_a_contiguous_cover(n, world):
    import bench

    spans = [bench.shard_range(n, r, world) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 == b0 and a0 <= a1
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_rows_chain_gate_uses_the_rows_oracle_and_a_relative_budget():
    """The bench's rows-chain entries check softmax(x * 0.5) against the oracle's rows
    restatement; outputs of ~1 / cols sit far below the f16 atol, so the gate is relative:
    a softmax of the wrong scale passes the f16 budget but fails the relative one."""
    import numpy as np
    import torch

    import bench

    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 4096, generator=g).half()
    ref = torch.from_numpy(bench.chain_oracle([x], bench.ROWS_BODY, ["full"]))
    want = torch.softmax(x.float() * 0.5, dim=-1)
    assert np.allclose(ref.float().numpy(), want.numpy(), rtol=1e-2, atol=1e-6)
    wrong = torch.softmax(x.float() * 0.4, dim=-1).half()
    assert bench.budget_frac(wrong, ref) <= 1.0  # the f16 atol of 2e-3 hides it
    assert bench.budget_frac(wrong, ref, tol=(1e-6, 1e-2)) > 1.0
    assert bench.budget_frac(ref, ref, tol=(1e-6, 1e-2)) == 0.0


def test_rotating_sets_cover_twice_the_l2():
    import bench

    for nbytes in (67_125_248, 8_396_800, 1_000, 10**10):
        k = bench.rotating_sets(nbytes)
        assert k >= 2 and (k * nbytes >= 2 * bench.L2_BYTES or k == 2 and nbytes >= bench.L2_BYTES)


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3"]) == 0
    assert capsys.readouterr().out == ""
