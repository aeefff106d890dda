"""Multi-rank logic of bench.py on CPU: two gloo ranks over 127.0.0.1.

The GPU run uses the same RankGroup over NCCL, one process per GPU; the data
path has no collective (weak scaling), only the timing and pass/fail votes do.
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


def test_weak_scaling_rate_counts_every_rank(two_ranks):
    # 2 ranks x 100 steps x 1e6 units in 15 ms (the slowest rank)
    for r in two_ranks:
        assert r["rate"] == pytest.approx(2 * 100 * 1.0e6 / 15e-3)


def test_each_rank_owns_its_own_data(two_ranks):
    a, b = two_ranks
    assert a["x_shape"] == b["x_shape"] == [4096, 4096]
    assert a["q_shape"] == b["q_shape"] == [8, 16, 2048, 64]
    assert a["x_head"] != b["x_head"]
    assert a["q_head"] != b["q_head"]


def test_reference_arm_runs_on_rank_zero_only(monkeypatch, capsys):
    import bench

    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3"]) == 0
    assert capsys.readouterr().out == ""
