"""One rank of the world_size-2 gloo test of bench.py's multi-rank logic.

usage: python tests/_rank_worker.py <rank> <world> <port> <out.json>

Each rank takes its contiguous share of a global chain problem (rows) and of a
global attention problem ((batch, head) slices), computes it with the oracle
on the CPU (standing in for the GPU kernels, which these CPU ranks cannot run),
and the shards are collected with the same RankGroup.gather
(all_gather_into_tensor) that bench.py runs over NCCL.
"""

import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main() -> int:
    rank, world, port, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch
    import torch.distributed as tdist

    import bench
    from oracle import attention as oa

    tdist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = bench.RankGroup(rank, world, torch.device("cpu"))
        g.barrier()
        ms_max = g.max(10.0 + 5.0 * rank)  # the last rank is the slowest
        all_pass = g.all_ok(True)
        one_fails = g.all_ok(rank == 0)  # every rank but rank 0 fails its check
        g.barrier()

        # chain: this rank's rows of the global problem, gathered
        rows, cols = 64, 256
        x, b, s = bench.chain_inputs(rows, cols)
        r0, r1 = bench.shard_range(rows, rank, world)
        y_rank = bench.chain_oracle([x[r0:r1].contiguous(), b, s], bench.CFG2_BODY, ["full", "col", "col"])
        y_all = g.gather(torch.from_numpy(y_rank))
        y_one = bench.chain_oracle([x, b, s], bench.CFG2_BODY, ["full", "col", "col"])
        chain_equal = bool(np.array_equal(y_all.numpy(), y_one))

        # attention: this rank's (batch, head) slices of a small global problem, gathered
        gen = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(2, 3, 40, 16, generator=gen).half() for _ in range(3))
        a, b_ = bench.shard_range(6, rank, world)
        part = [bench.slices_of(t, a, b_).numpy() for t in (q, k, v)]
        o_rank = oa.attention_fwd(*part, 0.25).reshape(-1, 40, 16)
        o_all = g.gather(torch.from_numpy(o_rank))
        o_one = oa.attention_fwd(q.numpy(), k.numpy(), v.numpy(), 0.25).reshape(-1, 40, 16)
        attn_equal = bool(np.array_equal(o_all.numpy(), o_one))

        res = {"rank": rank, "ms_max": ms_max, "all_pass": all_pass, "one_fails": one_fails,
               "rows": [r0, r1], "slices": [a, b_], "chain_shape": list(y_all.shape),
               "chain_equal": chain_equal, "attn_shape": list(o_all.shape), "attn_equal": attn_equal,
               "rate": bench.strong_rate(100, 1.0e6, ms_max)}
    finally:
        tdist.destroy_process_group()
    Path(out).write_text(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
