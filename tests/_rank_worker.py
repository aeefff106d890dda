"""One rank of the world_size-2 gloo test of bench.py's multi-rank logic.

usage: python tests/_rank_worker.py <rank> <world> <port> <out.json>
"""

import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def main() -> int:
    rank, world, port, out = int(sys.argv[1]), int(sys.argv[2]), int(sys.argv[3]), sys.argv[4]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch
    import torch.distributed as tdist

    import bench

    tdist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        g = bench.RankGroup(rank, world, torch.device("cpu"))
        g.barrier()
        ms_max = g.max(10.0 + 5.0 * rank)  # the last rank is the slowest
        all_pass = g.all_ok(True)
        one_fails = g.all_ok(rank == 0)  # every rank but rank 0 fails its check
        g.barrier()
        rate = bench.weak_rate(world, 100, 1.0e6, ms_max)
        x, b, s = bench.chain_inputs(rank)
        q, _, _ = bench.attention_inputs(rank)
        res = {"rank": rank, "ms_max": ms_max, "all_pass": all_pass, "one_fails": one_fails, "rate": rate,
               "x_head": x[0, :8].float().tolist(), "q_head": q[0, 0, 0, :8].float().tolist(),
               "x_shape": list(x.shape), "q_shape": list(q.shape)}
    finally:
        tdist.destroy_process_group()
    Path(out).write_text(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
