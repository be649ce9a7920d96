"""One rank of the world_size-2 gloo check of bench.py's multi-rank host logic; tests/test_bench_ranks.py starts two.

argv: rank world port out.json.  The rank joins a gloo group on 127.0.0.1, reduces per-rank timings with
bench.rank_max, draws its request ids, runs bench.reference_arm as a non-zero rank would, and writes what it saw.
"""
import datetime
import json
import os
import sys

rank, world, port, out = int(sys.argv[1]), int(sys.argv[2]), sys.argv[3], sys.argv[4]
os.environ["MASTER_ADDR"] = "127.0.0.1"
os.environ["MASTER_PORT"] = port
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch.distributed as dist  # noqa: E402

dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
import bench  # noqa: E402

# timings as an engine rank measures them (total, prefill, decode ms): rank 1 is slower in one, faster in another
mine = [100.0 + 10.0 * rank, 40.0 - rank, 60.0 + 0.5 * rank]
got = bench.rank_max(mine, "cpu")
ids = bench.prompt_ids(1000 + rank)


class _Args:
    steps, warmup = 1, 0


ref = "returned" if rank != 0 and bench.reference_arm(_Args(), rank, world) is None else "not run"
dist.barrier()
with open(out, "w") as f:
    json.dump({"rank": rank, "got": got, "ids": ids[:16].tolist(), "reference_arm": ref}, f)
dist.destroy_process_group()
