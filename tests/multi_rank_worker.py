"""One rank of the CPU sharding test (tests/test_multi_rank_cpu.py).

Launched as a separate process per rank with RANK / WORLD_SIZE / MASTER_ADDR /
MASTER_PORT in the environment; joins a gloo process group, decodes the
sessions that `session_range` assigns to it with the CPU oracle (no collective
on the data path), then gathers the per-session tokens and the max-over-ranks
of a per-rank time to rank 0, which writes them as JSON.

    python tests/multi_rank_worker.py <container.cact> <total_sessions> <out.json>
"""
import datetime
import importlib.util
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_pkg():
    pkg_dir = os.path.join(ROOT, "needle-rs_b200")
    spec = importlib.util.spec_from_file_location("needle_b200", os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["needle_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def session_tokens(model, orc, i):
    """Greedy tokens of session i: its own prompt, int8 KV on odd sessions."""
    p = np.random.default_rng(100 + i).integers(1, 512, 6 + i).astype(np.uint32)
    toks, _ = orc.greedy(model, p, 3, bool(i % 2))
    return [int(t) for t in toks]


def main():
    path, total, out = sys.argv[1], int(sys.argv[2]), sys.argv[3]
    import torch.distributed as dist
    import oracle as orc
    load_pkg()
    from needle_b200.shard import max_over_ranks, session_range
    dist.init_process_group("gloo", init_method="env://", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    s0, s1 = session_range(total, world, rank)
    orc.set_threads(1)
    model = orc.Model(open(path, "rb").read())
    mine = {i: session_tokens(model, orc, i) for i in range(s0, s1)}
    tmax = max_over_ranks(0.5 + rank, dist)
    gathered = [None] * world
    dist.all_gather_object(gathered, {"range": [s0, s1], "tokens": mine})
    if rank == 0:
        with open(out, "w") as f:
            json.dump({"world": world, "tmax": tmax, "parts": gathered}, f)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
