"""Session sharding across ranks, on CPU: the same host logic bench.py uses on
N GPUs (one process per GPU, contiguous session ranges, no collective on the
data path, max-over-ranks timing), exercised with two gloo ranks."""
import json
import os
import socket
import subprocess
import sys

import pytest
from conftest import nb, orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "tests"))
from multi_rank_worker import session_tokens  # noqa: E402

from needle_b200.shard import max_over_ranks, session_range  # noqa: E402


def test_session_ranges_cover_every_session_once():
    for total in (0, 1, 7, 8, 4096, 4097):
        for world in (1, 2, 3, 4, 8):
            ranges = [session_range(total, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        session_range(4, 0, 0)
    assert max_over_ranks(3.5) == 3.5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_decode_their_shards_like_one_process(tiny_raw, tmp_path):
    path = tmp_path / "tiny.cact"
    path.write_bytes(tiny_raw)
    out = tmp_path / "result.json"
    total, world = 5, 2
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()), WORLD_SIZE=str(world))
    procs = [subprocess.Popen([sys.executable, os.path.join(ROOT, "tests", "multi_rank_worker.py"), str(path),
                               str(total), str(out)], env=dict(env, RANK=str(r), LOCAL_RANK=str(r)))
             for r in range(world)]
    try:
        codes = [p.wait(timeout=180) for p in procs]
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    assert codes == [0] * world
    res = json.loads(out.read_text())
    assert res["world"] == world and res["tmax"] == 1.5
    merged = {}
    for part in res["parts"]:
        s0, s1 = part["range"]
        assert sorted(int(k) for k in part["tokens"]) == list(range(s0, s1))
        merged.update({int(k): v for k, v in part["tokens"].items()})
    model = orc.Model(tiny_raw)
    assert merged == {i: session_tokens(model, orc, i) for i in range(total)}
