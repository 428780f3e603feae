"""bench.py's reference arm on the CPU: the driver runs it as
`bench.py --impl reference`, rank 0 printing one JSON line with the same
metric and config as the GPU arm; other ranks print nothing and exit 0."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    return r.stdout.strip().splitlines()


def test_reference_arm_prints_one_line():
    sys.path.insert(0, ROOT)
    import bench
    lines = _run({"RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "tok/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "config4-decode" and d["config"]["sessions"] == 4096
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_reference_arm_other_ranks_exit_quietly():
    assert _run({"RANK": "1"}) == []
