"""bench.py's reference arm (`--impl reference`) on the CPU: one JSON line with
the headline arm's metric and config, the reference-arm keys (impl,
cpu_baseline, a zero-copy e2e), and silence on every rank but 0."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return [l for l in r.stdout.splitlines() if l.startswith("{")]


def test_reference_arm_line():
    sys.path.insert(0, ROOT)
    import bench
    lines = _run({"RANK": "0", "WORLD_SIZE": "1", "LOCAL_RANK": "0"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "tok/s"
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    args = bench.parse(["--steps", "1", "--warmup", "3"])
    assert d["config"] == json.loads(json.dumps(bench.headline_config(args, 1)))
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] > 0 and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_are_silent():
    assert _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []
