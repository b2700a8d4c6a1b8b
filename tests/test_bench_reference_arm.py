"""bench.py's host-side contract on the CPU: the reference arm (`--impl
reference`) prints one JSON line with the headline arm's metric and config, the
reference-arm keys (impl, cpu_baseline, a zero-copy e2e), and nothing on ranks
other than 0; the clock record summarises nvidia-smi samples (median SM clock,
throttle reasons seen Active) and tolerates unreadable values."""

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


def test_clock_summary_reads_nvidia_smi_lines():
    sys.path.insert(0, ROOT)
    import bench
    idle = "0, 1965, 1965, 300.5, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active\n"
    capped = "0, 1800, 1965, 999.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active\n"
    hot = "0, 1200, 1965, 700.0, 0x0000000000000008, Active, Not Active, Not Active, Not Active\n"
    s = bench.summarize_clocks([idle, capped, idle])
    assert s == {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    assert bench.summarize_clocks([idle, hot, hot])["reasons"] == ["hw_slowdown"]
    assert bench.summarize_clocks([idle, hot, hot])["sm_mhz"] == 1200.0
    # Unreadable values are skipped; incomplete lines and no lines give None.
    na = "0, [N/A], [N/A], [N/A], [N/A], Not Active, Not Active, Not Active, Not Active\n"
    assert bench.summarize_clocks([na]) == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 1}
    assert bench.summarize_clocks(["0, 1965\n"]) is None and bench.summarize_clocks([]) is None
