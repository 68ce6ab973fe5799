"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, rank 0 only.

The reference arm times the reference operator (the oracle's restatement of the eager op) on the host cores, so
it runs here; the GPU arm's line is checked on a B200.
"""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
KEYS = ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e")


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", *args],
                          cwd=REPO, env=env, capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    r = _run({}, "--steps", "1", "--warmup", "3", "--cpu-seconds", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert all(key in line for key in KEYS), sorted(set(KEYS) - set(line))
    assert line["impl"] == "reference" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 3 and line["n_gpus"] == 1
    assert line["config"]["workload"] and line["config"]["global_batch"] == 256
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["unit"] == line["unit"] and cb["cores"] >= 1
    assert cb["kind"] in ("port", "reference") and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # each step is a measured, bounded sample of the workload (32 of the 256 issue dates): ms_per_step is that
    # step's measured time and value its rate, so K steps fit inside the run
    flops = 12.0 * 32 * 16 * 512 * 512 * 128
    assert abs(line["ms_per_step"] - flops / (line["value"] * 1e12) * 1e3) <= 1e-6 * line["ms_per_step"]
    assert "32 issue dates" in line["step_is"]
    c1 = line["c1_cpu"]
    assert c1["shape_bhnd"] == [1, 8, 512, 64] and c1["ms_fwd_bwd"] > 0 and c1["cores"] == cb["cores"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--gpus", "2", "--steps", "1", "--warmup", "3", "--cpu-seconds", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
