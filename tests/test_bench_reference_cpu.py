"""The reference arm of bench.py (`--impl reference`: the CPU implementation of the path timed on the
host cores) keeps the JSON-line contract of the GPU arm, and under a multi-rank launch only rank 0
does the work.  Runs on CPU in about 15 s (one timed step of the oracle at the c2 workload)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env=None, *args):
    env = dict(os.environ, **(extra_env or {}))
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                          capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)


def test_reference_arm_json_line():
    p = _run(None, "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench  # noqa: E402  (the GPU arm's metric and unit)
    assert d["impl"] == "reference"
    assert d["metric"] == bench.METRIC and d["unit"] == bench.UNIT
    assert d["higher_is_better"] is False and d["value"] > 0
    assert d["steps"] == 1 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["global_batch"] == 32 and d["config"]["seq_len"] == 32768


def test_reference_arm_other_ranks_do_no_work():
    env = {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1", "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": "29555"}
    p = _run(env, "--gpus", "2", "--steps", "1", "--warmup", "0")
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
