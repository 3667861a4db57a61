"""bench.py's reference arm runs on any CPU box: one JSON line in the driver's format."""
import json
import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def _run(*extra, env=None):
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1",
           *extra]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=REPO)


def _line(r):
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    return json.loads(lines[0])


def test_default_workload_is_config5_strong_scaling():
    sys.path.insert(0, str(REPO))
    import bench

    a = bench.parse_args([])
    assert a.config == 5 and a.steps == 64 and a.gpus == 1
    assert bench.parse_args(["--config", "2"]).steps == 100


def test_reference_arm_prints_one_contract_line():
    d = _line(_run())
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["steps"] == 1
    assert d["config"]["workload"].startswith("config5") and d["scaling"] == "strong"
    assert d["config"]["global_batch"] == 512
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_config2():
    d = _line(_run("--config", "2"))
    assert d["config"]["workload"].startswith("config2") and d["config"]["global_batch"] == 64


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = _run(env=env)
    assert r.returncode == 0 and r.stdout.strip() == ""
