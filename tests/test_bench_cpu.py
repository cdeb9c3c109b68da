"""bench.py's reference arm (the reference's CPU step on a bounded sample)
runs without a GPU and prints one JSON line with the contract's keys, on the
metric BASELINE.json names."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    env = {k: v for k, v in os.environ.items() if k not in ("WORLD_SIZE", "RANK", "LOCAL_RANK")}
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    line = json.loads(lines[0])
    with open(os.path.join(REPO, "BASELINE.json")) as f:
        assert line["metric"] == json.load(f)["metric"]
    assert line["impl"] == "reference" and line["unit"] == "params/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["n_gpus"] == 1 and line["steps"] == 1 and line["warmup"] == 3
    assert line["ms_per_step"] > 0 and line["config"]["workload"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] == "reference" and cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_config4_cpu_baseline_runs_the_installed_reference():
    """Config 4's cpu_baseline times the reference's own HybridMuonAdamW.step
    (from baseline/_ref) when it is installed, else the restated arithmetic."""
    sys.path.insert(0, REPO)
    import bench
    sec, threads, kind = bench.reference_muon_cpu_time((256, 384))
    assert sec > 0 and threads >= 1
    installed = os.path.isdir(os.path.join(REPO, "baseline", "_ref", "streamtrain"))
    assert kind == ("reference" if installed else "port")
