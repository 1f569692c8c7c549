"""bench.py's command-line contract that runs without a GPU: the reference arm prints one
JSON line naming itself (its stock import fails offline, so the line carries the reason)
and exits 0; the module imports and its metric names the denoise time of the 14.4 s clip."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    rec = json.loads(lines[0])
    assert rec["impl"] == "reference"
    assert "value" in rec or rec.get("unavailable")


def test_metric_matches_baseline_json():
    sys.path.insert(0, ROOT)
    try:
        import bench
    finally:
        sys.path.remove(ROOT)
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        base = json.load(f)
    assert "denoise" in bench.METRIC and "14.4" in bench.METRIC
    assert "denoise" in base["metric"]
