"""The reference arm of bench.py (the reference's CPU path, run by the
driver beside this library's arm) prints one JSON line with the contract's
keys and the same metric and config as this library's arm."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_line():
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, cwd=REPO, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    line = json.loads(lines[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["steps"] == 1 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["kind"] in ("port", "reference")

    sys.path.insert(0, REPO)
    import bench

    assert line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    # The same config object as this library's arm on the same workload.
    assert line["config"] == bench.workload_config("c1", 1, True)
