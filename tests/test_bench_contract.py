"""bench.py's reference arm on the CPU: the JSON line the driver divides the repo arm's line by.

The driver computes the speed-up only when both arms print the same `metric` for the same config,
so the reference arm must name the metric exactly as the repo arm does (both call
bench.metric_name), carry `impl: reference`, a `cpu_baseline` describing its own run, and an
`e2e` with no host-device bytes. One step of the down config's bounded sample runs in ~20 s.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_reference_arm_line_matches_the_repo_arms_contract():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--config", "down", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == bench.metric_name("down")
    assert d["unit"] == "TFLOPS" and d["higher_is_better"] is True
    assert d["steps"] == 1 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["config"]["workload"] == "down_wgrad"  # the repo arm's f"{config}_wgrad"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
