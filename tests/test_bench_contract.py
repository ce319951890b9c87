"""The bench's reference arm runs on the host cores: check its JSON lines (CPU only).

Config 1 runs the oracle port on a bounded sample of query tiles (extrapolated, and marked
so); config 0 runs the unmodified reference itself under the Triton interpreter on the whole
layer (when the reference install is present)."""
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def run_arm(config, steps=1, warmup=0):
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--config", str(config), "--steps", str(steps), "--warmup", str(warmup)],
                       capture_output=True, text=True, timeout=600, cwd=REPO)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


def check_common(line):
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "config", "cpu_baseline", "e2e", "extrapolated"):
        assert key in line, key
    assert line["value"] > 0 and line["unit"] == "tokens/s"
    assert line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_port_sample_is_marked_extrapolated():
    line = run_arm(1)
    check_common(line)
    assert line["cpu_baseline"]["kind"] == "port" and line["extrapolated"] is True
    assert line["config"]["workload"].startswith("cfg1")
    # the timed sample itself fits the run: ms_per_step is the sample, not the layer estimate
    assert line["ms_per_step"] < line["est_ms_per_layer"]


def test_reference_arm_config0_runs_the_reference_itself():
    line = run_arm(0)
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    check_common(line)
    assert line["cpu_baseline"]["kind"] == "reference" and line["extrapolated"] is False
    assert line["config"]["workload"].startswith("cfg0")
