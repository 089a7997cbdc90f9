"""The JSON-line contract of bench.py's reference arm, run on the CPU.

`bench.py --impl reference` times the reference's own CPU implementation of
the config-2 path (oracle/_ref when the reference tree was compiled here,
else the C restatement) and prints one JSON line with the same metric,
unit and config as the GPU arm, `"impl": "reference"`, a `cpu_baseline`
that describes the run and an `e2e` object with no device copies."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def reference_line():
    env = dict(os.environ, OMP_NUM_THREADS=str(min(4, os.cpu_count() or 1)))
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_line(reference_line):
    d = reference_line
    assert d["impl"] == "reference"
    if "unavailable" in d:
        pytest.skip(d["unavailable"])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 1
    assert d["config"]["batch"] == 8 and d["config"]["L"] == 4096
    assert d["config"]["D"] == 1536 and d["config"]["N"] == 16
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert cb["value"] == pytest.approx(d["value"])
    e = d["e2e"]
    assert e["value"] == pytest.approx(d["value"]) and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
