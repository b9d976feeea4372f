"""The reference arm of bench.py runs without a GPU: the reference's own CPU
path (compiled from its sources into oracle/_ref) on bounded samples of the
workload, one process per host core, printing one JSON line with the same
metric, unit and config as the B200 arm.  Checked here on small samples of
c2, for both product methods."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("method", ["mfft", "schoolbook"])
def test_reference_arm_json_line(method):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "c2",
                        "--sample-n", "32", "--steps", "1", "--warmup", "3", "--method", method],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"].startswith("s per exact n x n W-bit matmul")
    assert line["unit"] == "s" and line["higher_is_better"] is False
    assert line["warmup"] >= 3 and line["steps"] == 1
    assert line["config"]["workload"] == "c2" and line["config"]["method"] == method
    assert line["config"]["sample_n"] == 32
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
    e = line["e2e"]
    assert e["value"] == line["value"] and e["h2d_bytes_per_step"] == 0
    assert e["d2h_bytes_per_step"] == 0
