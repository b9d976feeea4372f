"""The reference arm of bench.py runs without a GPU: the reference's own CPU
path (compiled from its sources into oracle/_ref) on bounded samples of the
workload -- its O(L n^2) phases at one size, one leaf per host core at
another, projected to the full size -- printing one JSON line with the same
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
                        "--sample-n", "32", "--leaf-n", "64", "--steps", "1", "--warmup", "3",
                        "--method", method],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"].startswith("s per exact n x n W-bit matmul")
    assert line["unit"] == "s" and line["higher_is_better"] is False
    assert line["warmup"] >= 3 and line["steps"] == 1
    assert line["config"]["workload"] == "c2" and line["config"]["method"] == method
    assert line["config"]["phase_n"] == 32 and line["config"]["leaf_n"] == 64
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert cb["projected"] is True and cb["single_thread_value"] > 0
    e = line["e2e"]
    assert e["value"] == line["value"] and e["h2d_bytes_per_step"] == 0
    assert e["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_one_line():
    """Launched the way the multi-GPU runs are (torchrun, world size 2): rank
    0 alone times the reference and prints the line; rank 1 exits 0 without
    work or output."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                        "--nproc-per-node", "2", "--master-addr", "127.0.0.1",
                        "--master-port", str(port), "bench.py", "--impl", "reference",
                        "--gpus", "2", "--workload", "c2", "--sample-n", "32", "--leaf-n", "64",
                        "--steps", "1",
                        "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["cpu_baseline"]["kind"] == "reference" and line["value"] > 0
