"""The reference's own CLI drives this path on the GPU.

oracle/_ref/mfft-bench-sm100 is the reference's exact-track driver
(src/main.c with its other sources, compiled where they lie by the `cli`
target of oracle/Makefile) linked against this repository's libmfftb200.so,
whose drop-in mm_mfft replaces src/mfft.c.  With `--only mfft` the driver
runs every `mfft` row (one per leaf-kernel name; the drop-in has one leaf,
the B200 path) on configs[0] -- n = 64, W = 8192, bigmat_rand inputs -- and
checks each output against its own textbook product mm_bigint_ijk
(src/main.c:125-131, src/methods.c:22-52), about 15 s of CPU time.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLI = os.path.join(ROOT, "oracle", "_ref", "mfft-bench-sm100")


def test_reference_cli_verifies_the_gpu_path():
    if not os.path.exists(CLI):
        pytest.skip("oracle/_ref/mfft-bench-sm100 not built (needs the reference sources)")
    r = subprocess.run([CLI, "--n", "64", "--width", "8192", "--only", "mfft", "--no-naive",
                        "--csv"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    rows = [ln.split(",") for ln in r.stdout.splitlines() if ln.startswith("mfft,")]
    assert len(rows) == 12, r.stdout[-2000:]
    # method,kernel,products,kernel_calls,seconds,speedup,exact
    assert all(row[6] == "yes" for row in rows), r.stdout[-2000:]
    assert all(int(row[2]) == 65536 for row in rows)  # the reference plan's product count
