"""The reference's own CLI drives this path on the GPU.

oracle/_ref/mfft-bench-sm100 is the reference's exact-track driver
(src/main.c with its other sources, compiled where they lie by the `cli`
target of oracle/Makefile) linked against this repository's libmfftb200.so,
whose drop-in mm_mfft / mfft_plan_init / mfft_plan_init_rec replace
src/mfft.c.  With `--only mfft,mfft-rec` the driver runs every `mfft` and
`mfft-rec` row (one per leaf-kernel name each; the drop-in has one leaf, the
B200 path) on configs[0] -- n = 64, W = 8192, bigmat_rand inputs -- and
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
    r = subprocess.run([CLI, "--n", "64", "--width", "8192", "--only", "mfft,mfft-rec",
                        "--no-naive", "--csv"], capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    # method,kernel,products,kernel_calls,seconds,speedup,exact
    flat = [ln.split(",") for ln in r.stdout.splitlines() if ln.startswith("mfft,")]
    rec = [ln.split(",") for ln in r.stdout.splitlines() if ln.startswith("mfft-rec,")]
    assert len(flat) == 12 and len(rec) == 12, r.stdout[-2000:]
    assert all(row[6] == "yes" for row in flat + rec), r.stdout[-2000:]
    # the product counts of the reference's flat and recursive plans
    assert all(int(row[2]) == 65536 for row in flat)
    assert all(int(row[2]) == 15552 for row in rec)
