"""The drop-in API from C: tests/c_dropin/dropin_c1.c includes only
include/mfftbench_b200.h and links only libmfftb200.so.  Without a GPU the
program must compile and link against the header's declarations; on a B200
it must reproduce the reference's own c1 digest (tests/golden, from the
reference's mm_mfft) with mm_mfft and agree with mm_limbplane."""
import os
import re
import subprocess

import pytest

import mfft_bench_b200 as m

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_dropin", "dropin_c1.c")


def _build(tmp_path):
    exe = str(tmp_path / "dropin_c1")
    libdir = os.path.dirname(m.LIB_PATH)
    r = subprocess.run(["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-I",
                        os.path.join(ROOT, "include"), SRC, "-L", libdir, "-lmfftb200",
                        "-Wl,-rpath," + libdir, "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_program_compiles_and_links(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_c_program_reproduces_reference_digest(tmp_path, golden):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, (r.returncode, r.stderr)
    got = re.search(r"digest ([0-9a-f]{16})", r.stdout).group(1)
    rec = next(c for c in golden["unsigned"] if c["n"] == 64 and c["L"] == 512)
    assert got == rec["digest"]
