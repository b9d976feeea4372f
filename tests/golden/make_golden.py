"""Generate the golden fixtures in tests/golden/ by running the REFERENCE.

Every output here comes from the reference's own C (hadilq/mfft-bench
``src/*.c``) compiled from source into ``oracle/_ref`` by ``oracle/Makefile``
and called with its own signatures (``src/mfftbench.h``): ``bigmat_rand``,
``mm_mfft``, ``conv_mfft``, ``normalize_planes``, ``fpx_init`` /
``fpx_encode`` / ``fpx_decode_f32`` and ``fpx_init_d`` / ``fpx_encode_d`` /
``fpx_decode_f64``.  Inputs that the reference has no generator for (signed
integers, N(0,1)*2^k floats and doubles) come from the oracle's generators or
a seeded numpy generator and are stored in the fixture next to the outputs.

Run from the repository root:  python tests/golden/make_golden.py [--big]
(--big adds the n=1024 W=256 digests, unsigned through mm_mfft and signed
through conv_mfft + normalize_planes, ~100 s of reference CPU time each).
"""
import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle.oracle import Oracle, RefLib  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
SEED_A, SEED_B = 12345, 12345 ^ 0xABCDEF


def unsigned_case(r, o, n, L, store_full):
    A = r.bigmat_rand(n, L, SEED_A)
    B = r.bigmat_rand(n, L, SEED_B)
    t0 = time.time()
    out = r.mm_mfft(A, B, n, L)
    dt = time.time() - t0
    rec = {"n": n, "L": L, "RL": 2 * L + 1, "digest": f"{o.digest(out):016x}",
           "ref_seconds": round(dt, 4)}
    if store_full:
        np.savez_compressed(os.path.join(OUT, f"mm_mfft_u_n{n}_L{L}.npz"), A=A, B=B, out=out)
    return rec


def signed_case(r, o, n, L, kind):
    if kind == "int64":
        x = o.int64_entries(n, SEED_A)
        y = o.int64_entries(n, SEED_B)
        A, B = o.int64_to_planes(x, n), o.int64_to_planes(y, n)
    else:
        A, B = o.signed_planes(n, L, SEED_A), o.signed_planes(n, L, SEED_B)
    A32, B32 = o.signlimb(A, n, L), o.signlimb(B, n, L)
    cw = r.conv_mfft(A32, B32, n, L)
    out = r.normalize_planes(cw, 2 * L - 1, n, 2 * L + 1)
    np.savez_compressed(os.path.join(OUT, f"signed_n{n}_L{L}.npz"), A=A, B=B, A32=A32, B32=B32,
                        cw=cw, out=out)
    return {"n": n, "L": L, "RL": 2 * L + 1, "digest": f"{o.digest(out):016x}"}


def signed_digest_case(r, o, n, L):
    """configs[1]'s signed W=16L product, whole output, digest only: the
    reference's signed route (sign-limb int32 planes -> conv_mfft ->
    normalize_planes, two's complement output; src/mfft.c:302-422,
    src/bigmat.c:48-60)."""
    A, B = o.signed_planes(n, L, SEED_A), o.signed_planes(n, L, SEED_B)
    A32, B32 = o.signlimb(A, n, L), o.signlimb(B, n, L)
    t0 = time.time()
    cw = r.conv_mfft(A32, B32, n, L)
    out = r.normalize_planes(cw, 2 * L - 1, n, 2 * L + 1)
    dt = time.time() - t0
    return {"n": n, "L": L, "RL": 2 * L + 1, "digest": f"{o.digest(out):016x}",
            "ref_seconds": round(dt, 4), "full": False}


def fp32_case(r, o, n, force_bits):
    A, B = o.normal_f32(n, SEED_A)
    C, (L, SA, SB) = r.fp32_gemm(A, B, n, force_bits)
    np.savez_compressed(os.path.join(OUT, f"fp32_n{n}_w{force_bits}.npz"), A=A, B=B, C=C,
                        L=L, SA=SA, SB=SB)
    return {"n": n, "force_bits": force_bits, "L": L, "SA": SA, "SB": SB,
            "digest_f32": f"{o.digest(C.view(np.uint16)):016x}"}


def fp64_case(r, o, n, force_bits, tag, lo_k, hi_k, seed):
    rng = np.random.default_rng(seed)
    A = rng.standard_normal(n * n) * np.exp2(rng.integers(lo_k, hi_k + 1, n * n))
    B = rng.standard_normal(n * n) * np.exp2(rng.integers(lo_k, hi_k + 1, n * n))
    A[::13] = 0.0
    B[5::17] = -0.0
    A[7] = np.inf
    B[11] = np.nan
    C, (L, SA, SB) = r.fp64_gemm(A, B, n, force_bits)
    np.savez_compressed(os.path.join(OUT, f"fp64_n{n}_w{force_bits}{tag}.npz"), A=A, B=B, C=C,
                        L=L, SA=SA, SB=SB)
    return {"n": n, "force_bits": force_bits, "tag": tag, "L": L, "SA": SA, "SB": SB,
            "digest_f64": f"{o.digest(C.view(np.uint16)):016x}"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--big", action="store_true")
    args = ap.parse_args()
    r, o = RefLib(), Oracle()
    meta = {"generator": "tests/golden/make_golden.py", "reference_lib": os.path.basename(r.path),
            "seeds": [SEED_A, SEED_B], "digest": "FNV-1a over uint16 words, plane-major",
            "unsigned": [], "signed": [], "fp32": [], "fp64": []}
    for n, L, full in ((8, 8, True), (16, 64, True), (48, 16, True), (64, 512, False)):
        meta["unsigned"].append(unsigned_case(r, o, n, L, full))
    if args.big:
        meta["unsigned"].append(unsigned_case(r, o, 1024, 16, False))
    for n, L, kind in ((32, 4, "int64"), (64, 4, "int64"), (48, 16, "planes")):
        meta["signed"].append(signed_case(r, o, n, L, kind))
    if args.big:
        meta["signed"].append(signed_digest_case(r, o, 1024, 16))
    for n, fb in ((64, 512), (64, 0), (96, 512)):
        meta["fp32"].append(fp32_case(r, o, n, fb))
    # fp64: the 512-bit grid, the adaptive grid, and an adaptive case whose
    # products fall into the subnormal range of binary64
    for n, fb, tag, lo_k, hi_k, seed in ((64, 512, "", -8, 8, 1), (64, 0, "", -30, 30, 2),
                                         (48, 0, "_tiny", -560, -530, 3)):
        meta["fp64"].append(fp64_case(r, o, n, fb, tag, lo_k, hi_k, seed))
    old = {}
    path = os.path.join(OUT, "golden.json")
    if os.path.exists(path):
        with open(path) as f:
            old = json.load(f)
    # keep a previously recorded --big digest when re-running without --big
    for kind in ("unsigned", "signed"):
        have = {(c["n"], c["L"]) for c in meta[kind]}
        for c in old.get(kind, []):
            if (c["n"], c["L"]) not in have:
                meta[kind].append(c)
    with open(path, "w") as f:
        json.dump(meta, f, indent=1)
    print(json.dumps(meta, indent=1))


if __name__ == "__main__":
    main()
