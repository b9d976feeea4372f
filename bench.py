#!/usr/bin/env python3
"""bench.py -- seconds per exact n x n W-bit integer matmul on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c5]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)
    python bench.py --impl reference ...                      (reference CPU arm)

Metric: "s per exact n x n W-bit matmul; effective int8 TOPS vs tcgen05 int8
peak".  One step = one exact product of the workload's two matrices (inputs
resident in HBM, device-timed with CUDA events on the launching stream, max
over ranks).  The default workload is c5 (n=16384, W=64 signed, the headline
configuration); the other benchmark configurations are selectable with
--workload c1..c4, plus f64 (the fp64 embedding on c4's shape).

Also reported on the same JSON line: the live roofline of the dominant kernel
(the tcgen05 pointwise contraction), an end-to-end number through the C ABI
with host buffers (H2D + compute + D2H every step), the reference CPU
baseline timed on a bounded sample, SM clocks sampled during the timed
region and the number of our kernel launches.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEED_A, SEED_B = 12345, 12345 ^ 0xABCDEF
RL_OF = lambda L: 2 * L + 1  # noqa: E731

WORKLOADS = {
    "c1": dict(n=64, kind="u16", L=512, signed=False,
               desc="configs[0]: n=64, W=8192 unsigned (bigmat_rand)"),
    "c2": dict(n=1024, kind="u16", L=16, signed=True,
               desc="configs[1]: n=1024, W=256 signed two's complement"),
    "c3": dict(n=4096, kind="u16", L=64, signed=False,
               desc="configs[2]: n=4096, W=1024 unsigned (bigmat_rand)"),
    "c4": dict(n=8192, kind="f32", force_bits=512,
               desc="configs[3]: n=8192 fp32 N(0,1)*2^k on the 512-bit grid"),
    "c5": dict(n=16384, kind="i64", signed=True,
               desc="configs[4]: n=16384, W=64 signed int64"),
    # not one of the benchmark configurations c1-c5: the fp64 embedding
    # (fpx_*_d) on c4's shape
    "f64": dict(n=8192, kind="f64", force_bits=512,
                desc="fp64 N(0,1)*2^k (k in [-8, 8]) on the 512-bit grid, n=8192"),
}
DEFAULT_N = {k: v["n"] for k, v in WORKLOADS.items()}


def normal_f64(n, seed):
    """The f64 workload's inputs: N(0,1) * 2^k, k uniform in [-8, 8]."""
    import numpy as np
    rng = np.random.default_rng(seed)
    A = rng.standard_normal(n * n) * np.exp2(rng.integers(-8, 9, n * n))
    B = rng.standard_normal(n * n) * np.exp2(rng.integers(-8, 9, n * n))
    return A, B

METRIC = "s per exact n x n W-bit matmul; effective int8 TOPS vs tcgen05 int8 peak"
SUBBLOCKS = 1
C_GATHER = "peer"


# ---------------------------------------------------------------------------- helpers
def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


# DRAM bytes (read + write) of one plane-product launch (one row block), from
# a one-pass ncu capture of dram__bytes_read.sum / dram__bytes_write.sum on
# the full workload (one pass checked on n = 4096 first), keyed by workload,
# kernel (3 t-grouped, 4 Karatsuba) and Karatsuba level.
POINTWISE_TRAFFIC = {
    ("c5", 4, 3): {"bytes_per_launch": 152.18e9 + 39.55e9,
                   "note": ("ncu, the second launch of a 1-GPU product (a row block of 3328 rows "
                            "x 16384 columns), level-3 Karatsuba kernel (two 96 KB stages): "
                            "152.2 GB read + 39.6 GB written in 148.0 ms; algorithmic: 144 A "
                            "operand planes of the block + 144 B operand planes (46.5 GB) read, "
                            "180 int32 job planes per element of the block (39.3 GB) written")},
    ("c5", 4, 2): {"bytes_per_launch": 197.62e9 + 45.51e9,
                   "note": ("ncu, the second launch of a 1-GPU product (a row block of 4096 rows "
                            "x 16384 columns), two-level Karatsuba kernel: 197.6 GB read + "
                            "45.5 GB written in 210.5 ms; algorithmic: 128 A operand planes of "
                            "the block + 128 B operand planes (43.0 GB) read, 168 int32 job "
                            "planes per element of the block (45.1 GB) written")},
    ("c5", 4, 1): {"bytes_per_launch": 310.06e9 + 52.87e9,
                   "note": ("ncu, the second launch of a 1-GPU product (a row block of the "
                            "plan's rblock rows x 16384 columns), one-level Karatsuba kernel: "
                            "310.1 GB read + "
                            "52.9 GB written in 363 ms; algorithmic: 96 A operand planes of the "
                            "block + 96 B operand planes (about 34 GB) read, 140 int32 job "
                            "planes per element of the block written")},
    ("c5", 3, 0): {"bytes_per_launch": 848.51e9 + 52.15e9,
                   "note": ("ncu, first row block of a 1-GPU product (11136 of 16384 rows), "
                            "t-grouped kernel with the half-point terms skipped: 848.5 GB read + "
                            "52.2 GB written; algorithmic operand bytes of that launch 43.9 GB "
                            "read + 46.7 GB of int32 job planes written")},
}

PW_KERNELS = {1: "pointwise_i8_kernel (tcgen05 kind::i8, one CTA per tile)",
              2: "pointwise2_i8_kernel (tcgen05 cta_group::2 kind::i8)",
              3: "pointwise3_i8_kernel (tcgen05 cta_group::2 kind::i8, 4 t-jobs per tile)",
              4: "pointwise_kara_i8_kernel (tcgen05 cta_group::2 kind::i8, Karatsuba: 3 "
                 "length-4 convolutions per point, at levels 2 and 3 each of the first two, "
                 "or all three, as 3 length-2 convolutions)"}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_count():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------- reference CPU work
# A full-size reference product takes hours at c3-c5 (about 14 h, 28 h and
# 14 h on one core), so its time is projected from two measured parts: one
# product is `calls` independent n x n mm_accum leaves (the plan's NB*K^2
# pointwise products, src/mfft.c:383-396; L^2 for the limb-plane schoolbook)
# plus O(L n^2) pack / transform / fold / normalize phases.  The phases are
# measured by running the reference's whole path at CPU_PHASE_N and
# subtracting its leaves; one leaf is timed at CPU_LEAF_N (n^3 scaling above
# it).  projected(n) = phases * (n/n_phase)^2 + calls * leaf * (n/n_leaf)^3.
CPU_PHASE_N = {"c1": 64, "c2": 256, "c3": 128, "c4": 256, "c5": 512, "f64": 256}
CPU_LEAF_N = {"c1": 64, "c2": 1024, "c3": 2048, "c4": 2048, "c5": 2048, "f64": 2048}


def _ref_path_sample(workload, n_s, method="mfft"):
    """Run the reference's own CPU hot path (oracle/_ref, compiled from the
    reference sources) once on an n_s sample of the workload; returns
    (seconds of the reference's timed region, leaf mm_accum calls).  The
    timed region is the product (encode/decode excluded as in
    src/mlgemm.c:1103-1106).  method "schoolbook" times the reference's
    limb-plane comparator (conv_limbplane / mm_limbplane, src/methods.c:94-123)
    instead of its MFFT."""
    import ctypes as C

    import numpy as np
    from oracle.oracle import Oracle, RefLib
    r, o = RefLib(), Oracle()
    calls = C.c_longlong.in_dll(r.lib, "g_kernel_calls")
    w = WORKLOADS[workload]
    if w["kind"] in ("u16", "i64"):
        L = w.get("L", 4)
        if w["kind"] == "i64":
            A = o.int64_to_planes(o.int64_entries(n_s, SEED_A), n_s)
            B = o.int64_to_planes(o.int64_entries(n_s, SEED_B), n_s)
        elif w["signed"]:
            A, B = o.signed_planes(n_s, L, SEED_A), o.signed_planes(n_s, L, SEED_B)
        else:
            A, B = r.bigmat_rand(n_s, L, SEED_A), r.bigmat_rand(n_s, L, SEED_B)
        signed = w["kind"] == "i64" or w["signed"]
        if signed:
            A32, B32 = o.signlimb(A, n_s, L), o.signlimb(B, n_s, L)
        calls.value = 0
        t0 = time.perf_counter()
        if signed:  # conv + normalize_planes (the reference's signed route)
            if method == "schoolbook":
                cw = np.zeros((2 * L - 1) * n_s * n_s, np.int64)
                r.lib.conv_limbplane(cw, A32, B32, n_s, L, 2)
            else:
                cw = r.conv_mfft(A32, B32, n_s, L)
            r.normalize_planes(cw, 2 * L - 1, n_s, RL_OF(L))
        elif method == "schoolbook":
            r.mm_limbplane(A, B, n_s, L)
        else:
            r.mm_mfft(A, B, n_s, L)
        return time.perf_counter() - t0, int(calls.value)
    from oracle.oracle import RefFpx
    c = RefFpx()
    if w["kind"] == "f64":
        A, B = normal_f64(n_s, SEED_A)
        r.lib.fpx_init_d(C.byref(c), A, B, n_s, w["force_bits"])
        r.lib.fpx_encode_d(C.byref(c), A, B)
    else:
        A, B = o.normal_f32(n_s, SEED_A)
        r.lib.fpx_init(C.byref(c), A, B, n_s, w["force_bits"])
        r.lib.fpx_encode(C.byref(c), A, B)
    nn = n_s * n_s
    A32 = np.ctypeslib.as_array(c.A32, shape=(c.L * nn,))
    B32 = np.ctypeslib.as_array(c.B32, shape=(c.L * nn,))
    cw = np.ctypeslib.as_array(c.Cw, shape=((2 * c.L - 1) * nn,))
    plan = r.plan(c.L)
    calls.value = 0
    t0 = time.perf_counter()
    if method == "schoolbook":
        r.lib.conv_limbplane(cw, A32, B32, n_s, c.L, 2)
    else:
        r.lib.conv_mfft(cw, A32, B32, n_s, c.L, C.byref(plan), 2)
    t = time.perf_counter() - t0
    r.lib.fpx_free(C.byref(c))
    return t, int(calls.value)


def _ref_leaf_seconds(args):
    """One reference leaf: mm_accum(KERNEL_PACKED) (src/kernel.c:1015-1033)
    of n x n int32 planes holding 16-bit limb magnitudes, as the MFFT's
    transformed planes do; returns its seconds."""
    n, seed = args
    import numpy as np
    from oracle.oracle import KERNEL_PACKED, RefLib
    r = RefLib()
    g = np.random.default_rng(seed)
    A = g.integers(-65535, 65536, n * n, dtype=np.int32)
    B = g.integers(-65535, 65536, n * n, dtype=np.int32)
    Cc = np.zeros(n * n, np.int64)
    t0 = time.perf_counter()
    r.lib.mm_accum(Cc, A, B, n, 1, KERNEL_PACKED)
    return time.perf_counter() - t0


def _ref_whole_seconds(args):
    workload, n, method = args
    return _ref_path_sample(workload, n, method)[0]


class RefProjection:
    """The reference's CPU path projected to the workload's full size, on one
    core and on `cores` cores.  The reference path is single-threaded
    (mm_packed has no OpenMP, conv_mfft is serial), so `cores` cores run
    `cores` independent products at once: the all-core figure is the
    throughput-equivalent seconds per product, with every leaf timed while
    `cores` leaves run concurrently (shared caches and memory bandwidth)."""

    def __init__(self, workload, method, cores):
        w = WORKLOADS[workload]
        self.workload, self.method, self.cores = workload, method, cores
        self.n = w["n"]
        self.n_s = min(CPU_PHASE_N[workload], self.n)
        self.n_l = min(CPU_LEAF_N[workload], self.n)
        # the full size runs whole (c1): the measured path is the value, and
        # the concurrent rounds run whole paths instead of leaves
        self.whole = self.n_s == self.n
        t_path, self.calls = _ref_path_sample(workload, self.n_s, method)
        self.t_path = t_path
        if self.whole:
            self.phases, self.leaf_single = 0.0, t_path
            return
        leaf_s = min(_ref_leaf_seconds((self.n_s, 1)) for _ in range(2))
        self.phases = max(0.0, t_path - self.calls * leaf_s)
        self.leaf_single = _ref_leaf_seconds((self.n_l, 2))

    def value(self, leaf):
        if self.whole:
            return leaf
        return (self.phases * (self.n / self.n_s) ** 2
                + self.calls * leaf * (self.n / self.n_l) ** 3)

    def concurrent_leaf(self, pool):
        if self.whole:
            ts = pool.map(_ref_whole_seconds, [(self.workload, self.n, self.method)] * self.cores)
        else:
            ts = pool.map(_ref_leaf_seconds, [(self.n_l, 3 + i) for i in range(self.cores)])
        return statistics.mean(ts)

    def describe(self, leaf_conc):
        what = "limb-plane schoolbook" if self.method == "schoolbook" else "MFFT path"
        if self.whole:
            return (f"measured: reference {what} (oracle/_ref, packed leaf) run whole at n={self.n}: "
                    f"{self.t_path:.3f} s alone, {leaf_conc:.3f} s with {self.cores} copies running "
                    f"concurrently; the all-core value is {self.cores} concurrent single-threaded "
                    f"products (the reference path is single-threaded) divided by {self.cores}")
        return (f"projected: reference {what} (oracle/_ref, packed leaf) = phases measured at "
                f"n={self.n_s} ({self.phases:.3f} s) x (n/{self.n_s})^2 + {self.calls} leaves x "
                f"one mm_accum at n={self.n_l} x (n/{self.n_l})^3; leaf alone "
                f"{self.leaf_single:.3f} s, with {self.cores} leaves running concurrently "
                f"{leaf_conc:.3f} s; the all-core value is {self.cores} concurrent single-threaded "
                f"products (the reference path is single-threaded) divided by {self.cores}")


def reference_line(args):
    """--impl reference: the reference's CPU path on all host cores; every
    step is one round of T concurrent leaf timings (one per core) feeding the
    projection above."""
    import multiprocessing as mp
    w = WORKLOADS[args.workload]
    T = cpu_count()
    proj = RefProjection(args.workload, args.method, T)
    ctx = mp.get_context("spawn")
    rounds, leaves = [], []
    with ctx.Pool(T) as pool:
        for step in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            leaf = proj.concurrent_leaf(pool)
            dt = time.perf_counter() - t0
            if step >= args.warmup:
                rounds.append(dt)
                leaves.append(leaf)
    leaf = statistics.mean(leaves)
    value = proj.value(leaf) / T
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": statistics.mean(rounds) * 1e3, "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "int64", "data": "synthetic",
            "config": {"workload": args.workload, "desc": w["desc"], "n": w["n"],
                       "phase_n": proj.n_s, "leaf_n": proj.n_l, "method": args.method},
            "cpu_baseline": {"value": value, "unit": "s", "cores": T, "kind": "reference",
                             "projected": not proj.whole, "sample": proj.describe(leaf),
                             "single_thread_value": proj.value(proj.leaf_single)},
            "e2e": {"value": value, "unit": "s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_line(workload, method):
    """The headline line's cpu_baseline: the same projection on all host
    cores, plus the one-core figure."""
    import multiprocessing as mp
    T = cpu_count()
    proj = RefProjection(workload, method, T)
    with mp.get_context("spawn").Pool(T) as pool:
        leaf = proj.concurrent_leaf(pool)
    return {"value": proj.value(leaf) / T, "unit": "s", "cores": T, "kind": "reference",
            "projected": not proj.whole, "sample": proj.describe(leaf),
            "single_thread_value": proj.value(proj.leaf_single)}


# ---------------------------------------------------------------------------- B200 arm
class Workload:
    """Device-resident inputs and one exact product per step.

    With world > 1, rank r owns rows [r0, r1) of A, B and C (row-block
    sharding).  Each step all-gathers B from the ranks' row blocks, computes
    this rank's rows of C, and gathers C's rows to rank 0 in the reference's
    plane-major layout."""

    def __init__(self, name, ctx, torch, rank, world, device):
        from mfft_bench_b200 import dist as D
        self.name, self.w = name, WORKLOADS[name]
        self.ctx, self.torch, self.rank, self.world = ctx, torch, rank, world
        w = self.w
        n = self.n = w["n"]
        self.ranges = D.all_ranges(n, world)
        self.r0, self.r1 = self.ranges[rank]
        self.rows = self.r1 - self.r0
        dev = device
        if w["kind"] == "i64":
            self.RL, self.planes, self.bytes_in = 9, 1, 8
            A = torch.empty(n * n, dtype=torch.int64, device=dev)
            B = torch.empty(n * n, dtype=torch.int64, device=dev)
            ctx.gen_int64(A, SEED_A)
            ctx.gen_int64(B, SEED_B)
        elif w["kind"] == "u16":
            L = w["L"]
            self.RL, self.planes, self.bytes_in = RL_OF(L), L, 2 * L
            A = torch.empty(L * n * n, dtype=torch.uint16, device=dev)
            B = torch.empty(L * n * n, dtype=torch.uint16, device=dev)
            ctx.gen_bigmat(A, n, L, SEED_A)
            ctx.gen_bigmat(B, n, L, SEED_B)
        elif w["kind"] == "f64":
            self.RL, self.planes, self.bytes_in = 1, 1, 8
            hA, hB = normal_f64(n, SEED_A)
            A = torch.from_numpy(hA).to(dev)
            B = torch.from_numpy(hB).to(dev)
        else:
            from mfft_bench_b200 import gen_normal_f32
            self.RL, self.planes, self.bytes_in = 1, 1, 4
            hA, hB = gen_normal_f32(n, SEED_A)
            A = torch.from_numpy(hA).to(dev)
            B = torch.from_numpy(hB).to(dev)
        ctx.sync()
        self.A, self.B = A, B
        # this rank's row block of every B plane (what it owns before the gather)
        P = self.planes
        self.B_local = B.view(P, n, n)[:, self.r0:self.r1, :].contiguous().view(-1) \
            if world > 1 else None
        odt = {"f32": torch.float32, "f64": torch.float64}.get(w["kind"], torch.uint16)
        self.out = torch.empty(max(1, self.RL * self.rows * n), dtype=odt, device=dev)
        # C's rows reach rank 0 either through a CUDA IPC mapping of its
        # output buffer, written by every rank's final kernel (the default:
        # compute and gather in one step), or by NCCL point-to-point transfers
        self.peer = None
        if world > 1 and C_GATHER == "peer" and SUBBLOCKS == 1:
            self.peer = D.PeerOutput(self.RL * n * n, str(odt).replace("torch.", ""))
            self.full_out = self.peer.tensor
            self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
        else:
            self.full_out = self.out if world == 1 else (
                torch.empty(self.RL * n * n, dtype=odt, device=dev) if rank == 0 else None)
        # optionally (--subblocks > 1) a rank computes its rows in sub-blocks
        # and ships each one to rank 0 while the next computes (B is transformed
        # once per step).  Off by default: NCCL's copy kernels then share the
        # SMs with the persistent pointwise kernel, which cost more than the
        # overlap saved on 8 GPUs.
        self.subs = D.plan_subblocks(self.ranges, SUBBLOCKS if world > 1 else 1)
        self.nsub = len(self.subs[0])
        self.sub_out = []
        off = 0
        for a, b in self.subs[rank]:
            cnt = self.RL * (b - a) * n
            self.sub_out.append(self.out[off:off + cnt])
            off += cnt

    def gather_B(self):
        from mfft_bench_b200 import dist as D
        P, n = self.planes, self.n
        rows = self.rows
        Bv = self.B.view(P, n * n)
        for u in range(P):
            loc = self.B_local.view(P, rows * n)[u] if rows else self.B_local[:0]
            D.allgather_rows(self._as_gatherable(loc), self._as_gatherable(Bv[u]), n, self.ranges)

    def _as_gatherable(self, t):
        # NCCL has no uint16: move 16-bit limbs as int16 (same bytes)
        return t.view(self.torch.int16) if t.dtype == self.torch.uint16 else t

    def step(self):
        """One product; sharded across ranks when world > 1."""
        from mfft_bench_b200 import dist as D
        w, ctx, n = self.w, self.ctx, self.n
        if self.world == 1:
            self._compute((self.r0, self.r1), self.out)
            return
        self.gather_B()
        if self.peer is not None:
            # this rank's rows of every plane straight into rank 0's buffer
            ctx.set_reuse_b(False)
            self._compute((self.r0, self.r1), self.peer.ptr + self.r0 * n * self.out.element_size(),
                          plane_stride=n * n)
            # stream-ordered completion: each rank's all-reduce starts after
            # its final kernel (NCCL's stream waits on this one), and rank 0's
            # stream continues only after every rank's all-reduce -- so after
            # every rank's stores -- with no host synchronisation in the step
            self.torch.distributed.all_reduce(self.flag)
            return
        works = []
        for si in range(self.nsub):
            a, b = self.subs[self.rank][si]
            ctx.set_reuse_b(si > 0)  # B is packed/transformed on the first sub-block of each step
            self._compute((a, b), self.sub_out[si])
            seg = [self.subs[r][si] for r in range(self.world)]
            works += D.gather_sub_to_root_async(self.sub_out[si], self.full_out, n, self.RL, seg)
        ctx.set_reuse_b(False)
        for wk in works:
            wk.wait()

    def _compute(self, rows, out, plane_stride=0):
        w, ctx, n = self.w, self.ctx, self.n
        ctx.set_output_plane_stride(plane_stride)
        if w["kind"] == "i64":
            ctx.mm_i64(self.A, self.B, n, RL=self.RL, out=out, rows=rows)
        elif w["kind"] == "u16":
            ctx.mm_u16(self.A, self.B, n, w["L"], signed=w["signed"], RL=self.RL, out=out,
                       rows=rows)
        elif w["kind"] == "f64":
            ctx.fp64(self.A, self.B, n, w["force_bits"], out=out, rows=rows)
        else:
            ctx.fp32(self.A, self.B, n, w["force_bits"], out=out, rows=rows)


def cublas_int8_sustained(torch, stream, seconds=2.0, n=8192):
    """Same-run context for the power-capped roofline: cuBLASLt int8 GEMM
    (torch._int_mm, int8 x int8 -> int32) run back to back for `seconds`,
    timed with CUDA events.  A library GEMM, used only as a yardstick."""
    try:
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t().contiguous().t()
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        iters = 0
        e0.record(stream)
        while time.perf_counter() - t0 < seconds:
            for _ in range(20):
                torch._int_mm(a, b)
            iters += 20
            torch.cuda.synchronize()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        return 2.0 * n ** 3 * iters / (ms * 1e-3) / 1e12
    except Exception:
        return None


def accuracy_vs_fp64(wl, torch):
    """fp32 workloads: the product (one exact result, rounded once to fp32)
    against an fp64 GEMM of the same fp32 inputs (torch.matmul in float64,
    cuBLAS dgemm), and a plain fp32 GEMM (TF32 off) against the same, for
    context.  rel_err_fro is the reference's rel_err (src/mlgemm.c:563-571):
    sqrt(sum (C - R)^2 / sum R^2); max_rel_err is max |C - R| / |R| over the
    entries with R != 0."""
    n = wl.n
    A = wl.A.view(n, n)
    B = wl.B.view(n, n)
    R = A.double() @ B.double()
    C = wl.full_out.view(n, n).double()
    nz = R != 0

    def errs(X):
        d = X - R
        fro = float((d.square().sum() / R.square().sum()).sqrt())
        mx = float((d.abs()[nz] / R.abs()[nz]).max())
        return fro, mx

    fro, mx = errs(C)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    S = (A @ B).double()
    torch.backends.cuda.matmul.allow_tf32 = tf32
    sfro, smx = errs(S)
    same = float((wl.full_out.view(n, n) == R.float()).double().mean())
    del R, C, S
    torch.cuda.empty_cache()
    return {"vs": "fp64 GEMM (cuBLAS dgemm) of the same fp32 inputs",
            "max_rel_err_vs_fp64": mx, "rel_err_fro_vs_fp64": fro,
            "share_equal_to_fp64_rounded_to_fp32": same,
            "fp32_sgemm_max_rel_err_vs_fp64": smx, "fp32_sgemm_rel_err_fro_vs_fp64": sfro}


def e2e_measure(ctx, wl, steps, torch):
    """The same product through the host-pointer C ABI (one GPU): pinned host
    inputs, H2D + compute + D2H inside the timed region every step."""
    w, n = wl.w, wl.n
    hA = wl.A.cpu().pin_memory()
    hB = wl.B.cpu().pin_memory()
    hout = torch.empty(wl.RL * n * n, dtype=wl.out.dtype).pin_memory()

    def u16(t):
        return t.view(torch.int16).numpy().view("uint16")

    def run():
        if w["kind"] == "i64":
            ctx.mm_i64(hA.numpy(), hB.numpy(), n, RL=wl.RL, out=hout.numpy())
        elif w["kind"] == "u16":
            ctx.mm_u16(u16(hA), u16(hB), n, w["L"], signed=w["signed"], RL=wl.RL, out=u16(hout))
        elif w["kind"] == "f64":
            ctx.fp64(hA.numpy(), hB.numpy(), n, w["force_bits"], out=hout.numpy())
        else:
            ctx.fp32(hA.numpy(), hB.numpy(), n, w["force_bits"], out=hout.numpy())

    run()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        run()
        ts.append(time.perf_counter() - t0)
    h2d = 2 * n * n * wl.bytes_in
    d2h = wl.RL * n * n * wl.out.element_size()
    return {"value": statistics.mean(ts), "unit": "s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps}


def e2e_measure_dist(wl, steps, torch, dist, device):
    """N GPUs: every rank copies its own row blocks of A and B from pinned
    host memory, B is all-gathered, the rank computes its rows of C and reads
    them back into its own pinned host buffer over its own PCIe link (all N
    links busy at once; C's rows are not funnelled through rank 0).  Also
    reported: the same step with C gathered to rank 0 on the GPUs and read
    back by rank 0 alone.  Time = max over ranks of the mean step."""
    n, P = wl.n, wl.planes
    rows = wl.rows
    Av = wl.A.view(P, n, n)
    hA = Av[:, wl.r0:wl.r1, :].contiguous().cpu().pin_memory()
    hB = wl.B_local.cpu().pin_memory()
    hrows = torch.empty(max(1, wl.RL * rows * n), dtype=wl.out.dtype).pin_memory()
    hout = torch.empty(wl.RL * n * n, dtype=wl.out.dtype).pin_memory() if wl.rank == 0 else None

    def upload():
        Av[:, wl.r0:wl.r1, :].copy_(hA.view(P, rows, n).to(device, non_blocking=True))
        wl.B_local.copy_(hB.to(device, non_blocking=True))

    def run_local():
        upload()
        wl.gather_B()
        wl._compute((wl.r0, wl.r1), wl.out)
        hrows.copy_(wl.out[:hrows.numel()], non_blocking=True)
        torch.cuda.synchronize()

    def run_root():
        upload()
        wl.step()
        if wl.rank == 0:
            hout.copy_(wl.full_out, non_blocking=True)
        torch.cuda.synchronize()

    def timed(fn):
        fn()
        ts = []
        for _ in range(steps):
            dist.barrier()
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        t = torch.tensor([statistics.mean(ts)], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    local, root = timed(run_local), timed(run_root)
    h2d = 2 * n * n * wl.bytes_in
    d2h = wl.RL * n * n * wl.out.element_size()
    return {"value": local, "unit": "s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "note": ("each rank uploads its row blocks of A and B and reads back its own "
                     "rows of C (plane-major [RL][rows][n]) over its own PCIe link; "
                     "bytes are totals over all ranks"),
            "value_gather_to_rank0": root}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="c5", choices=sorted(WORKLOADS))
    ap.add_argument("--n", type=int, default=0,
                    help="override the workload's matrix size (small profiling cases)")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-int8-ref", action="store_true")
    ap.add_argument("--subblocks", type=int, default=1,
                    help="row sub-blocks per rank whose gathers overlap the next block's compute")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--c-gather", default="peer", choices=["peer", "nccl"],
                    help="N > 1: C's rows reach rank 0 through stores of every rank's final "
                         "kernel into an IPC mapping of rank 0's buffer (peer) or through NCCL "
                         "point-to-point transfers after the compute (nccl)")
    ap.add_argument("--sample-n", type=int, default=0,
                    help="matrix size of the reference CPU phase sample (default: per workload)")
    ap.add_argument("--leaf-n", type=int, default=0,
                    help="matrix size of the timed reference leaf (default: per workload)")
    ap.add_argument("--method", default="mfft", choices=["mfft", "schoolbook"],
                    help="mfft: the MFFT hot path (the headline); schoolbook: the limb-plane "
                         "comparator on the same tensor-core kernel")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.sample_n > 0:
        CPU_PHASE_N[args.workload] = args.sample_n
    if args.leaf_n > 0:
        CPU_LEAF_N[args.workload] = args.leaf_n
    global SUBBLOCKS, C_GATHER
    SUBBLOCKS = max(1, args.subblocks)
    C_GATHER = args.c_gather
    if args.n > 0:
        WORKLOADS[args.workload] = dict(WORKLOADS[args.workload], n=args.n)

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)

    if args.impl == "reference":
        if rank == 0:
            reference_line(args)
        return

    import torch
    import torch.distributed as dist

    import mfft_bench_b200 as m

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    stream = torch.cuda.current_stream()
    ctx = m.Context(local_rank, stream=stream)
    ctx.set_method(args.method)
    wl = Workload(args.workload, ctx, torch, rank, world, device)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        wl.step()
    ctx.sync()
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    ctx.set_profile(2)  # per-kernel events, recorded without host syncs
    launches_per_step = None
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        wl.step()
        if launches_per_step is None:
            launches_per_step = ctx.launches()
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ctx.sync()
    ms = t_start.elapsed_time(t_end) / args.steps
    ph = ctx.phase_ms()
    if ctx.phase_dropped():  # per-kernel times must cover every timed launch
        raise RuntimeError(f"{ctx.phase_dropped()} launches past the profile's capacity; "
                           "time fewer steps")
    ctx.set_profile(0)
    if world > 1:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    n = wl.n
    w = WORKLOADS[args.workload]
    pi = ctx.last_plan()
    peaks, peak_kind = load_peaks()
    # Denominator of the tensor roofline: the dense tcgen05 kind::i8 rate,
    # 8192 int8 MACs per SM per clock (B200's nominal 4.5 dense int8 POPS is
    # that rate over 148 SMs at about 1.86 GHz), times the SMs, times the
    # median SM clock sampled during the timed region -- the power cap, not
    # the kernel, sets that clock.  Side numbers: twice the measured bf16
    # cuBLAS rates of MEASURED_PEAKS.json (kind::i8 issues twice the MACs per
    # clock of kind::f16), burst and sustained.
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    clk_mhz = clk.get("sm_mhz") or clk.get("sm_max_mhz") or 1965.0
    peak_int8 = 2.0 * 8192 * sms * clk_mhz * 1e6 / 1e12
    peak_2x_sus = 2.0 * float(peaks.get("bf16_tflops_sustained", 1400.0))
    peak_2x_burst = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    line = {"metric": METRIC, "value": ms / 1e3, "unit": "s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8",
            "data": ("synthetic (seeded numpy PCG64 N(0,1)*2^k)" if w["kind"] == "f64" else
                     "synthetic (seeded splitmix64, reference generators)"),
            "config": {"workload": args.workload, "desc": w["desc"], "n": n, "method": args.method,
                       "parallelism": (f"row-blocks x{world}, C rows to rank 0 by "
                                       + ("stores of the final kernel into a peer mapping"
                                          if wl.peer is not None else "NCCL point-to-point"))
                                      if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (no flush needed)"},
            "gpu_launches": (launches_per_step or 0) * args.steps,
            "clocks": clk}
    if True:
        macs = pi.get("int8_macs")
        pw_ms = ph["pointwise"] / args.steps
        if macs:
            macs_rank = macs * (wl.rows / n)
            achieved = 2 * macs_rank / (pw_ms * 1e-3) / 1e12
            useful_rank = pi["schoolbook7_macs"] * (wl.rows / n)
            useful = 2 * useful_rank / (pw_ms * 1e-3) / 1e12
            line["roofline"] = {
                "bound": "tensor", "kernel": PW_KERNELS.get(pi.get("pw_kernel"), "unknown"),
                "achieved": achieved, "peak": peak_int8, "unit": "TFLOP/s",
                "frac": achieved / peak_int8, "traffic": None,
                "peak_basis": (f"dense tcgen05 kind::i8: 8192 MACs/SM/clock x {sms} SMs x "
                               f"{clk_mhz:.0f} MHz (median SM clock sampled during the timed "
                               f"region)"),
                "ops_per_step": 2 * macs_rank, "pointwise_ms_per_step": pw_ms,
                # useful work: the product counted as a schoolbook over 7-bit
                # digits, 2 n^3 ceil(W/7)^2 ops, so a plan that issues more
                # plane products than needed cannot raise it
                "useful_ops_per_step": 2 * useful_rank, "useful_achieved": useful,
                "useful_frac": useful / peak_int8,
                "peak_2x_bf16_sustained": peak_2x_sus,
                "frac_vs_2x_bf16_sustained": achieved / peak_2x_sus,
                "peak_2x_bf16_burst": peak_2x_burst,
                "frac_vs_2x_bf16_burst": achieved / peak_2x_burst,
                "bf16_peaks_from": f"{peak_kind} MEASURED_PEAKS.json"}
            line["int8_tops_issued"] = 2 * macs / (ms * 1e-3) / 1e12
            line["useful_tops"] = 2 * pi["schoolbook7_macs"] / (ms * 1e-3) / 1e12
            line["plan"] = {k: pi[k] for k in ("b", "S", "NB", "K", "dA", "dB", "nchunk", "njobs",
                                               "half_points", "kara", "dsum", "rblock")}
        line["phase_ms_per_step"] = {k: v / args.steps for k, v in ph.items() if k != "total"}
        share = ph["pointwise"] / max(1e-9, sum(v for k, v in ph.items() if k != "total"))
        line["pointwise_share"] = share
    tr = POINTWISE_TRAFFIC.get((args.workload, pi.get("pw_kernel"), pi.get("kara", 0)))
    if ("roofline" in line and tr and world == 1 and n == DEFAULT_N[args.workload]
            and pi.get("kind") == 0):
        line["roofline"]["traffic"] = tr["bytes_per_launch"]
        line["roofline"]["traffic_note"] = tr["note"]

    if world == 1 and "roofline" in line and not args.no_int8_ref:
        ref_tops = cublas_int8_sustained(torch, stream)
        line["roofline"]["int8_cublas_sustained_tops"] = ref_tops
        if ref_tops:
            line["roofline"]["frac_vs_cublas_int8_sustained"] = line["roofline"]["achieved"] / ref_tops
    if w["kind"] == "f32" and rank == 0 and wl.full_out is not None:
        line["accuracy"] = accuracy_vs_fp64(wl, torch)
    if not args.no_e2e:
        if world == 1:
            line["e2e"] = e2e_measure(ctx, wl, min(3, args.steps), torch)
        else:
            line["e2e"] = e2e_measure_dist(wl, min(3, args.steps), torch, dist, device)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_baseline_line(args.workload, args.method)
        except Exception as e:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "unit": "s", "cores": 0, "kind": "reference",
                                    "sample": f"unavailable: {e}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if wl.peer is not None:
        wl.peer.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
