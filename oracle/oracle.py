"""TEST INFRASTRUCTURE ONLY -- ctypes bindings for the CPU oracle.

Two checkers live here:

* ``Oracle``: this repository's C restatement of the reference hot path
  (``oracle/mfft_oracle.c``, built into ``oracle/liboracle.so``).
* ``RefLib``: the reference's own C sources (hadilq/mfft-bench ``src/``)
  compiled from source by ``oracle/Makefile`` into ``oracle/_ref/``.  Its
  entry points are called with the reference's exact signatures
  (``src/mfftbench.h``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this module.  The
product package never does.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")


class OrcPlan(C.Structure):
    _fields_ = [("L", C.c_int), ("S", C.c_int), ("NB", C.c_int), ("K", C.c_int),
                ("g", C.c_int), ("nprod", C.c_longlong)]


class RefPlan(C.Structure):
    """``mfft_plan`` of src/mfftbench.h:139-143."""
    _fields_ = [("L", C.c_int), ("S", C.c_int), ("NB", C.c_int), ("K", C.c_int),
                ("g", C.c_int), ("rec", C.c_int), ("nprod", C.c_longlong)]


class RefFpx(C.Structure):
    """``fpx_ctx`` of src/mfftbench.h:182-189."""
    _fields_ = [("n", C.c_int), ("L", C.c_int), ("sig", C.c_int), ("SA", C.c_int),
                ("SB", C.c_int), ("spreadA", C.c_int), ("spreadB", C.c_int),
                ("A32", C.POINTER(C.c_int32)), ("B32", C.POINTER(C.c_int32)),
                ("Cw", C.POINTER(C.c_int64)), ("enc_secs", C.c_double),
                ("dec_secs", C.c_double)]


KERNEL_IKJ, KERNEL_BLOCKED, KERNEL_PACKED = 0, 1, 2


def _load(path):
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built; run `make -C oracle`")
    return C.CDLL(path)


class Oracle:
    def __init__(self):
        L = self.lib = _load(os.path.join(HERE, "liboracle.so"))
        L.orc_bigmat_rand.argtypes = [_u16p, C.c_int, C.c_int, C.c_uint64]
        L.orc_gen_signed_planes.argtypes = [_u16p, C.c_int, C.c_int, C.c_uint64]
        L.orc_gen_int64.argtypes = [_i64p, C.c_size_t, C.c_uint64]
        L.orc_int64_to_planes.argtypes = [_i64p, C.c_int, _u16p]
        L.orc_gen_normal_f32.argtypes = [_f32p, _f32p, C.c_size_t, C.c_uint64]
        L.orc_planes_to_signlimb.argtypes = [_u16p, C.c_int, C.c_int, _i32p]
        L.orc_plan_init.argtypes = [C.POINTER(OrcPlan), C.c_int, C.c_int]
        L.orc_conv_mfft.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int, C.POINTER(OrcPlan)]
        L.orc_conv_limbplane.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int]
        L.orc_normalize_planes.argtypes = [_i64p, C.c_int, C.c_int, _u16p, C.c_int]
        L.orc_mm_mfft.argtypes = [_u16p, _u16p, C.c_int, C.c_int, C.POINTER(OrcPlan), _u16p,
                                  C.c_int]
        L.orc_mm_signed.argtypes = [_u16p, _u16p, C.c_int, C.c_int, _u16p, C.c_int]
        L.orc_entry_product.argtypes = [_u16p, _u16p, C.c_int, C.c_int, C.c_int, C.c_int,
                                        _i32p, _i32p, _u16p, C.c_int]
        L.orc_digest_u16.argtypes = [_u16p, C.c_size_t]
        L.orc_digest_u16.restype = C.c_uint64
        L.orc_fpx_entries.argtypes = [_f32p, _f32p, C.c_int, C.c_int, C.c_int, _i32p, _i32p,
                                      _f32p]
        L.orc_decode_f32_entry.argtypes = [_i64p, C.c_int, C.c_int]
        L.orc_decode_f32_entry.restype = C.c_float
        L.orc_fpx64_entries.argtypes = [_f64p, _f64p, C.c_int, C.c_int, C.c_int, _i32p, _i32p,
                                        _f64p]
        L.orc_decode_f64_entry.argtypes = [_i64p, C.c_int, C.c_int]
        L.orc_decode_f64_entry.restype = C.c_double
        L.orc_checksum_modp.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                        C.c_int, _u16p, C.c_int]
        L.orc_checksum_modp.restype = C.c_longlong

    # ---------------------------------------------------------- generators
    def bigmat_rand(self, n, L, seed):
        m = np.empty(n * n * L, np.uint16)
        self.lib.orc_bigmat_rand(m, n, L, seed)
        return m

    def signed_planes(self, n, L, seed):
        m = np.empty(n * n * L, np.uint16)
        self.lib.orc_gen_signed_planes(m, n, L, seed)
        return m

    def int64_entries(self, n, seed):
        x = np.empty(n * n, np.int64)
        self.lib.orc_gen_int64(x, x.size, seed)
        return x

    def int64_to_planes(self, x, n):
        p = np.empty(4 * n * n, np.uint16)
        self.lib.orc_int64_to_planes(np.ascontiguousarray(x, np.int64), n, p)
        return p

    def normal_f32(self, n, seed):
        a = np.empty(n * n, np.float32)
        b = np.empty(n * n, np.float32)
        self.lib.orc_gen_normal_f32(a, b, n * n, seed)
        return a, b

    # ---------------------------------------------------------- products
    def plan(self, L, sigma=0):
        p = OrcPlan()
        if self.lib.orc_plan_init(C.byref(p), L, sigma) != 0:
            return None
        return p

    def signlimb(self, planes, n, L):
        out = np.empty(L * n * n, np.int32)
        self.lib.orc_planes_to_signlimb(planes, n, L, out)
        return out

    def conv_mfft(self, A32, B32, n, L, plan=None):
        plan = plan or self.plan(L)
        cw = np.zeros((2 * L - 1) * n * n, np.int64)
        self.lib.orc_conv_mfft(cw, A32, B32, n, L, C.byref(plan))
        return cw

    def conv_limbplane(self, A32, B32, n, L):
        cw = np.zeros((2 * L - 1) * n * n, np.int64)
        self.lib.orc_conv_limbplane(cw, A32, B32, n, L)
        return cw

    def normalize_planes(self, cw, nplanes, n, RL):
        out = np.empty(RL * n * n, np.uint16)
        self.lib.orc_normalize_planes(np.ascontiguousarray(cw, np.int64), nplanes, n, out, RL)
        return out

    def mm_mfft(self, A, B, n, L, RL=None, plan=None):
        RL = RL or 2 * L + 1
        plan = plan or self.plan(L)
        out = np.empty(RL * n * n, np.uint16)
        self.lib.orc_mm_mfft(A, B, n, L, C.byref(plan), out, RL)
        return out

    def mm_signed(self, A, B, n, L, RL=None):
        RL = RL or 2 * L + 1
        out = np.empty(RL * n * n, np.uint16)
        self.lib.orc_mm_signed(A, B, n, L, out, RL)
        return out

    def entries(self, A, B, n, L, is_signed, rows, cols, RL=None):
        RL = RL or 2 * L + 1
        rows = np.ascontiguousarray(rows, np.int32)
        cols = np.ascontiguousarray(cols, np.int32)
        out = np.empty(RL * rows.size, np.uint16)
        self.lib.orc_entry_product(A, B, n, L, int(is_signed), rows.size, rows, cols, out, RL)
        return out.reshape(RL, rows.size)

    def digest(self, v):
        v = np.ascontiguousarray(v, np.uint16)
        return int(self.lib.orc_digest_u16(v, v.size))

    def fpx_entries(self, A, B, n, force_bits, rows, cols):
        rows = np.ascontiguousarray(rows, np.int32)
        cols = np.ascontiguousarray(cols, np.int32)
        out = np.empty(rows.size, np.float32)
        self.lib.orc_fpx_entries(A, B, n, force_bits, rows.size, rows, cols, out)
        return out

    def checksum(self, A, B, n, L, is_signed, Cplanes, RL, fmt=None):
        """Row/column sums of C vs A*(B*1) and (1^T A)*B mod 2^61-1; returns
        the number of mismatching rows + columns (0 = pass)."""
        A = np.ascontiguousarray(A)
        B = np.ascontiguousarray(B)
        if fmt is None:
            fmt = 1 if A.dtype == np.int64 else 0
        return int(self.lib.orc_checksum_modp(A.ctypes.data, B.ctypes.data, fmt, n, L,
                                              int(is_signed), np.ascontiguousarray(Cplanes),
                                              RL))

    def decode_f32_entry(self, cw, L, S):
        return float(self.lib.orc_decode_f32_entry(np.ascontiguousarray(cw, np.int64), L, S))

    def decode_f64_entry(self, cw, L, S):
        return float(self.lib.orc_decode_f64_entry(np.ascontiguousarray(cw, np.int64), L, S))

    def fpx64_entries(self, A, B, n, force_bits, rows, cols):
        rows = np.ascontiguousarray(rows, np.int32)
        cols = np.ascontiguousarray(cols, np.int32)
        out = np.empty(rows.size, np.float64)
        self.lib.orc_fpx64_entries(np.ascontiguousarray(A, np.float64),
                                   np.ascontiguousarray(B, np.float64), n, force_bits, rows.size,
                                   rows, cols, out)
        return out


def _host_has_avx512():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = line.split()
                    return "avx512f" in flags and "avx512bw" in flags and "avx512vl" in flags
    except OSError:
        pass
    return False


def ref_library_path():
    v = "v4" if _host_has_avx512() else "v3"
    return os.path.join(HERE, "_ref", f"libmfftref_{v}.so")


class RefLib:
    """The reference's own hot-path C, compiled from source (oracle/Makefile)."""

    def __init__(self, path=None):
        self.path = path or ref_library_path()
        L = self.lib = _load(self.path)
        L.bigmat_rand.argtypes = [_u16p, C.c_int, C.c_int, C.c_uint64]
        L.mfft_plan_init.argtypes = [C.POINTER(RefPlan), C.c_int, C.c_int]
        L.mm_mfft.argtypes = [_u16p, _u16p, C.c_int, C.c_int, C.POINTER(RefPlan), C.c_int,
                              _u16p, C.c_int]
        L.mfft_plan_init_rec.argtypes = [C.POINTER(RefPlan), C.c_int, C.c_int, C.c_int]
        L.ssa_negconv.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.mm_limbplane.argtypes = [_u16p, _u16p, C.c_int, C.c_int, C.c_int, _u16p, C.c_int]
        L.conv_mfft.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int, C.POINTER(RefPlan),
                                C.c_int]
        L.conv_limbplane.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int, C.c_int]
        L.normalize_planes.argtypes = [_i64p, C.c_int, C.c_int, _u16p, C.c_int]
        L.mm_accum.argtypes = [_i64p, _i32p, _i32p, C.c_int, C.c_int, C.c_int]
        L.fpx_init.argtypes = [C.POINTER(RefFpx), _f32p, _f32p, C.c_int, C.c_int]
        L.fpx_encode.argtypes = [C.POINTER(RefFpx), _f32p, _f32p]
        L.fpx_decode_f32.argtypes = [C.POINTER(RefFpx), _f32p]
        L.fpx_init_d.argtypes = [C.POINTER(RefFpx), _f64p, _f64p, C.c_int, C.c_int]
        L.fpx_encode_d.argtypes = [C.POINTER(RefFpx), _f64p, _f64p]
        L.fpx_decode_f64.argtypes = [C.POINTER(RefFpx), _f64p]
        L.fpx_free.argtypes = [C.POINTER(RefFpx)]
        L.roots_selftest.argtypes = [C.c_int, C.c_int]
        L.roots_build_H.argtypes = [C.c_int]
        L.roots_build_H.restype = C.POINTER(C.c_int)

    def plan(self, L, sigma=0):
        p = RefPlan()
        if self.lib.mfft_plan_init(C.byref(p), L, sigma) != 0:
            return None
        return p

    def plan_rec(self, L, n, sigma=0):
        """src/mfft.c:665-686, the recursive plan."""
        p = RefPlan()
        if self.lib.mfft_plan_init_rec(C.byref(p), L, n, sigma) != 0:
            return None
        return p

    def ssa_negconv(self, A32, B32, K, n, Mbits, kernel=KERNEL_PACKED):
        """src/mfft.c:560-662: A * B mod (y^K + 1) over n x n int32 planes."""
        out = np.zeros(K * n * n, np.int64)
        self.lib.ssa_negconv(out, np.ascontiguousarray(A32, np.int32),
                             np.ascontiguousarray(B32, np.int32), K, n, Mbits, kernel)
        return out

    def bigmat_rand(self, n, L, seed):
        m = np.empty(n * n * L, np.uint16)
        self.lib.bigmat_rand(m, n, L, seed)
        return m

    def mm_mfft(self, A, B, n, L, RL=None, kernel=KERNEL_PACKED, plan=None):
        RL = RL or 2 * L + 1
        out = np.zeros(RL * n * n, np.uint16)
        self.lib.mm_mfft(A, B, n, L, C.byref(plan or self.plan(L)), kernel, out, RL)
        return out

    def mm_limbplane(self, A, B, n, L, RL=None, kernel=KERNEL_PACKED):
        RL = RL or 2 * L + 1
        out = np.zeros(RL * n * n, np.uint16)
        self.lib.mm_limbplane(A, B, n, L, kernel, out, RL)
        return out

    def conv_mfft(self, A32, B32, n, L, kernel=KERNEL_PACKED):
        cw = np.zeros((2 * L - 1) * n * n, np.int64)
        self.lib.conv_mfft(cw, A32, B32, n, L, C.byref(self.plan(L)), kernel)
        return cw

    def normalize_planes(self, cw, nplanes, n, RL):
        out = np.empty(RL * n * n, np.uint16)
        self.lib.normalize_planes(np.ascontiguousarray(cw, np.int64), nplanes, n, out, RL)
        return out

    def fp32_gemm(self, A, B, n, force_bits, kernel=KERNEL_PACKED):
        """fpx_init -> fpx_encode -> conv_mfft (flat plan) -> fpx_decode_f32."""
        c = RefFpx()
        if self.lib.fpx_init(C.byref(c), A, B, n, force_bits) != 0:
            raise RuntimeError("fpx_init failed")
        try:
            self.lib.fpx_encode(C.byref(c), A, B)
            nn = n * n
            A32 = np.ctypeslib.as_array(c.A32, shape=(c.L * nn,))
            B32 = np.ctypeslib.as_array(c.B32, shape=(c.L * nn,))
            cw = np.ctypeslib.as_array(c.Cw, shape=((2 * c.L - 1) * nn,))
            plan = self.plan(c.L)
            self.lib.conv_mfft(cw, np.ascontiguousarray(A32), np.ascontiguousarray(B32), n,
                               c.L, C.byref(plan), kernel)
            out = np.empty(nn, np.float32)
            self.lib.fpx_decode_f32(C.byref(c), out)
            return out, (c.L, c.SA, c.SB)
        finally:
            self.lib.fpx_free(C.byref(c))

    def fp64_gemm(self, A, B, n, force_bits, kernel=KERNEL_PACKED):
        """fpx_init_d -> fpx_encode_d -> conv_mfft (flat plan) -> fpx_decode_f64."""
        c = RefFpx()
        A = np.ascontiguousarray(A, np.float64)
        B = np.ascontiguousarray(B, np.float64)
        if self.lib.fpx_init_d(C.byref(c), A, B, n, force_bits) != 0:
            raise RuntimeError("fpx_init_d failed")
        try:
            self.lib.fpx_encode_d(C.byref(c), A, B)
            nn = n * n
            A32 = np.ctypeslib.as_array(c.A32, shape=(c.L * nn,))
            B32 = np.ctypeslib.as_array(c.B32, shape=(c.L * nn,))
            cw = np.ctypeslib.as_array(c.Cw, shape=((2 * c.L - 1) * nn,))
            plan = self.plan(c.L)
            self.lib.conv_mfft(cw, np.ascontiguousarray(A32), np.ascontiguousarray(B32), n,
                               c.L, C.byref(plan), kernel)
            out = np.empty(nn, np.float64)
            self.lib.fpx_decode_f64(C.byref(c), out)
            return out, (c.L, c.SA, c.SB)
        finally:
            self.lib.fpx_free(C.byref(c))
