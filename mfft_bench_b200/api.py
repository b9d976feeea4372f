"""Python mirror of the reference hot-path interface, backed by libmfftb200.

Names and argument meaning follow hadilq/mfft-bench ``src/mfftbench.h``:
``mfft_plan_init``, ``mm_mfft``, ``conv_mfft``, ``normalize_planes``,
``bigmat_rand``, ``fpx_init`` / ``fpx_encode`` / ``fpx_decode_f32``.  Host
arrays are numpy; the :class:`Context` methods also accept CUDA torch tensors
and then run asynchronously on device memory (no host round trip).

Every product runs on the B200 through the C ABI.  There is no CPU path: a
failing call raises :class:`MfftError` with the library's status.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import FpxCtx, MfftPlan, PlanInfo, lib

KERNEL_PACKED = 2
KERNEL_SM100 = 12
PLAN_VALUE, PLAN_LIMB = 0, 1


class MfftError(RuntimeError):
    def __init__(self, status, msg=""):
        self.status = status
        text = lib.mfftgpu_status_string(status).decode()
        super().__init__(f"mfftgpu status {status} ({text}){': ' + msg if msg else ''}")


def _ptr(x):
    if isinstance(x, int):  # a raw device address (e.g. a peer mapping)
        return C.c_void_p(x)
    if isinstance(x, np.ndarray):
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays must be C-contiguous")
        return C.c_void_p(x.ctypes.data)
    return C.c_void_p(x.data_ptr())


def _is_cuda(x):
    return hasattr(x, "is_cuda") and x.is_cuda


def plan_info(n, mode, wA, wB=None):
    """The int8 tensor-core plan the library uses (see csrc/plan.h)."""
    pi = PlanInfo()
    rc = lib.mfftgpu_plan_info_get(n, mode, wA, wB if wB is not None else wA, C.byref(pi))
    if rc:
        raise MfftError(rc, "plan")
    return pi.as_dict()


def device_count():
    return lib.mfftgpu_device_count()


class Context:
    """One CUDA device, stream and workspace (``mfftgpu_ctx``)."""

    def __init__(self, device=0, stream=None, workspace_bytes=None):
        self._h = C.c_void_p()
        rc = lib.mfftgpu_create(C.byref(self._h), device)
        if rc:
            raise MfftError(rc, f"create(device={device})")
        self.device = device
        if stream is not None:
            self.set_stream(stream)
        if workspace_bytes:
            lib.mfftgpu_set_workspace_limit(self._h, int(workspace_bytes))

    # -- plumbing
    def close(self):
        if self._h:
            lib.mfftgpu_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc, what):
        if rc:
            raise MfftError(rc, f"{what}: {lib.mfftgpu_last_error(self._h).decode()}")

    def set_stream(self, stream):
        s = stream if isinstance(stream, int) else int(stream.cuda_stream)
        self._check(lib.mfftgpu_set_stream(self._h, C.c_void_p(s)), "set_stream")

    def set_timeout_ns(self, ns):
        self._check(lib.mfftgpu_set_timeout_ns(self._h, int(ns)), "set_timeout_ns")

    def set_workspace_limit(self, nbytes):
        self._check(lib.mfftgpu_set_workspace_limit(self._h, int(nbytes)), "workspace")

    def set_profile(self, mode=1):
        """0 off, 1 time the last product, 2 accumulate over products."""
        self._check(lib.mfftgpu_set_profile(self._h, int(mode)), "set_profile")

    def sync(self):
        self._check(lib.mfftgpu_sync(self._h), "sync")

    def set_reuse_b(self, on=True):
        """Reuse the previous product's transformed B when B is the same
        buffer (unchanged contents are the caller's promise)."""
        self._check(lib.mfftgpu_set_reuse_b(self._h, 1 if on else 0), "set_reuse_b")

    def set_method(self, method):
        """'mfft' (default) or 'schoolbook' (limb-plane digit products on the
        same tensor-core kernel) for value-mode products; identical results."""
        mid = {"mfft": 0, "schoolbook": 1}[method]
        self._check(lib.mfftgpu_set_method(self._h, mid), "set_method")

    def set_output_plane_stride(self, elems):
        """Integer outputs of the device-pointer calls: plane w of the computed
        rows at out + w * elems (0: compact [RL][rows][n])."""
        self._check(lib.mfftgpu_set_output_plane_stride(self._h, int(elems)),
                    "set_output_plane_stride")

    def set_half_points(self, on):
        """Skip (True, the default) or compute the plane products that are zero
        at the evaluation points 0 and NB/2; identical results."""
        self._check(lib.mfftgpu_set_half_points(self._h, int(bool(on))), "set_half_points")

    def set_digit_sums(self, on):
        """Digit sums on the two-digit plans (default on): three int8 plane
        products per term instead of four; same bits."""
        self._check(lib.mfftgpu_set_digit_sums(self._h, int(bool(on))), "set_digit_sums")

    def set_karatsuba(self, level):
        """Karatsuba pointwise level on plans that allow it: 0 off, 1 one
        level (True), 2 P0 and P1 split again, 3 P2 as well (the default);
        same bits."""
        self._check(lib.mfftgpu_set_karatsuba(self._h, int(level)), "set_karatsuba")

    def set_kernel_variant(self, stage, variant):
        """Pick the kernel of a stage ('forward', 'pointwise' or 'inverse'; 0 = auto).
        Every variant computes the same bits; this is for comparisons."""
        sid = {"forward": 1, "pointwise": 2, "inverse": 3}[stage]
        self._check(lib.mfftgpu_set_kernel_variant(self._h, sid, int(variant)),
                    "set_kernel_variant")

    def phase_ms(self):
        out = (C.c_float * 5)()
        lib.mfftgpu_last_phase_ms(self._h, out)
        return dict(zip(("pack", "forward", "pointwise", "inverse", "total"), list(out)))

    def launches(self):
        return lib.mfftgpu_last_launches(self._h)

    def phase_dropped(self):
        """Launches past the profile's capacity (their time is not in phase_ms)."""
        return lib.mfftgpu_last_phase_dropped(self._h)

    def last_plan(self):
        pi = PlanInfo()
        self._check(lib.mfftgpu_last_plan(self._h, C.byref(pi)), "last_plan")
        return pi.as_dict()

    # -- products
    def mm_u16(self, A, B, n, L, signed=False, RL=None, out=None, rows=None):
        """Exact product of L-limb uint16 plane-major matrices (mm_mfft).

        numpy inputs: synchronous, returns a numpy [RL*n*n] uint16 array.
        torch CUDA inputs: asynchronous, writes/returns a torch uint16 tensor
        holding rows[0]..rows[1] of every output plane."""
        RL = 2 * L + 1 if RL is None else RL
        if _is_cuda(A):
            import torch
            r0, r1 = rows or (0, n)
            if out is None:
                out = torch.empty(max(RL * (r1 - r0) * n, 1), dtype=torch.uint16,
                                  device=A.device)
            self._check(lib.mfftgpu_mm_u16_dev(self._h, _ptr(A), _ptr(B), n, L, int(signed),
                                               _ptr(out), RL, r0, r1), "mm_u16_dev")
            return out
        out = np.empty(max(RL * n * n, 1), np.uint16) if out is None else out
        self._check(lib.mfftgpu_mm_u16(self._h, _ptr(A), _ptr(B), n, L, int(signed), _ptr(out),
                                       RL), "mm_u16")
        return out

    def mm_i64(self, A, B, n, RL=9, out=None, rows=None):
        """Exact product of int64 row-major matrices; RL two's complement
        16-bit limb planes."""
        if _is_cuda(A):
            import torch
            r0, r1 = rows or (0, n)
            if out is None:
                out = torch.empty(max(RL * (r1 - r0) * n, 1), dtype=torch.uint16,
                                  device=A.device)
            self._check(lib.mfftgpu_mm_i64_dev(self._h, _ptr(A), _ptr(B), n, _ptr(out), RL, r0,
                                               r1), "mm_i64_dev")
            return out
        out = np.empty(max(RL * n * n, 1), np.uint16) if out is None else out
        self._check(lib.mfftgpu_mm_i64(self._h, _ptr(A), _ptr(B), n, _ptr(out), RL), "mm_i64")
        return out

    def conv_i32(self, A32, B32, n, L, out=None):
        """conv_mfft: 2L-1 unnormalised int64 limb-convolution planes."""
        if _is_cuda(A32):
            import torch
            if out is None:
                out = torch.empty((2 * L - 1) * n * n, dtype=torch.int64, device=A32.device)
            self._check(lib.mfftgpu_conv_i32_dev(self._h, _ptr(A32), _ptr(B32), n, L, _ptr(out)),
                        "conv_i32_dev")
            return out
        out = np.empty((2 * L - 1) * n * n, np.int64) if out is None else out
        self._check(lib.mfftgpu_conv_i32(self._h, _ptr(A32), _ptr(B32), n, L, _ptr(out)),
                    "conv_i32")
        return out

    def fp32(self, A, B, n, force_bits=512, out=None, rows=None):
        """fp32 GEMM through the exact fixed-point embedding (fpfixed.c)."""
        if _is_cuda(A):
            import torch
            r0, r1 = rows or (0, n)
            if out is None:
                out = torch.empty((r1 - r0) * n, dtype=torch.float32, device=A.device)
            self._check(lib.mfftgpu_fp32_dev(self._h, _ptr(A), _ptr(B), n, force_bits,
                                             _ptr(out), r0, r1), "fp32_dev")
            return out
        out = np.empty(n * n, np.float32) if out is None else out
        self._check(lib.mfftgpu_fp32(self._h, _ptr(A), _ptr(B), n, force_bits, _ptr(out)),
                    "fp32")
        return out

    def fp64(self, A, B, n, force_bits=512, out=None, rows=None):
        """fp64 GEMM through the exact fixed-point embedding (fpx_*_d)."""
        if _is_cuda(A):
            import torch
            r0, r1 = rows or (0, n)
            if out is None:
                out = torch.empty((r1 - r0) * n, dtype=torch.float64, device=A.device)
            self._check(lib.mfftgpu_fp64_dev(self._h, _ptr(A), _ptr(B), n, force_bits,
                                             _ptr(out), r0, r1), "fp64_dev")
            return out
        out = np.empty(n * n, np.float64) if out is None else out
        self._check(lib.mfftgpu_fp64(self._h, _ptr(A), _ptr(B), n, force_bits, _ptr(out)),
                    "fp64")
        return out

    def gen_bigmat(self, m, n, L, seed):
        """bigmat_rand on the device into the uint16 CUDA tensor m."""
        self._check(lib.mfftgpu_gen_bigmat_dev(self._h, _ptr(m), n, L, seed), "gen_bigmat")
        return m

    def gen_int64(self, x, seed):
        self._check(lib.mfftgpu_gen_int64_dev(self._h, _ptr(x), x.numel(), seed), "gen_int64")
        return x

    def selftest_pointwise(self, rows, cols, kdim, NB, K, dA=1, dB=1, nchunk=1, block_n=256,
                           variant=0):
        mism = C.c_longlong(-1)
        self._check(lib.mfftgpu_selftest_pointwise(self._h, rows, cols, kdim, NB, K, dA, dB,
                                                   nchunk, block_n, variant, C.byref(mism)),
                    "selftest_pointwise")
        return mism.value

    def selftest_school(self, rows, cols, kdim, LbA, LbB, U):
        """Mismatching elements of the schoolbook job table on the tensor-core
        kernel vs a CUDA-core evaluation (expected 0)."""
        mism = C.c_longlong(-1)
        self._check(lib.mfftgpu_selftest_school(self._h, rows, cols, kdim, LbA, LbB, U,
                                                C.byref(mism)), "selftest_school")
        return mism.value

    def selftest_timeout(self, timeout_ns=50_000_000):
        """Status of a pointwise launch whose producer never loads (expected:
        MFFTGPU_ERR_TIMEOUT = 4, and the context stays usable)."""
        return lib.mfftgpu_selftest_timeout(self._h, int(timeout_ns))


# ---------------------------------------------------------------------------
# reference-named entry points (host buffers), src/mfftbench.h
# ---------------------------------------------------------------------------
def mfft_plan_init(L, sigma=0):
    """src/mfft.c:77-95; returns an ``mfft_plan`` or None when L is invalid."""
    p = MfftPlan()
    return p if lib.mfft_plan_init(C.byref(p), L, sigma) == 0 else None


def mfft_plan_init_rec(L, n, sigma=0):
    """src/mfft.c:665-686: the recursive plan (``rec`` = 1) for n x n
    matrices, or None when L admits none."""
    p = MfftPlan()
    return p if lib.mfft_plan_init_rec(C.byref(p), L, n, sigma) == 0 else None


def ssa_negconv(A32, B32, K, n, Mbits=0, kernel=KERNEL_SM100):
    """src/mfft.c:560-662 through the drop-in C symbol: the K int64 planes of
    A * B mod (y^K + 1), A and B K int32 planes of n x n matrices."""
    C_ = np.zeros(K * n * n, np.int64)
    A32, B32 = np.ascontiguousarray(A32, np.int32), np.ascontiguousarray(B32, np.int32)
    lib.ssa_negconv(_ptr(C_), _ptr(A32), _ptr(B32), K, n, Mbits, kernel)
    _status("ssa_negconv")
    return C_


def bigmat_rand(n, L, seed):
    m = np.empty(n * n * L, np.uint16)
    lib.bigmat_rand(_ptr(m), n, L, C.c_uint64(seed))
    return m


def normalize_planes(acc, nplanes, n, RL):
    out = np.empty(RL * n * n, np.uint16)
    lib.normalize_planes(_ptr(np.ascontiguousarray(acc, np.int64)), nplanes, n, _ptr(out), RL)
    return out


def _status(what):
    st = lib.mfftb_last_status()
    if st:
        raise MfftError(st, what)


def mm_mfft(Apl, Bpl, n, L, plan=None, kernel=KERNEL_SM100, RL=None):
    """src/mfft.c:424-438 through the drop-in C symbol ``mm_mfft``."""
    RL = 2 * L + 1 if RL is None else RL
    out = np.zeros(RL * n * n, np.uint16)
    plan = plan or mfft_plan_init(L)
    lib.mm_mfft(_ptr(Apl), _ptr(Bpl), n, L, C.byref(plan) if plan else None, kernel, _ptr(out),
                RL)
    _status("mm_mfft")
    return out


def mm_mfft_signed(Apl, Bpl, n, L, RL=None):
    RL = 2 * L + 1 if RL is None else RL
    out = np.zeros(RL * n * n, np.uint16)
    lib.mm_mfft_signed(_ptr(Apl), _ptr(Bpl), n, L, _ptr(out), RL)
    _status("mm_mfft_signed")
    return out


def conv_mfft(A32, B32, n, L, plan=None, kernel=KERNEL_SM100):
    """src/mfft.c:302-422 through the drop-in C symbol ``conv_mfft``."""
    cw = np.zeros((2 * L - 1) * n * n, np.int64)
    plan = plan or mfft_plan_init(L)
    lib.conv_mfft(_ptr(cw), _ptr(A32), _ptr(B32), n, L, C.byref(plan) if plan else None, kernel)
    _status("conv_mfft")
    return cw


class Fpx:
    """fpx_init / fpx_encode / conv_mfft / fpx_decode_f32 (src/fpfixed.c)."""

    def __init__(self, A, B, n, force_bits=512):
        self.c = FpxCtx()
        self.n = n
        self.A, self.B = np.ascontiguousarray(A, np.float32), np.ascontiguousarray(B, np.float32)
        if lib.fpx_init(C.byref(self.c), _ptr(self.A), _ptr(self.B), n, force_bits) != 0:
            raise MfftError(1, "fpx_init")

    def encode(self):
        lib.fpx_encode(C.byref(self.c), _ptr(self.A), _ptr(self.B))

    def conv(self):
        n, L = self.n, self.c.L
        lib.conv_mfft(C.c_void_p(C.addressof(self.c.Cw.contents)),
                      C.c_void_p(C.addressof(self.c.A32.contents)),
                      C.c_void_p(C.addressof(self.c.B32.contents)), n, L, None, KERNEL_SM100)
        _status("conv_mfft")

    def decode_f32(self):
        out = np.empty(self.n * self.n, np.float32)
        lib.fpx_decode_f32(C.byref(self.c), _ptr(out))
        return out

    def free(self):
        lib.fpx_free(C.byref(self.c))


class Fpx64(Fpx):
    """fpx_init_d / fpx_encode_d / conv_mfft / fpx_decode_f64 / fpx_decode_ld
    (src/fpfixed.c:109-172, 291-322)."""

    def __init__(self, A, B, n, force_bits=512):
        self.c = FpxCtx()
        self.n = n
        self.A, self.B = np.ascontiguousarray(A, np.float64), np.ascontiguousarray(B, np.float64)
        if lib.fpx_init_d(C.byref(self.c), _ptr(self.A), _ptr(self.B), n, force_bits) != 0:
            raise MfftError(1, "fpx_init_d")

    def encode(self):
        lib.fpx_encode_d(C.byref(self.c), _ptr(self.A), _ptr(self.B))

    def decode_f64(self):
        out = np.empty(self.n * self.n, np.float64)
        lib.fpx_decode_f64(C.byref(self.c), _ptr(out))
        return out

    def decode_ld(self):
        out = np.empty(self.n * self.n, np.longdouble)
        lib.fpx_decode_ld(C.byref(self.c), _ptr(out))
        return out


def fpx_gemm_f64(A, B, n, force_bits=512):
    out = np.empty(n * n, np.float64)
    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    rc = lib.fpx_gemm_f64(_ptr(A), _ptr(B), n, force_bits, _ptr(out))
    if rc:
        raise MfftError(rc, "fpx_gemm_f64")
    return out


def fpx_gemm_f64_limbplane(A, B, n, force_bits=512):
    out = np.empty(n * n, np.float64)
    A = np.ascontiguousarray(A, np.float64)
    B = np.ascontiguousarray(B, np.float64)
    rc = lib.fpx_gemm_f64_limbplane(_ptr(A), _ptr(B), n, force_bits, _ptr(out))
    if rc:
        raise MfftError(rc, "fpx_gemm_f64_limbplane")
    return out


def fpx_gemm_f32(A, B, n, force_bits=512):
    out = np.empty(n * n, np.float32)
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    rc = lib.fpx_gemm_f32(_ptr(A), _ptr(B), n, force_bits, _ptr(out))
    if rc:
        raise MfftError(rc, "fpx_gemm_f32")
    return out


def mm_limbplane(Apl, Bpl, n, L, kernel=KERNEL_SM100, RL=None):
    """src/methods.c:106-123 through the drop-in C symbol ``mm_limbplane``
    (schoolbook digit-plane products on the tensor cores)."""
    RL = 2 * L + 1 if RL is None else RL
    out = np.zeros(RL * n * n, np.uint16)
    lib.mm_limbplane(_ptr(Apl), _ptr(Bpl), n, L, kernel, _ptr(out), RL)
    _status("mm_limbplane")
    return out


def mm_limbplane_signed(Apl, Bpl, n, L, RL=None):
    RL = 2 * L + 1 if RL is None else RL
    out = np.zeros(RL * n * n, np.uint16)
    lib.mm_limbplane_signed(_ptr(Apl), _ptr(Bpl), n, L, _ptr(out), RL)
    _status("mm_limbplane_signed")
    return out


def conv_limbplane(A32, B32, n, L, kernel=KERNEL_SM100):
    """src/methods.c:94-104 through the drop-in C symbol ``conv_limbplane``."""
    cw = np.zeros((2 * L - 1) * n * n, np.int64)
    lib.conv_limbplane(_ptr(cw), _ptr(A32), _ptr(B32), n, L, kernel)
    _status("conv_limbplane")
    return cw


def fpx_gemm_f32_limbplane(A, B, n, force_bits=512):
    out = np.empty(n * n, np.float32)
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    rc = lib.fpx_gemm_f32_limbplane(_ptr(A), _ptr(B), n, force_bits, _ptr(out))
    if rc:
        raise MfftError(rc, "fpx_gemm_f32_limbplane")
    return out


def gen_normal_f32(n, seed):
    """The fp32 workload (N(0,1) * 2^k, k in [-8, 8]) for A and B, host arrays."""
    A = np.empty(n * n, np.float32)
    B = np.empty(n * n, np.float32)
    lib.mfftgpu_gen_normal_f32(_ptr(A), _ptr(B), n * n, C.c_uint64(seed))
    return A, B


def decode_words_f64(words, bit_off, S):
    """Host run of the device fp64 rounding rule (self-test)."""
    w = np.array(words, dtype=np.uint32)
    return float(lib.mfftgpu_decode_words_f64(_ptr(w), w.size, bit_off, S))


def decode_words_round(words, bit_off, bits):
    """(sign, sig, shift) of the shared extract + round_to rule."""
    w = np.array(words, dtype=np.uint32)
    sig, shift = C.c_uint64(0), C.c_int(0)
    sgn = lib.mfftgpu_decode_words_round(_ptr(w), w.size, bit_off, bits, C.byref(sig),
                                         C.byref(shift))
    return sgn, sig.value, shift.value


def decode_words_f32(words, bit_off, S):
    """Host run of the device fp32 rounding rule (self-test)."""
    w = np.array(words, dtype=np.uint32)
    return float(lib.mfftgpu_decode_words_f32(_ptr(w), w.size, bit_off, S))
