"""ctypes binding of libmfftb200.so (the C ABI in include/mfftgpu.h and
include/mfftbench_b200.h).

The library is the product: there is no Python or CPU fallback.  Importing
this module when the .so is missing raises immediately.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "lib", "libmfftb200.so")
HEADERS = [os.path.join(ROOT, "include", "mfftgpu.h"),
           os.path.join(ROOT, "include", "mfftbench_b200.h")]

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python mfft_bench_b200/build.py`"
                      " (the CUDA library is required; there is no fallback)")

lib = C.CDLL(LIB_PATH)

vp = C.c_void_p
i32, i64, u64, sz = C.c_int, C.c_longlong, C.c_uint64, C.c_size_t


class PlanInfo(C.Structure):
    _fields_ = [(f, C.c_int) for f in
                ("n", "n_int", "mode", "b", "LbA", "LbB", "S", "NB", "K", "g", "ncA", "ncB",
                 "dA", "dB", "nW", "nchunk", "njobs", "positions")] + [
        ("acc_bound", C.c_longlong), ("inv_bound_log2", C.c_double),
        ("int8_macs", C.c_double), ("schoolbook_macs", C.c_double), ("pw_kernel", C.c_int),
        ("kind", C.c_int), ("U", C.c_int), ("balanced", C.c_int), ("half_points", C.c_int),
        ("wA", C.c_int), ("wB", C.c_int), ("schoolbook7_macs", C.c_double), ("kara", C.c_int),
        ("rblock", C.c_int), ("dsum", C.c_int)]

    def as_dict(self):
        return {f: getattr(self, f) for f, _ in self._fields_}


class MfftPlan(C.Structure):
    """``mfft_plan`` (src/mfftbench.h:139-143)."""
    _fields_ = [("L", C.c_int), ("S", C.c_int), ("NB", C.c_int), ("K", C.c_int),
                ("g", C.c_int), ("rec", C.c_int), ("nprod", C.c_longlong)]


class FpxCtx(C.Structure):
    """``fpx_ctx`` (src/mfftbench.h:182-189)."""
    _fields_ = [("n", C.c_int), ("L", C.c_int), ("sig", C.c_int), ("SA", C.c_int),
                ("SB", C.c_int), ("spreadA", C.c_int), ("spreadB", C.c_int),
                ("A32", C.POINTER(C.c_int32)), ("B32", C.POINTER(C.c_int32)),
                ("Cw", C.POINTER(C.c_int64)), ("enc_secs", C.c_double),
                ("dec_secs", C.c_double)]


def _sig(name, res, *args):
    f = getattr(lib, name)
    f.restype = res
    f.argtypes = list(args)
    return f


# native ABI
_sig("mfftgpu_create", i32, C.POINTER(vp), i32)
_sig("mfftgpu_destroy", i32, vp)
_sig("mfftgpu_set_stream", i32, vp, vp)
_sig("mfftgpu_set_workspace_limit", i32, vp, sz)
_sig("mfftgpu_set_timeout_ns", i32, vp, C.c_ulonglong)
_sig("mfftgpu_sync", i32, vp)
_sig("mfftgpu_set_reuse_b", i32, vp, i32)
_sig("mfftgpu_set_kernel_variant", i32, vp, i32, i32)
_sig("mfftgpu_set_karatsuba", i32, vp, i32)
_sig("mfftgpu_set_digit_sums", i32, vp, i32)
_sig("mfftgpu_set_half_points", i32, vp, i32)
_sig("mfftgpu_set_method", i32, vp, i32)
_sig("mfftgpu_set_output_plane_stride", i32, vp, C.c_longlong)
_sig("mfftgpu_ipc_alloc", i32, C.c_size_t, C.POINTER(C.c_void_p), vp)
_sig("mfftgpu_ipc_open", i32, vp, C.POINTER(C.c_void_p))
_sig("mfftgpu_ipc_close", i32, vp)
_sig("mfftgpu_ipc_free", i32, vp)
_sig("mfftgpu_get_method", i32, vp)
_sig("mfftgpu_last_error", C.c_char_p, vp)
_sig("mfftgpu_status_string", C.c_char_p, i32)
_sig("mfftgpu_device_count", i32)
_sig("mfftgpu_plan_info_get", i32, i32, i32, i32, i32, C.POINTER(PlanInfo))
_sig("mfftgpu_last_plan", i32, vp, C.POINTER(PlanInfo))
_sig("mfftgpu_last_phase_ms", i32, vp, C.POINTER(C.c_float))
_sig("mfftgpu_last_launches", i32, vp)
_sig("mfftgpu_last_phase_dropped", i32, vp)
_sig("mfftgpu_set_profile", i32, vp, i32)
_sig("mfftgpu_mm_u16_dev", i32, vp, vp, vp, i32, i32, i32, vp, i32, i32, i32)
_sig("mfftgpu_mm_u16", i32, vp, vp, vp, i32, i32, i32, vp, i32)
_sig("mfftgpu_mm_i64_dev", i32, vp, vp, vp, i32, vp, i32, i32, i32)
_sig("mfftgpu_mm_i64", i32, vp, vp, vp, i32, vp, i32)
_sig("mfftgpu_conv_i32_dev", i32, vp, vp, vp, i32, i32, vp)
_sig("mfftgpu_conv_i32", i32, vp, vp, vp, i32, i32, vp)
_sig("mfftgpu_fp32_dev", i32, vp, vp, vp, i32, i32, vp, i32, i32)
_sig("mfftgpu_fp32", i32, vp, vp, vp, i32, i32, vp)
_sig("mfftgpu_fp64_dev", i32, vp, vp, vp, i32, i32, vp, i32, i32)
_sig("mfftgpu_fp64", i32, vp, vp, vp, i32, i32, vp)
_sig("mfftgpu_gen_bigmat_dev", i32, vp, vp, i32, i32, u64)
_sig("mfftgpu_gen_int64_dev", i32, vp, vp, sz, u64)
_sig("mfftgpu_selftest_timeout", i32, vp, C.c_ulonglong)
_sig("mfftgpu_gen_normal_f32", None, vp, vp, sz, u64)
_sig("mfftgpu_mm_i64_noalloc", i32, vp, vp, i32, vp, i32, vp)
_sig("mfftgpu_decode_words_f32", C.c_float, vp, i32, i32, i32)
_sig("mfftgpu_decode_words_f64", C.c_double, vp, i32, i32, i32)
_sig("mfftgpu_decode_words_round", i32, vp, i32, i32, i32, C.POINTER(C.c_uint64),
     C.POINTER(C.c_int))
_sig("mfftgpu_selftest_pointwise", i32, vp, i32, i32, i32, i32, i32, i32, i32, i32, i32, i32,
     C.POINTER(C.c_longlong))
_sig("mfftgpu_selftest_school", i32, vp, i32, i32, i32, i32, i32, i32, C.POINTER(C.c_longlong))

# reference-compatible ABI
_sig("kernel_name", C.c_char_p, i32)
_sig("kernel_from_name", i32, C.c_char_p)
_sig("bigmat_rand", None, vp, i32, i32, u64)
_sig("normalize_planes", None, vp, i32, i32, vp, i32)
_sig("bigres_equal", i32, vp, vp, i32, i32, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32))
_sig("mfft_plan_init", i32, C.POINTER(MfftPlan), i32, i32)
_sig("mfft_plan_init_rec", i32, C.POINTER(MfftPlan), i32, i32, i32)
_sig("mfft_plan_products", C.c_longlong, C.POINTER(MfftPlan))
_sig("mfft_plan_maxbits", C.c_double, C.POINTER(MfftPlan), i32)
_sig("mm_mfft", None, vp, vp, i32, i32, C.POINTER(MfftPlan), i32, vp, i32)
_sig("mm_mfft_signed", None, vp, vp, i32, i32, vp, i32)
_sig("conv_mfft", None, vp, vp, vp, i32, i32, C.POINTER(MfftPlan), i32)
_sig("ssa_negconv", None, vp, vp, vp, i32, i32, i32, i32)
_sig("fpx_init", i32, C.POINTER(FpxCtx), vp, vp, i32, i32)
_sig("fpx_encode", None, C.POINTER(FpxCtx), vp, vp)
_sig("fpx_decode_f32", None, C.POINTER(FpxCtx), vp)
_sig("fpx_free", None, C.POINTER(FpxCtx))
_sig("fpx_gemm_f32", i32, vp, vp, i32, i32, vp)
_sig("fpx_init_d", i32, C.POINTER(FpxCtx), vp, vp, i32, i32)
_sig("fpx_encode_d", None, C.POINTER(FpxCtx), vp, vp)
_sig("fpx_decode_f64", None, C.POINTER(FpxCtx), vp)
_sig("fpx_decode_ld", None, C.POINTER(FpxCtx), vp)
_sig("fpx_gemm_f64", i32, vp, vp, i32, i32, vp)
_sig("fpx_gemm_f64_limbplane", i32, vp, vp, i32, i32, vp)
_sig("mm_limbplane", None, vp, vp, i32, i32, i32, vp, i32)
_sig("mm_limbplane_signed", None, vp, vp, i32, i32, vp, i32)
_sig("conv_limbplane", None, vp, vp, vp, i32, i32, i32)
_sig("fpx_gemm_f32_limbplane", i32, vp, vp, i32, i32, vp)
_sig("mfftb_last_status", i32)


def declared_functions():
    """Every function name declared in include/*.h (for the export check)."""
    names = set()
    for h in HEADERS:
        with open(h) as f:
            text = f.read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([A-Za-z_]\w*)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name not in ("if", "while", "for", "return", "sizeof", "defined"):
                names.add(name)
        for m in re.finditer(r"^extern\s+[\w\s\*]+?\b([A-Za-z_]\w*)\s*;", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)
