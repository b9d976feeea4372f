"""mfft_bench_b200 -- B200 (sm_100a) implementation of hadilq/mfft-bench's
exact-integer MFFT matmul hot path (mm_mfft / conv_mfft + the fp32 fpfixed
embedding), behind the reference's own C API.

The compute path is libmfftb200.so (hand-written CUDA for sm_100a:
limb-split pack, forward/inverse MFFT transforms, tcgen05 int8 pointwise
contraction, fused fold/carry/round).  Python only binds it.
"""
from .api import (KERNEL_PACKED, KERNEL_SM100, PLAN_LIMB, PLAN_VALUE, Context, Fpx,  # noqa: F401
                  MfftError, bigmat_rand, conv_mfft, decode_words_f32, device_count,
                  Fpx64, conv_limbplane, decode_words_f64, decode_words_round, fpx_gemm_f32,
                  fpx_gemm_f32_limbplane, fpx_gemm_f64, fpx_gemm_f64_limbplane, gen_normal_f32,
                  mfft_plan_init, mfft_plan_init_rec, mm_limbplane, mm_limbplane_signed, mm_mfft, mm_mfft_signed,
                  normalize_planes, plan_info, ssa_negconv)
from ._lib import LIB_PATH  # noqa: F401
