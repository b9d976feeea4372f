/* mfftbench_b200.h -- drop-in replacement of the hot-path part of
 * hadilq/mfft-bench's src/mfftbench.h, backed by the B200 library
 * (libmfftb200.so).  A program that calls mm_mfft / conv_mfft / fpx_* links
 * libmfftb200 instead of src/mfft.c + src/kernel.c + src/fpfixed.c and keeps
 * its source unchanged.
 *
 * Types and signatures are identical to the reference so that existing
 * callers compile and link unchanged; each declaration names the reference
 * line it replaces.  Differences in behaviour:
 *   - the product always runs on the GPU; the kernel_t argument is accepted
 *     and ignored (every leaf is the tcgen05 int8 contraction);
 *   - the mfft_plan argument is validated (L must match) but the GPU plans
 *     its own limb radix/block size for int8 tensor cores; results are
 *     bit-identical for every plan;
 *   - failures print "mfft: ..." to stderr and leave the output zeroed (the
 *     reference's out-of-memory behaviour, src/mfft.c:317-320); the status
 *     of the last call is available from mfftb_last_status().
 * The device is the CUDA current device at first use, or $MFFTGPU_DEVICE.
 */
#ifndef MFFTBENCH_B200_H
#define MFFTBENCH_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef LIMB_BITS
#define LIMB_BITS 16 /* src/mfftbench.h:20-27; the GPU path supports 16 only */
#endif
#define LIMB_MASK ((uint32_t)((1u << LIMB_BITS) - 1u))

/* src/mfftbench.h:33-47, plus KERNEL_SM100 for callers that want to name the
 * GPU leaf explicitly. */
typedef enum {
    KERNEL_IKJ = 0,
    KERNEL_BLOCKED,
    KERNEL_PACKED,
    KERNEL_STRASSEN,
    KERNEL_WINOGRAD,
    KERNEL_BITPLANE,
    KERNEL_CONVK,
    KERNEL_CONVKARA,
    KERNEL_BOOLPACK,
    KERNEL_BITPACK,
    KERNEL_BOOLSTRASSEN,
    KERNEL_BOOLTILED,
    KERNEL_SM100,
    KERNEL__COUNT
} kernel_t;

const char *kernel_name(kernel_t k);        /* src/mfftbench.h:49, src/kernel.c:21-25 */
int kernel_from_name(const char *s);        /* src/mfftbench.h:50, src/kernel.c:31-36 */

/* number of n x n int8 plane products (digit-pair GEMM equivalents) the last
 * product issued; the reference counts mm_accum calls (src/kernel.c:13) */
extern long long g_kernel_calls;

/* src/mfftbench.h:58-70: phase timers, filled from device events when
 * g_mfft_profile is set.  pack = limb split, build_ops = 0 (the op list is
 * folded into the transform kernels), transform = forward + inverse,
 * pointwise = tcgen05 contraction, fold = inverse-side fold/carry share. */
typedef struct {
    double pack, build_ops, transform, pointwise, fold;
    long long n_build, n_fft;
} mfft_profile_t;
extern int g_mfft_profile;
extern mfft_profile_t g_mfft_prof;
void mfft_profile_reset(void);               /* src/mfft.c:46-49 */
void mfft_profile_print(const char *label);  /* src/mfft.c:51-73 */

/* big-integer matrices, src/mfftbench.h:74-91 (host utilities) */
uint16_t *bigmat_alloc(int n, int L);                                  /* src/bigmat.c:15-18 */
void bigmat_rand(uint16_t *m, int n, int L, uint64_t seed);            /* src/bigmat.c:29-35 */
uint16_t *bigmat_to_entry_major(const uint16_t *plane, int n, int L);  /* src/bigmat.c:37-46 */
void normalize_planes(const int64_t *acc, int nplanes, int n, uint16_t *out,
                      int RL);                                         /* src/bigmat.c:48-60 */
int bigres_equal(const uint16_t *a, const uint16_t *b, int n, int RL, int *bad_i, int *bad_j,
                 int *bad_w);                                          /* src/bigmat.c:62-75 */
double now_sec(void);                                                  /* src/bigmat.c:8-13 */

/* MFFT plan, src/mfftbench.h:139-154 */
typedef struct {
    int L, S, NB, K, g;
    int rec;
    long long nprod;
} mfft_plan;
int mfft_plan_init(mfft_plan *p, int L, int sigma_override);   /* src/mfft.c:77-95 */
/* the recursive plan (rec = 1): same S/NB/K choice and product count as the
 * reference's; mm_mfft / conv_mfft run it on the B200 path like any plan */
int mfft_plan_init_rec(mfft_plan *p, int L, int n, int sigma_override); /* src/mfft.c:665-686 */
/* C (K int64 planes) = A * B mod (y^K + 1) over n x n int32 planes, exact;
 * Mbits (the reference's magnitude hint) is not needed by the GPU product */
void ssa_negconv(int64_t *C, const int32_t *A, const int32_t *B, int K, int n, int Mbits,
                 kernel_t kern);                                /* src/mfft.c:560-662 */
long long mfft_plan_products(const mfft_plan *p);               /* src/mfft.c:97-100 */
double mfft_plan_maxbits(const mfft_plan *p, int n);            /* src/mfft.c:102-110 */
void mfft_plan_describe(const mfft_plan *p, int n);             /* src/mfft.c:112-122 */

/* the hot path, src/mfftbench.h:156-159 */
void mm_mfft(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, const mfft_plan *p,
             kernel_t k, uint16_t *out, int RL);                /* src/mfft.c:424-438 */
void conv_mfft(int64_t *Cw, const int32_t *A32, const int32_t *B32, int n, int L,
               const mfft_plan *p, kernel_t k);                 /* src/mfft.c:302-422 */

/* fp32 fixed-point embedding, src/mfftbench.h:182-199 */
typedef struct {
    int n, L, sig;
    int SA, SB;
    int spreadA, spreadB;
    int32_t *A32, *B32;
    int64_t *Cw;
    double enc_secs, dec_secs;
} fpx_ctx;
int fpx_init(fpx_ctx *c, const float *A, const float *B, int n, int force_bits); /* src/fpfixed.c:96-108 */
void fpx_encode(fpx_ctx *c, const float *A, const float *B);                    /* src/fpfixed.c:195-204 */
void fpx_decode_f32(fpx_ctx *c, float *C);                                       /* src/fpfixed.c:269-285 */
int fpx_init_d(fpx_ctx *c, const double *A, const double *B, int n, int force_bits); /* src/fpfixed.c:130-140 */
void fpx_encode_d(fpx_ctx *c, const double *A, const double *B);                    /* src/fpfixed.c:162-172 */
void fpx_decode_f64(fpx_ctx *c, double *C);                                       /* src/fpfixed.c:308-322 */
void fpx_decode_ld(fpx_ctx *c, long double *C);                                   /* src/fpfixed.c:291-306 */
void fpx_free(fpx_ctx *c);                                                       /* src/fpfixed.c:324-328 */

/* status of the last drop-in call (MFFTGPU_* codes of mfftgpu.h); no
 * counterpart in the reference, whose hot-path functions return void */
int mfftb_last_status(void);

/* signed variant of mm_mfft: the limb planes are two's complement 16L-bit
 * integers (the reference reaches signed products through conv_mfft +
 * normalize_planes, src/fpfixed.c:187-192 + src/bigmat.c:48-60) */
void mm_mfft_signed(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, uint16_t *out, int RL);

/* fp32 GEMM on the fixed-point grid, fused on the device: fpx_init +
 * fpx_encode + conv_mfft + fpx_decode_f32 in one call (src/mlgemm.c:1107-1175
 * without the host round trip of the limb planes) */
int fpx_gemm_f32(const float *A, const float *B, int n, int force_bits, float *C);
/* fp64 counterpart: fpx_init_d + fpx_encode_d + conv_mfft + fpx_decode_f64
 * fused on the device */
int fpx_gemm_f64(const double *A, const double *B, int n, int force_bits, double *C);

/* The limb-plane schoolbook method on the same tensor-core kernel: exact,
 * bit-identical to the MFFT entry points, with LbA*LbB digit-plane products
 * instead of the transform's NB*K^2 (the reference's comparator rows:
 * mm_limbplane / conv_limbplane src/methods.c:94-123 declared at
 * src/mfftbench.h:100-106, and the GPU limb-*-exact rows of
 * cuda/gemm_bench.cu:913-998). */
void mm_limbplane(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, kernel_t k,
                  uint16_t *out, int RL);                       /* src/methods.c:106-123 */
void conv_limbplane(int64_t *Cw, const int32_t *A32, const int32_t *B32, int n, int L,
                    kernel_t k);                                /* src/methods.c:94-104 */
void mm_limbplane_signed(const uint16_t *Apl, const uint16_t *Bpl, int n, int L, uint16_t *out,
                         int RL);
int fpx_gemm_f32_limbplane(const float *A, const float *B, int n, int force_bits, float *C);
int fpx_gemm_f64_limbplane(const double *A, const double *B, int n, int force_bits, double *C);

#ifdef __cplusplus
}
#endif
#endif
