/* mfftgpu.h -- native C ABI of libmfftb200, the B200 (sm_100a) implementation
 * of hadilq/mfft-bench's exact-integer MFFT matmul path.
 *
 * Every entry point returns an int status (MFFTGPU_OK = 0) and never exits
 * the process.  A context owns one CUDA device, one stream, a grow-only
 * device workspace and a device status word.  "_dev" entry points take
 * device pointers and are asynchronous on the context stream (call
 * mfftgpu_sync for the status of the device-side checks); the other
 * entry points take host pointers, copy inputs in, compute, copy results
 * out and synchronise.
 *
 * Layouts follow the reference (src/mfftbench.h:74-82): a matrix of
 * multi-limb integers is plane-major, p[u*n*n + i*n + j] = limb u of entry
 * (i, j), limbs of 16 bits, least significant first.  Products come back as
 * RL limbs of two's complement.  A row range [row_begin, row_end) computes
 * only those rows of C (row-block sharding across GPUs); out then holds
 * (row_end - row_begin) rows per plane.
 *
 * The reference's own API (mm_mfft, conv_mfft, fpx_*) is provided on top of
 * this by include/mfftbench_b200.h.
 */
#ifndef MFFTGPU_H
#define MFFTGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    MFFTGPU_OK = 0,
    MFFTGPU_ERR_ARG = 1,
    MFFTGPU_ERR_NOMEM = 2,
    MFFTGPU_ERR_CUDA = 3,
    MFFTGPU_ERR_TIMEOUT = 4,
    MFFTGPU_ERR_RANGE = 5,
    MFFTGPU_ERR_NODEVICE = 6,
    MFFTGPU_ERR_PLAN = 7,
    MFFTGPU_ERR_UNSUPPORTED = 8,
};

typedef struct mfftgpu_ctx mfftgpu_ctx;

/* Plan summary (see mfft_bench_b200/csrc/plan.h). */
typedef struct {
    int n, n_int, mode, b, LbA, LbB, S, NB, K, g, ncA, ncB, dA, dB, nW, nchunk, njobs,
        positions;
    long long acc_bound;
    double inv_bound_log2;
    double int8_macs;        /* issued int8 MACs for the whole n x n product */
    double schoolbook_macs;  /* n^3 * LbA * LbB: a schoolbook over this plan's own digits */
    int pw_kernel;           /* plane-product kernel of the last product: 1 one CTA per
                                tile, 2 CTA pairs, 3 t-grouped CTA pairs, 4 Karatsuba
                                CTA pairs; 0 not run */
    int kind;                /* 0 MFFT; 1 limb-plane schoolbook (NB = 1, no transform:
                                job t of chunk ch sums A_u B_(t-u), u in [ch*U, ch*U+U)) */
    int U;                   /* schoolbook: digit planes of A per contraction chunk */
    int balanced;            /* 1: balanced digits in [-2^(b-1), 2^(b-1)) (int64 operands) */
    int half_points;         /* 1: the last product skipped the zero plane products of the
                                points 0 and NB/2 (int8_macs counts the issued ones) */
    int wA, wB;              /* bits per entry: magnitude bits, or 16 x limbs (limb mode) */
    double schoolbook7_macs; /* n^3 * ceil(wA/7) * ceil(wB/7): the useful work of the
                                product, counted as a schoolbook over 7-bit digits */
    int kara;                /* Karatsuba level: 1, three full length-4 convolutions per
                                point (njobs = NB * 21 job planes); 2, the first two of them
                                as three length-2 convolutions each (NB * 25); 3, all three
                                (NB * 27); 0 off */
    int rblock;              /* rows per row block of the last product (each block is one
                                launch of every A-side kernel); 0 from mfftgpu_plan_info_get */
    int dsum;                /* 1: digit sums -- the two int8 digits lo, hi of a transformed
                                value plus lo + hi, three digit-pair classes (lo*lo, hi*hi,
                                sum*sum) instead of four digit pairs; dA = dB = 3, nW = 3 */
} mfftgpu_plan_info;

/* --- context --------------------------------------------------------------
 * Replaces the reference's implicit process-global state (g_mfft_prof,
 * src/mfft.c:43-44; scratch malloc'd per call, src/mfft.c:310-316). */
int mfftgpu_create(mfftgpu_ctx **ctx, int device);
int mfftgpu_destroy(mfftgpu_ctx *ctx);
int mfftgpu_set_stream(mfftgpu_ctx *ctx, void *cuda_stream);
int mfftgpu_set_workspace_limit(mfftgpu_ctx *ctx, size_t bytes);
int mfftgpu_set_timeout_ns(mfftgpu_ctx *ctx, unsigned long long ns);
int mfftgpu_sync(mfftgpu_ctx *ctx);
/* While on, a product whose B (same pointer, size, format and plan) matches
 * the previous product's reuses the transformed B planes kept in the
 * workspace instead of packing and transforming B again -- e.g. for a row
 * range split into several calls.  The caller guarantees B's contents did not
 * change; turning it off drops the cached planes. */
int mfftgpu_set_reuse_b(mfftgpu_ctx *ctx, int on);
/* Product method for value-mode products (mm_u16, mm_i64, fp32):
 * 0 MFFT (default); 1 limb-plane schoolbook on the same tensor-core kernel
 * (digit-plane products A_u B_v accumulated per output position, no
 * transform) -- the GPU counterpart of the reference's mm_limbplane and
 * limb-*-exact rows.  Limb-mode conv always uses MFFT.  Results are
 * bit-identical either way. */
int mfftgpu_set_method(mfftgpu_ctx *ctx, int method);
int mfftgpu_get_method(mfftgpu_ctx *ctx);
/* Layout of the integer outputs of the _dev entry points: 0 (default) writes
 * the computed rows compactly, [RL][row_end-row_begin][n]; a non-zero stride
 * puts plane w of those rows at out + w * stride (e.g. stride n*n with out at
 * row row_begin of a full [RL][n][n] array -- possibly another GPU's memory
 * mapped with mfftgpu_ipc_open, so the final kernel of a sharded product
 * stores its rows straight into the rank that assembles C).  The host-pointer
 * entry points are not affected. */
int mfftgpu_set_output_plane_stride(mfftgpu_ctx *ctx, long long elems);

/* Device buffers shared between the processes of one node (CUDA IPC):
 * mfftgpu_ipc_alloc allocates `bytes` on the current device and writes its
 * 64-byte handle; another process maps it with mfftgpu_ipc_open (peer access
 * over NVLink) and unmaps it with mfftgpu_ipc_close; the owner frees it with
 * mfftgpu_ipc_free after every mapping is closed. */
int mfftgpu_ipc_alloc(size_t bytes, void **ptr, void *handle);
int mfftgpu_ipc_open(const void *handle, void **ptr);
int mfftgpu_ipc_close(void *ptr);
int mfftgpu_ipc_free(void *ptr);
/* Kernel choice per stage, for comparisons; results are identical.
 * stage 1 (forward transform): 0 auto, 1 the generic kernel;
 * stage 2 (plane products): 0 auto, 1 one CTA per tile, 2 CTA pairs,
 *   3 t-grouped CTA pairs (error at launch if the plan does not fit it);
 * stage 3 (inverse + carry): 0 auto, 1 the generic shared-memory kernel,
 *   2 the lane kernel wherever it covers the plan (also NB*K <= 64 plans,
 *   which auto gives the register kernel). */
int mfftgpu_set_kernel_variant(mfftgpu_ctx *ctx, int stage, int variant);
/* Karatsuba pointwise level (0 to 3; the default 3, or $MFFTGPU_KARA).
 * Plans with K = 8 and one int8 digit whose sums a0 + a1 still fit int8 (the
 * W = 64 configuration) take each point's ring product as three full
 * convolutions of length 4, P0 = a0 b0, P1 = a1 b1, P2 = (a0 + a1)(b0 + b1)
 * with a = a0 + y^4 a1: 48 plane products per point instead of 64, 16 at the
 * points 0 and NB/2 (level 1).  Level 2 splits P0 and P1 the same way into
 * three length-2 convolutions each (their sums of two transformed values
 * still fit int8): 40 plane products per point, 12 at the points 0 and NB/2.
 * Level 3 splits P2 as well (a0 + a1 takes one digit per transform block,
 * like a single value): 36 per point.  Results are identical at every
 * level; other values return MFFTGPU_ERR_ARG. */
int mfftgpu_set_karatsuba(mfftgpu_ctx *ctx, int level);
/* Digit sums, on = 1 (the default, or $MFFTGPU_DSUM): plans that split each
 * transformed value into two int8 digits x = lo + 2^7 hi (c1, c3) also form
 * lo + hi, which stays in int8 when |hi| <= 64, and take the middle digit
 * class lo_A hi_B + hi_A lo_B as (lo_A + hi_A)(lo_B + hi_B) - lo_A lo_B -
 * hi_A hi_B: three int8 plane products per term instead of four.  Results
 * are identical either way. */
int mfftgpu_set_digit_sums(mfftgpu_ctx *ctx, int on);
/* At the evaluation points 0 and NB/2 the transformed blocks keep only their
 * low K/2 coefficients, so three quarters of those points' plane products
 * are zero; on = 1 (the default, or $MFFTGPU_HALF_POINTS) lets the t-grouped
 * plane-product kernel skip them, 0 computes them.  Results are identical. */
int mfftgpu_set_half_points(mfftgpu_ctx *ctx, int on);
const char *mfftgpu_last_error(mfftgpu_ctx *ctx);
const char *mfftgpu_status_string(int status);
int mfftgpu_device_count(void);

/* Plan the product (mode 0: value re-radix, 1: limb mode as used by
 * conv_mfft, 2: value re-radix with the limb-plane schoolbook method, 3: the
 * same for int64 operands, which may use balanced 8-bit digits).
 * wA/wB: magnitude bits (modes 0, 2, 3) or limb counts (mode 1). */
int mfftgpu_plan_info_get(int n, int mode, int wA, int wB, mfftgpu_plan_info *out);
/* The plan of the last product run on this context (the fp32 plan depends on
 * the exponent window of the data). */
int mfftgpu_last_plan(mfftgpu_ctx *ctx, mfftgpu_plan_info *out);

/* Per-kernel device timing (mirrors the reference's --profile split,
 * src/mfft.c:43-73).  mode 0: off; 1: the last product; 2: accumulate over
 * every product since this call.  Events are recorded on the context stream
 * without host synchronisation, so profiling does not perturb a timed loop.
 * mfftgpu_last_phase_ms waits for the events and returns milliseconds:
 * [pack, forward, pointwise, inverse+carry, first-to-last event]. */
int mfftgpu_set_profile(mfftgpu_ctx *ctx, int mode);
int mfftgpu_last_phase_ms(mfftgpu_ctx *ctx, float out[5]);
/* Launches the profile could not record (past its 2048-launch capacity);
 * their time is missing from mfftgpu_last_phase_ms. */
int mfftgpu_last_phase_dropped(mfftgpu_ctx *ctx);
/* Number of kernel launches of the last product. */
int mfftgpu_last_launches(mfftgpu_ctx *ctx);

/* --- exact integer products ------------------------------------------------
 * Replaces mm_mfft (src/mfft.c:424-438, src/mfftbench.h:156-157).  A, B: L
 * uint16 limb planes each; is_signed = 1 reads them as two's complement
 * 16L-bit integers (the reference's signed convention via conv_mfft +
 * normalize_planes).  out: RL limb planes of the rows asked for. */
int mfftgpu_mm_u16_dev(mfftgpu_ctx *ctx, const uint16_t *A, const uint16_t *B, int n, int L,
                       int is_signed, uint16_t *out, int RL, int row_begin, int row_end);
int mfftgpu_mm_u16(mfftgpu_ctx *ctx, const uint16_t *A, const uint16_t *B, int n, int L,
                   int is_signed, uint16_t *out, int RL);

/* W <= 64-bit signed entries, row-major int64 (A[i*n + j]). */
int mfftgpu_mm_i64_dev(mfftgpu_ctx *ctx, const int64_t *A, const int64_t *B, int n,
                       uint16_t *out, int RL, int row_begin, int row_end);
int mfftgpu_mm_i64(mfftgpu_ctx *ctx, const int64_t *A, const int64_t *B, int n, uint16_t *out,
                   int RL);

/* Replaces conv_mfft (src/mfft.c:302-422): int32 limb planes with
 * |limb| <= 65535 (the signed-limb convention of src/fpfixed.c:187-192);
 * writes the 2L-1 unnormalised int64 convolution planes
 * Cw[w] = sum_{u+v=w} A_u B_v, bit-identical to the reference. */
int mfftgpu_conv_i32_dev(mfftgpu_ctx *ctx, const int32_t *A32, const int32_t *B32, int n, int L,
                         int64_t *Cw);
int mfftgpu_conv_i32(mfftgpu_ctx *ctx, const int32_t *A32, const int32_t *B32, int n, int L,
                     int64_t *Cw);

/* --- fp32 fixed-point embedding --------------------------------------------
 * fpx_init + fpx_encode + conv + fpx_decode_f32 (src/fpfixed.c:96-285) fused
 * on the device: C = A * B computed exactly on the grid (force_bits > 0:
 * SA = SB = force_bits/2; 0: adaptive grid from the data) and rounded once to
 * fp32.  Row-major fp32 n x n. */
int mfftgpu_fp32_dev(mfftgpu_ctx *ctx, const float *A, const float *B, int n, int force_bits,
                     float *C, int row_begin, int row_end);
int mfftgpu_fp32(mfftgpu_ctx *ctx, const float *A, const float *B, int n, int force_bits,
                 float *C);

/* --- fp64 fixed-point embedding --------------------------------------------
 * fpx_init_d + fpx_encode_d + conv + fpx_decode_f64 (src/fpfixed.c:109-160,
 * 308-322) fused on the device: 53-bit significands on the same grid, each
 * entry touching up to 5 limbs, rounded once to fp64.  Row-major fp64 n x n. */
int mfftgpu_fp64_dev(mfftgpu_ctx *ctx, const double *A, const double *B, int n, int force_bits,
                     double *C, int row_begin, int row_end);
int mfftgpu_fp64(mfftgpu_ctx *ctx, const double *A, const double *B, int n, int force_bits,
                 double *C);

/* Exact product of signed 64-bit row-major matrices, like mfftgpu_mm_i64_dev,
 * but with no device allocation at all: for callers that may not call
 * cudaMalloc (a framework that owns all device memory through its own pool,
 * or a latency-critical path that cannot take cudaMalloc's implicit device
 * synchronisation).  No counterpart in the reference.
 * A, B, out: device pointers the caller allocated (out: RL planes of n*n).
 * Every intermediate lives in one fixed 32 MiB static device array per GPU,
 * held by each GPU that loads the library until the process exits; n > 256
 * does not fit and returns MFFTGPU_ERR_ARG.  The work is enqueued on
 * `stream` (a cudaStream_t; NULL = legacy default stream) on the current
 * device, and the call is synchronous: it waits for that stream to return
 * the status of the device-side checks.  The first call on each device
 * checks the device and looks up the array's device address, once, and
 * keeps both for the life of the device context (after cudaDeviceReset they
 * are stale); make that first call before any stream capture.  All calls
 * share the one array: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller. */
int mfftgpu_mm_i64_noalloc(const int64_t *A, const int64_t *B, int n, uint16_t *out, int RL,
                           void *stream);

/* --- device-side input generators (bench workloads) ------------------------
 * bigmat_rand (src/bigmat.c:20-35) evaluated in parallel: draw i of the
 * splitmix64 stream from `seed` is a pure function of (seed, i). */
int mfftgpu_gen_bigmat_dev(mfftgpu_ctx *ctx, uint16_t *m, int n, int L, uint64_t seed);
int mfftgpu_gen_int64_dev(mfftgpu_ctx *ctx, int64_t *x, size_t count, uint64_t seed);
/* fp32 workload on the host: N(0,1) * 2^k, k uniform in [-8, 8]; one
 * splitmix64 stream, A's entries first, 3 draws per entry (Box-Muller u1, u2,
 * then k).  The reference's ML track only generates U(-1,1)
 * (src/mlgemm.c:657-680). */
void mfftgpu_gen_normal_f32(float *A, float *B, size_t count, uint64_t seed);

/* Self-test of the tcgen05 pointwise kernel: random int8 Ahat/F planes for
 * the given job shape, the kernel's int32 job planes compared element by
 * element with a CUDA-core evaluation of the same job table.  variant: 0 the
 * product path's choice, 1 one CTA per 128-row tile, 2 CTA pairs (256-row
 * tiles, tcgen05 cta_group::2), 3 t-grouped CTA pairs, 4 the Karatsuba job
 * table (K = 8, one digit, one chunk: NB * 12 operand planes per side, NB * 21
 * job planes) on its CTA-pair kernel, 5 the same at level 2 (NB * 16 operand
 * planes, NB * 25 job planes), 6 at level 3 (NB * 18, NB * 27), 7 a
 * digit-sum job table (dA = dB = 3: class w multiplies digit w of A by digit
 * w of B) on the kernel the product path picks for the shape.  *mismatches receives the number of
 * differing elements. */
int mfftgpu_selftest_pointwise(mfftgpu_ctx *ctx, int rows, int cols, int kdim, int NB, int K,
                               int dA, int dB, int nchunk, int block_n, int variant,
                               long long *mismatches);
/* The same check for the schoolbook job table: LbA / LbB random int8 digit
 * planes, chunks of U planes of A, every job (t, ch) with a term compared. */
int mfftgpu_selftest_school(mfftgpu_ctx *ctx, int rows, int cols, int kdim, int LbA, int LbB,
                            int U, long long *mismatches);

/* Self-test of the bounded device waits: launches the pointwise kernel with
 * a producer that never loads, so its consumers must give up after
 * timeout_ns.  Returns MFFTGPU_ERR_TIMEOUT when the timeout path works; the
 * context stays usable afterwards. */
int mfftgpu_selftest_timeout(mfftgpu_ctx *ctx, unsigned long long timeout_ns);

/* host self-tests of the device fp32 / fp64 rounding rules (no GPU needed) */
float mfftgpu_decode_words_f32(uint32_t *words, int nwords, int bit_off, int S);
double mfftgpu_decode_words_f64(uint32_t *words, int nwords, int bit_off, int S);
/* the shared front half of those rules (extract + round_to of
 * src/fpfixed.c:212-265) for any significand width `bits` <= 63: returns 0
 * for zero, else the sign, with value = sig * 2^shift on the grid */
int mfftgpu_decode_words_round(uint32_t *words, int nwords, int bit_off, int bits, uint64_t *sig,
                               int *shift);

#ifdef __cplusplus
}
#endif
#endif
