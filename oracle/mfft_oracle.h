/* mfft_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's exact-integer MFFT matmul path
 * (hadilq/mfft-bench src/mfft.c, src/bigmat.c, src/fpfixed.c) used as the
 * checker for the B200 path.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product library never links
 * or calls anything here.
 *
 * Parity pin: every function below is checked in tests/test_oracle.py against
 * (a) golden digests measured by running the reference itself, and (b) the
 * reference's own sources compiled from source into oracle/_ref/.
 */
#ifndef MFFT_ORACLE_H
#define MFFT_ORACLE_H
#include <stdint.h>
#include <stddef.h>

typedef struct { int L, S, NB, K, g; long long nprod; } orc_plan;

uint64_t orc_sm64(uint64_t *state);
void orc_bigmat_rand(uint16_t *m, int n, int L, uint64_t seed);
void orc_gen_signed_planes(uint16_t *m, int n, int L, uint64_t seed);
void orc_gen_int64(int64_t *x, size_t count, uint64_t seed);
void orc_int64_to_planes(const int64_t *x, int n, uint16_t *planes);
void orc_gen_normal_f32(float *A, float *B, size_t count, uint64_t seed);
void orc_planes_to_signlimb(const uint16_t *pl, int n, int L, int32_t *out);
int  orc_plan_init(orc_plan *p, int L, int sigma);
void orc_conv_mfft(int64_t *Cw, const int32_t *A, const int32_t *B, int n, int L,
                   const orc_plan *p);
void orc_conv_limbplane(int64_t *Cw, const int32_t *A, const int32_t *B, int n, int L);
void orc_normalize_planes(const int64_t *acc, int nplanes, int n, uint16_t *out, int RL);
void orc_mm_mfft(const uint16_t *A, const uint16_t *B, int n, int L, const orc_plan *p,
                 uint16_t *out, int RL);
void orc_mm_signed(const uint16_t *A, const uint16_t *B, int n, int L, uint16_t *out, int RL);
void orc_entry_product(const uint16_t *A, const uint16_t *B, int n, int L, int is_signed,
                       int nsamp, const int *rows, const int *cols, uint16_t *out, int RL);
uint64_t orc_digest_u16(const uint16_t *v, size_t count);

typedef struct { int n, L, SA, SB; int32_t *A32, *B32; int64_t *Cw; } orc_fpx;
int  orc_fpx_init(orc_fpx *c, const float *A, const float *B, int n, int force_bits);
void orc_fpx_encode(orc_fpx *c, const float *A, const float *B);
void orc_fpx_decode_f32(const orc_fpx *c, float *C);
void orc_fpx_free(orc_fpx *c);
void orc_fpx_entries(const float *A, const float *B, int n, int force_bits, int nsamp,
                     const int *rows, const int *cols, float *out);
float orc_decode_f32_entry(const int64_t *cw, int L, int S);
double orc_decode_f64_entry(const int64_t *cw, int L, int S);
void orc_fpx64_entries(const double *A, const double *B, int n, int force_bits, int nsamp,
                       const int *rows, const int *cols, double *out);
long long orc_checksum_modp(const void *A, const void *B, int fmt, int n, int L, int is_signed,
                            const uint16_t *C, int RL);

#endif
