/* A C program that uses this library through the reference's own API
 * (include/mfftbench_b200.h), the way a caller of the reference's mm_mfft
 * would: benchmark configuration c1 by default (n = 64, W = 8192 unsigned,
 * L = 512 limbs), inputs from bigmat_rand with seeds 12345 and
 * 12345 ^ 0xABCDEF, mfft_plan_init, mm_mfft, then mm_limbplane as an
 * independent product and bigres_equal.  Prints the FNV-1a digest of the
 * mm_mfft output (plane-major uint16) and exits non-zero on any failure.
 *
 *     dropin_c1 [n L]
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "mfftbench_b200.h"

int main(int argc, char **argv)
{
    const int n = argc > 2 ? atoi(argv[1]) : 64;
    const int L = argc > 2 ? atoi(argv[2]) : 512;
    const int RL = 2 * L + 1;
    const size_t nn = (size_t)n * n;
    uint16_t *A = bigmat_alloc(n, L), *B = bigmat_alloc(n, L);
    uint16_t *C = malloc((size_t)RL * nn * sizeof(uint16_t));
    uint16_t *D = malloc((size_t)RL * nn * sizeof(uint16_t));
    if (!A || !B || !C || !D) {
        fprintf(stderr, "out of memory\n");
        return 2;
    }
    bigmat_rand(A, n, L, 12345);
    bigmat_rand(B, n, L, 12345 ^ 0xABCDEF);

    mfft_plan p;
    if (mfft_plan_init(&p, L, 0) != 0) {
        fprintf(stderr, "mfft_plan_init rejected L=%d\n", L);
        return 3;
    }
    mm_mfft(A, B, n, L, &p, KERNEL_PACKED, C, RL);
    if (mfftb_last_status()) return 4;
    mm_limbplane(A, B, n, L, KERNEL_PACKED, D, RL);
    if (mfftb_last_status()) return 5;
    int bi = -1, bj = -1, bw = -1;
    if (!bigres_equal(C, D, n, RL, &bi, &bj, &bw)) {
        fprintf(stderr, "mm_mfft != mm_limbplane at (%d,%d) limb %d\n", bi, bj, bw);
        return 6;
    }
    uint64_t h = 0xcbf29ce484222325ULL;
    for (size_t i = 0; i < (size_t)RL * nn; i++) {
        h ^= C[i];
        h *= 0x100000001b3ULL;
    }
    printf("n=%d L=%d plan S=%d NB=%d K=%d digest %016llx\n", n, L, p.S, p.NB, p.K,
           (unsigned long long)h);
    free(A);
    free(B);
    free(C);
    free(D);
    return 0;
}
