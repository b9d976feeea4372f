/* cli_stub.c -- the one symbol the reference's CLI needs that this
 * repository's library does not provide, for the `cli` target of
 * oracle/Makefile: the reference's exact-track driver (src/main.c, with its
 * methods/kernel/bigmat/roots/fpfixed/mlgemm/lowprec sources, compiled where
 * they lie) linked against libmfftb200.so, whose drop-in mm_mfft / conv_mfft /
 * mfft_plan_init / mfft_plan_maxbits / mfft_profile_* replace src/mfft.c.
 *
 * The recursive MFFT planner (mfft_plan_init_rec, src/mfft.c:486-527) is not
 * built here; returning -1 tells the driver that no recursive plan exists, so
 * it skips its mfft-rec rows (src/main.c:284-291). */
#include <stdint.h>

typedef struct mfft_plan mfft_plan;

int mfft_plan_init_rec(mfft_plan *p, int L, int n, int sigma_override)
{
    (void)p;
    (void)L;
    (void)n;
    (void)sigma_override;
    return -1;
}
