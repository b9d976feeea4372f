// pointwise.cu -- persistent, warp-specialised tcgen05 (kind::i8) kernels for
// the plane products (MFFT pointwise step and schoolbook digit-plane
// products); see pointwise.cuh for the job semantics.
//
// All three kernels: warp 0 streams K-major int8 tiles into a shared-memory
// ring with TMA (128-byte swizzle, no multicast), one thread of warp 1 issues
// tcgen05.mma (K = 32 per instruction) into int32 TMEM accumulators, warps
// 2-5 drain them (tcgen05.ld) and store int32 job planes; every wait is
// bounded.  pointwise_launch picks:
//   * pointwise_i8_kernel: one CTA per SM, M = 128, N = block_n, two
//     256-column accumulators (the epilogue overlaps the next tile) -- small n;
//   * pointwise2_i8_kernel: CTA pairs (cta_group::2), 256 x 256 tiles;
//   * pointwise3_i8_kernel: CTA pairs, 256 x 128 tiles of 4 jobs that share
//     their A planes and overlapping F windows, wave-aligned tile order -- the
//     default for one-chunk MFFT plans and the only one for schoolbook plans.
//     It issues only the terms that can be non-zero: at the MFFT points 0 and
//     NB/2 the triangle c1 < K/2, t - c1 < K/2 (pw_point_range), in
//     schoolbook mode the planes that exist (pw_school_range).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>

#include "ptx.cuh"
#include "pointwise.cuh"
#include "runtime.h"

namespace mfftb {

// Tile order.  raster 0: job-major, then groups of group_m row tiles x all
// column tiles.  raster 1: evaluation point j outermost; inside, groups of
// group_m row tiles x all column tiles, and for each (row tile, column tile)
// the NI = K*nW*nchunk jobs of point j back to back -- they read the same A
// rows and overlapping windows of the same F planes, so concurrent CTAs
// share operand tiles in L2.
__device__ __forceinline__ void pw_tile_decode(const PwParams& p, long long tile, int& q, int& mt,
                                               int& nt) {
    const int GM = p.group_m;
    if (p.raster == 0) {
        long long per_job = (long long)p.tiles_m * p.tiles_n;
        q = (int)(tile / per_job);
        int r = (int)(tile % per_job);
        int group = GM * p.tiles_n;
        int g = r / group;
        int first_m = g * GM;
        int gm = p.tiles_m - first_m < GM ? p.tiles_m - first_m : GM;
        int local = r % group;
        mt = first_m + local % gm;
        nt = local / gm;
        return;
    }
    const int NI = p.jobs.K * p.jobs.nW * p.jobs.nchunk;
    const long long per_j = (long long)p.tiles_m * p.tiles_n * NI;
    const int j = (int)(tile / per_j);
    long long r = tile % per_j;
    const long long group = (long long)GM * p.tiles_n * NI;
    const int g = (int)(r / group);
    const int first_m = g * GM;
    const int gm = p.tiles_m - first_m < GM ? p.tiles_m - first_m : GM;
    long long local = r % group;
    const int inner = (int)(local % NI);
    local /= NI;
    mt = first_m + (int)(local % gm);
    nt = (int)(local / gm);
    q = j * NI + inner;
}

__global__ void __launch_bounds__(PW_THREADS, 1)
    pointwise_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmF, const PwParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + PW_STAGES * PW_A_STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + PW_STAGES * PW_B_STAGE_BYTES);
    // bars[0..S): full, [S..2S): empty, [2S..2S+2): tmem full, [2S+2..2S+4): tmem empty,
    // [2S+4]: drain
    const uint32_t bar_full = smem_u32(bars);
    const uint32_t bar_empty = smem_u32(bars + PW_STAGES);
    const uint32_t bar_tfull = smem_u32(bars + 2 * PW_STAGES);
    const uint32_t bar_tempty = smem_u32(bars + 2 * PW_STAGES + 2);
    const uint32_t bar_drain = smem_u32(bars + 2 * PW_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * PW_STAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PW_STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 128);
        }
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmF);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), PW_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const unsigned long long tmo = p.timeout_ns;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer
        int stage = 0;
        uint32_t phase = 0;
        int issued_parity[PW_STAGES];
        for (int s = 0; s < PW_STAGES; ++s) issued_parity[s] = -1;
        const uint32_t tx_bytes = PW_A_STAGE_BYTES + p.block_n * PW_BK;
        // stall_producer: nothing is ever loaded, so every consumer wait must
        // run into its deadline and the kernel must still end cleanly
        const long long first_tile = p.stall_producer ? p.num_tiles : (long long)blockIdx.x;
        for (long long tile = first_tile; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            for (int s = s0; s < s1; ++s) {
                int pa, pf;
                pw_segment_planes(p.jobs, j, t, w, s, pa, pf);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                                           global_timer_ns() + tmo))
                        goto producer_done;
                    mbar_arrive_expect_tx(bar_full + 8 * stage, tx_bytes);
                    tma_load_3d(smem_u32(sA + stage * PW_A_STAGE_BYTES), &tmA, bar_full + 8 * stage,
                                kb * PW_BK, mt * PW_BM, pa);
                    tma_load_3d(smem_u32(sB + stage * PW_B_STAGE_BYTES), &tmF, bar_full + 8 * stage,
                                kb * PW_BK, nt * p.block_n, pf);
                    issued_parity[stage] = (int)phase;
                    if (++stage == PW_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    producer_done:
        // Every TMA load this thread issued must have landed before the CTA
        // may exit (its shared memory is the destination).
        for (int s = 0; s < PW_STAGES; ++s)
            if (issued_parity[s] >= 0)
                if (!mbar_wait_deadline(bar_full + 8 * s, (uint32_t)issued_parity[s],
                                        global_timer_ns() + tmo))
                    *abort_flag = 1;
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------ MMA issuer
        const uint32_t idesc = idesc_i8(PW_BM, p.block_n);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (long long tile = blockIdx.x; tile < p.num_tiles && !*abort_flag; tile += gridDim.x) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            const int nsteps = (s1 - s0) * p.kblocks;
            if (!mbar_wait_bounded(bar_tempty + 8 * acc, acc_phase ^ 1, abort_flag,
                                   global_timer_ns() + tmo))
                break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
            for (int it = 0; it < nsteps; ++it) {
                if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag,
                                       global_timer_ns() + tmo))
                    goto mma_done;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + stage * PW_A_STAGE_BYTES);
                const uint32_t b0 = smem_u32(sB + stage * PW_B_STAGE_BYTES);
#pragma unroll
                for (int kk = 0; kk < PW_BK / 32; ++kk) {
                    mma_i8(d_tmem, sdesc_kmajor_sw128(a0 + kk * 32), sdesc_kmajor_sw128(b0 + kk * 32),
                           idesc, (it | kk) != 0 ? 1u : 0u);
                }
                mma_commit(bar_empty + 8 * stage);
                if (++stage == PW_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit(bar_tfull + 8 * acc);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    mma_done:
        // all MMAs issued by this thread complete before TMEM is released
        mma_commit(bar_drain);
        if (!mbar_wait_deadline(bar_drain, 0, global_timer_ns() + tmo)) *abort_flag = 1;
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        int acc = 0;
        uint32_t acc_phase = 0;
        for (long long tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            if (!mbar_wait_bounded(bar_tfull + 8 * acc, acc_phase, abort_flag,
                                   global_timer_ns() + tmo))
                break;
            tc_fence_after();
            const bool empty_job = (s1 <= s0);
            const int row = mt * PW_BM + quarter * 32 + lane;
            const int col0 = nt * p.block_n;
            int32_t* orow = p.out + (long long)q * p.out_plane + (long long)row * p.ldo + col0;
            const int colmax = p.cols - col0;
            for (int c = 0; c < p.block_n / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                       (uint32_t)(acc * 256 + c * 32),
                                   v);
                tmem_ld_wait();
                if (row < p.rows) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        const int col = c * 32 + e;
                        if (col < colmax) {
                            int4 o;
                            o.x = empty_job ? 0 : (int)v[e];
                            o.y = empty_job ? 0 : (int)v[e + 1];
                            o.z = empty_job ? 0 : (int)v[e + 2];
                            o.w = empty_job ? 0 : (int)v[e + 3];
                            *reinterpret_cast<int4*>(orow + col) = o;
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(bar_tempty + 8 * acc);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicCAS(p.err, 0, MFFTB_ERR_TIMEOUT);
    if (warp == 1) tmem_dealloc(tmem_base, PW_TMEM_COLS);
}

// ---------------------------------------------------------------- CTA-pair variant
// Same job table, tiles of 256 rows x 256 columns per CTA pair (a cluster of
// two CTAs on two SMs).  The leader CTA issues tcgen05.mma.cta_group::2
// (M = 256, N = 256): A rows 0-127 come from the leader's shared memory and
// 128-255 from the peer's; the 256 B rows (output columns) are split 128/128
// the same way, so each SM streams 32 KB per 128-byte k-step instead of 48 KB
// for the same MACs, and the ring is 6 stages deep.  Each CTA's TMEM holds
// its 128 output rows.  Both CTAs' TMA loads complete on the leader's "full"
// barrier; the leader's commits arrive on both CTAs' "empty" / "TMEM full"
// barriers; both epilogues arrive on the leader's "TMEM empty" barrier.
constexpr int PW2_STAGES = 6;
constexpr int PW2_BN = 256;
constexpr int PW2_A_BYTES = 128 * PW_BK;
constexpr int PW2_B_BYTES = (PW2_BN / 2) * PW_BK;
constexpr int PW2_SMEM_BYTES = 1024 + PW2_STAGES * (PW2_A_BYTES + PW2_B_BYTES) + 256;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PW_THREADS, 1)
    pointwise2_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmF, const PwParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + PW2_STAGES * PW2_A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + PW2_STAGES * PW2_B_BYTES);
    const uint32_t bar_full = smem_u32(bars);
    const uint32_t bar_empty = smem_u32(bars + PW2_STAGES);
    const uint32_t bar_tfull = smem_u32(bars + 2 * PW2_STAGES);
    const uint32_t bar_tempty = smem_u32(bars + 2 * PW2_STAGES + 2);
    const uint32_t bar_drain = smem_u32(bars + 2 * PW2_STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * PW2_STAGES + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const long long pair = blockIdx.x >> 1;
    const long long npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PW2_STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(bar_tfull + 8 * a, 1);
            mbar_init(bar_tempty + 8 * a, 2 * 128);
        }
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmF);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), PW_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // barrier inits and TMEM allocation visible to the pair
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const unsigned long long tmo = p.timeout_ns;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        int issued_parity[PW2_STAGES];
        for (int s = 0; s < PW2_STAGES; ++s) issued_parity[s] = -1;
        const uint32_t tx_bytes = 2 * (PW2_A_BYTES + PW2_B_BYTES);
        const long long first_tile = p.stall_producer ? p.num_tiles : pair;
        for (long long tile = first_tile; tile < p.num_tiles && !*abort_flag; tile += npairs) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            for (int s = s0; s < s1; ++s) {
                int pa, pf;
                pw_segment_planes(p.jobs, j, t, w, s, pa, pf);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                                           global_timer_ns() + tmo))
                        goto producer_done;
                    const uint32_t full_leader = mapa_shared(bar_full + 8 * stage, 0);
                    if (leader) mbar_arrive_expect_tx(bar_full + 8 * stage, tx_bytes);
                    tma_load_3d_pair(smem_u32(sA + stage * PW2_A_BYTES), &tmA, full_leader,
                                     kb * PW_BK, mt * 256 + (int)rank * 128, pa);
                    tma_load_3d_pair(smem_u32(sB + stage * PW2_B_BYTES), &tmF, full_leader,
                                     kb * PW_BK, nt * PW2_BN + (int)rank * (PW2_BN / 2), pf);
                    issued_parity[stage] = (int)phase;
                    if (++stage == PW2_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    producer_done:
        // every stage this CTA loaded is consumed by the pair's MMA (which
        // implies the load landed) before the CTA may leave
        for (int s = 0; s < PW2_STAGES; ++s)
            if (issued_parity[s] >= 0)
                if (!mbar_wait_deadline(bar_empty + 8 * s, (uint32_t)issued_parity[s],
                                        global_timer_ns() + tmo))
                    *abort_flag = 1;
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------ MMA issuer (leader only)
        const uint32_t idesc = idesc_i8(256, PW2_BN);
        int stage = 0;
        uint32_t phase = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles && !*abort_flag; tile += npairs) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            const int nsteps = (s1 - s0) * p.kblocks;
            if (!mbar_wait_bounded(bar_tempty + 8 * acc, acc_phase ^ 1, abort_flag,
                                   global_timer_ns() + tmo))
                break;
            tc_fence_after();
            const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
            for (int it = 0; it < nsteps; ++it) {
                if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag,
                                       global_timer_ns() + tmo))
                    goto mma_done;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + stage * PW2_A_BYTES);
                const uint32_t b0 = smem_u32(sB + stage * PW2_B_BYTES);
#pragma unroll
                for (int kk = 0; kk < PW_BK / 32; ++kk) {
                    mma_i8_pair(d_tmem, sdesc_kmajor_sw128(a0 + kk * 32),
                                sdesc_kmajor_sw128(b0 + kk * 32), idesc, (it | kk) != 0 ? 1u : 0u);
                }
                mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
                if (++stage == PW2_STAGES) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit_pair_mc(bar_tfull + 8 * acc, 0x3);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    mma_done:
        mma_commit_pair(bar_drain);
        if (!mbar_wait_deadline(bar_drain, 0, global_timer_ns() + tmo)) *abort_flag = 1;
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles; tile += npairs) {
            int q, mt, nt, j, t, w, ch, s0, s1;
            pw_tile_decode(p, tile, q, mt, nt);
            pw_job_decode(p.jobs, q, j, t, w, ch);
            pw_chunk_range(p.jobs, w, ch, s0, s1);
            if (!mbar_wait_bounded(bar_tfull + 8 * acc, acc_phase, abort_flag,
                                   global_timer_ns() + tmo))
                break;
            tc_fence_after();
            const bool empty_job = (s1 <= s0);
            const int row = mt * 256 + (int)rank * 128 + quarter * 32 + lane;
            const int col0 = nt * PW2_BN;
            int32_t* orow = p.out + (long long)q * p.out_plane + (long long)row * p.ldo + col0;
            const int colmax = p.cols - col0;
            for (int c = 0; c < PW2_BN / 32; ++c) {
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                       (uint32_t)(acc * 256 + c * 32),
                                   v);
                tmem_ld_wait();
                if (row < p.rows) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        const int col = c * 32 + e;
                        if (col < colmax) {
                            int4 o;
                            o.x = empty_job ? 0 : (int)v[e];
                            o.y = empty_job ? 0 : (int)v[e + 1];
                            o.z = empty_job ? 0 : (int)v[e + 2];
                            o.w = empty_job ? 0 : (int)v[e + 3];
                            *reinterpret_cast<int4*>(orow + col) = o;
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(mapa_shared(bar_tempty + 8 * acc, 0));
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // neither CTA leaves while the pair may still signal it
    tc_fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicCAS(p.err, 0, MFFTB_ERR_TIMEOUT);
    if (warp == 1) tmem_dealloc_pair(tmem_base, PW_TMEM_COLS);
}

// ---------------------------------------------------------------- t-grouped CTA-pair variant
// For plans with one contraction chunk and K a multiple of 4.  A tile group
// is (point j, digit-weight class w, t0..t0+3); its stages walk the class's
// digit pairs (da, db) in turn.  The K jobs
// (j, t) of one evaluation point share their A operand (Ahat_j, all c1) and
// read overlapping windows of the F stack (plane K-1-t+c1).  A CTA pair
// computes 4 of them at once -- t = t0..t0+3, one 256 x 128 TMEM accumulator
// each (4 x 128 = 512 columns) -- from stages that hold 2 consecutive c1
// planes of A (2 x 16 KB per CTA) and the 5 F planes those 8 (c1, t) pairs
// need (5 x 8 KB): 72 KB per stage feed 32 pair MMAs (256 x 128 x 32), so
// every operand byte loaded into shared memory is used 3.2 times on average
// instead of once.  At the half points (pw_half_point) a stage whose eight
// (c1, t) slots all hold zero terms is skipped, the other stages load and
// multiply only the planes of their possibly non-zero terms, and the
// epilogue writes a job without terms (t = K-1) as zeros.
constexpr int PW3_STAGES = 3;
constexpr int PW3_TG = 4;             // jobs per tile group
constexpr int PW3_CPS = 2;            // c1 planes per stage
constexpr int PW3_NF = PW3_TG + PW3_CPS - 1;
constexpr int PW3_BN = 128;           // output columns per pair tile (MMA N)
constexpr int PW3_A_BYTES = 128 * PW_BK;             // one A plane tile per CTA
constexpr int PW3_F_BYTES = (PW3_BN / 2) * PW_BK;    // one F plane half-tile per CTA
constexpr int PW3_STAGE_BYTES = PW3_CPS * PW3_A_BYTES + PW3_NF * PW3_F_BYTES;
constexpr int PW3_SMEM_BYTES = 1024 + PW3_STAGES * PW3_STAGE_BYTES + 256;

__device__ __forceinline__ void pw3_tile_decode(const PwParams& p, long long tile, int& j, int& w,
                                                int& t0, int& mt, int& nt) {
    const int ngroups = p.jobs.K / PW3_TG;
    const long long per_sj = (long long)p.tiles_m * p.tiles_n;
    const int sj = (int)(tile / per_sj);
    const int r = (int)(tile % per_sj);
    const int GM = p.group_m;
    const int group = GM * p.tiles_n;
    const int g = r / group;
    const int first_m = g * GM;
    const int gm = p.tiles_m - first_m < GM ? p.tiles_m - first_m : GM;
    const int local = r % group;
    mt = first_m + local % gm;
    nt = local / gm;
    if (p.jobs.school) {  // group sj = (t group, chunk); w carries the chunk
        j = 0;
        w = sj % p.jobs.nchunk;
        t0 = (sj / p.jobs.nchunk) * PW3_TG;
        return;
    }
    j = sj / (p.jobs.nW * ngroups);
    const int rem = sj % (p.jobs.nW * ngroups);
    w = rem / ngroups;
    t0 = (rem % ngroups) * PW3_TG;
}

// Schoolbook tile (t0..t0+3, chunk ch): the union [lo, hi] of its jobs' u
// ranges, walked in pairs of u per pipeline stage; returns the pair count.
__device__ __forceinline__ int pw3_school_pairs(const PwJobs& J, int t0, int ch, int& lo) {
    int l0, h0, l3, h3;
    pw_school_range(J, t0, ch, l0, h0);
    pw_school_range(J, t0 + PW3_TG - 1, ch, l3, h3);
    lo = l0;
    const int hi = h3;  // lo grows and hi grows with t: the union is [lo(t0), hi(t0+3)]
    return hi >= lo ? (hi - lo + 2) / 2 : 0;
}

// Which planes stage c (c1 = c, c+1) of a tile must load: bit cc of needA for
// A plane c + cc, bit f of needF for F slot f, from the slots (tt, cc) whose
// term can be non-zero (c + cc in [lo[tt], hi[tt]]).  The MMA thread applies
// the same test slot by slot; a stage with needA == 0 is skipped by both.
__device__ __forceinline__ void pw3_stage_need(const int (&lo)[PW3_TG], const int (&hi)[PW3_TG],
                                               int c, uint32_t& needA, uint32_t& needF) {
    needA = 0;
    needF = 0;
#pragma unroll
    for (int cc = 0; cc < PW3_CPS; ++cc)
#pragma unroll
        for (int tt = 0; tt < PW3_TG; ++tt)
            if (c + cc >= lo[tt] && c + cc <= hi[tt]) {
                needA |= 1u << cc;
                needF |= 1u << (PW3_TG - 1 - tt + cc);
            }
}

// MFFT tile (j, t0..t0+3): the c1 range of each job (everything at an
// ordinary point, the triangle of possibly non-zero terms at a half point)
__device__ __forceinline__ void pw3_point_ranges(const PwJobs& J, int j, int t0,
                                                 int (&lo)[PW3_TG], int (&hi)[PW3_TG]) {
#pragma unroll
    for (int tt = 0; tt < PW3_TG; ++tt) pw_point_range(J, j, t0 + tt, lo[tt], hi[tt]);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PW_THREADS, 1)
    pointwise3_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmF, const PwParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PW3_STAGES * PW3_STAGE_BYTES);
    const uint32_t bar_full = smem_u32(bars);
    const uint32_t bar_empty = smem_u32(bars + PW3_STAGES);
    const uint32_t bar_tfull = smem_u32(bars + 2 * PW3_STAGES);
    const uint32_t bar_tempty = smem_u32(bars + 2 * PW3_STAGES + 1);
    const uint32_t bar_drain = smem_u32(bars + 2 * PW3_STAGES + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * PW3_STAGES + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const long long pair = blockIdx.x >> 1;
    const long long npairs = gridDim.x >> 1;
    const int K = p.jobs.K;
    const int cps_per_kb = K / PW3_CPS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PW3_STAGES; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_tfull, 1);
        mbar_init(bar_tempty, 2 * 128);
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmF);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), PW_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const unsigned long long tmo = p.timeout_ns;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        int issued_parity[PW3_STAGES];
        for (int s = 0; s < PW3_STAGES; ++s) issued_parity[s] = -1;
        const long long first_tile = p.stall_producer ? p.num_tiles : pair;
        bool align = p.wave_counter != nullptr;
        long long wave = 0;
        for (long long tile = first_tile; tile < p.num_tiles && !*abort_flag;
             tile += npairs, ++wave) {
            if (align && (wave + 1) * npairs <= p.num_tiles) {
                atomicAdd(p.wave_counter, 1u);
                const unsigned target = gridDim.x * (unsigned)(wave + 1);
                const uint64_t dl = global_timer_ns() + 2000000ull;  // 2 ms
                while (*reinterpret_cast<volatile unsigned*>(p.wave_counter) < target) {
                    if (global_timer_ns() > dl) {
                        align = false;  // give up aligning; never wait again
                        break;
                    }
                }
            }
            int j, w, t0, mt, nt;
            pw3_tile_decode(p, tile, j, w, t0, mt, nt);
            if (p.jobs.school) {
                int ulo;
                const int npairs_u = pw3_school_pairs(p.jobs, t0, w, ulo);
                int rlo[PW3_TG], rhi[PW3_TG];
#pragma unroll
                for (int tt = 0; tt < PW3_TG; ++tt) pw_school_range(p.jobs, t0 + tt, w, rlo[tt], rhi[tt]);
                for (int cp = 0; cp < npairs_u; ++cp) {
                    const int c = ulo + 2 * cp;
                    // only the planes some valid (t, u) slot of this stage reads are
                    // loaded (the MMA thread applies the same validity test)
                    uint32_t needA = 0, needF = 0;
#pragma unroll
                    for (int cc = 0; cc < PW3_CPS; ++cc)
#pragma unroll
                        for (int tt = 0; tt < PW3_TG; ++tt)
                            if (c + cc >= rlo[tt] && c + cc <= rhi[tt]) {
                                needA |= 1u << cc;
                                needF |= 1u << (PW3_TG - 1 - tt + cc);
                            }
                    const uint32_t stage_tx =
                        2u * ((uint32_t)__popc(needA) * PW3_A_BYTES + (uint32_t)__popc(needF) * PW3_F_BYTES);
                    for (int kb = 0; kb < p.kblocks; ++kb) {
                        if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                                               global_timer_ns() + tmo))
                            goto producer_done;
                        const uint32_t full_leader = mapa_shared(bar_full + 8 * stage, 0);
                        if (leader) mbar_arrive_expect_tx(bar_full + 8 * stage, stage_tx);
                        uint8_t* st = smem + stage * PW3_STAGE_BYTES;
                        // A planes c, c+1; B planes t0+3-c-f in slot f (out-of-range
                        // plane coordinates load zeros)
#pragma unroll
                        for (int cc = 0; cc < PW3_CPS; ++cc)
                            if (needA & (1u << cc))
                                tma_load_3d_pair(smem_u32(st + cc * PW3_A_BYTES), &tmA, full_leader,
                                                 kb * PW_BK, mt * 256 + (int)rank * 128, c + cc);
#pragma unroll
                        for (int f = 0; f < PW3_NF; ++f)
                            if (needF & (1u << f))
                                tma_load_3d_pair(
                                    smem_u32(st + PW3_CPS * PW3_A_BYTES + f * PW3_F_BYTES), &tmF,
                                    full_leader, kb * PW_BK, nt * PW3_BN + (int)rank * (PW3_BN / 2),
                                    t0 + PW3_TG - 1 - c - f);
                        issued_parity[stage] = (int)phase;
                        if (++stage == PW3_STAGES) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
                continue;
            }
            int plo[PW3_TG], phi[PW3_TG];
            pw3_point_ranges(p.jobs, j, t0, plo, phi);
            const int npr = pw_class_pairs(p.jobs, w);
            for (int pi = 0; pi < npr; ++pi) {
            const int da = pw_class_first_da(p.jobs, w) + pi, db = pw_class_db(p.jobs, w, da);
            const int a_base = (j * p.jobs.dA + da) * K;            // Ahat planes (j, da, .)
            const int f_base = (j * p.jobs.dB + db) * (2 * K - 1);  // F planes (j, db, .)
            for (int cp = 0; cp < cps_per_kb; ++cp) {
                const int c = cp * PW3_CPS;
                const int p_lo = K - PW3_TG - t0 + c;
                uint32_t needA, needF;  // all planes at an ordinary point
                pw3_stage_need(plo, phi, c, needA, needF);
                if (needA == 0) continue;  // every term of the stage is zero (half point)
                const uint32_t stage_tx =
                    2u * ((uint32_t)__popc(needA) * PW3_A_BYTES + (uint32_t)__popc(needF) * PW3_F_BYTES);
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                                           global_timer_ns() + tmo))
                        goto producer_done;
                    const uint32_t full_leader = mapa_shared(bar_full + 8 * stage, 0);
                    if (leader) mbar_arrive_expect_tx(bar_full + 8 * stage, stage_tx);
                    uint8_t* st = smem + stage * PW3_STAGE_BYTES;
#pragma unroll
                    for (int cc = 0; cc < PW3_CPS; ++cc)
                        if (needA & (1u << cc))
                            tma_load_3d_pair(smem_u32(st + cc * PW3_A_BYTES), &tmA, full_leader,
                                             kb * PW_BK, mt * 256 + (int)rank * 128, a_base + c + cc);
#pragma unroll
                    for (int f = 0; f < PW3_NF; ++f)
                        if (needF & (1u << f))
                            tma_load_3d_pair(
                                smem_u32(st + PW3_CPS * PW3_A_BYTES + f * PW3_F_BYTES), &tmF,
                                full_leader, kb * PW_BK, nt * PW3_BN + (int)rank * (PW3_BN / 2),
                                f_base + p_lo + f);
                    issued_parity[stage] = (int)phase;
                    if (++stage == PW3_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            }
        }
    producer_done:
        for (int s = 0; s < PW3_STAGES; ++s)
            if (issued_parity[s] >= 0)
                if (!mbar_wait_deadline(bar_empty + 8 * s, (uint32_t)issued_parity[s],
                                        global_timer_ns() + tmo))
                    *abort_flag = 1;
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------ MMA issuer (leader only)
        const uint32_t idesc = idesc_i8(256, PW3_BN);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles && !*abort_flag; tile += npairs) {
            int j, w, t0, mt, nt;
            pw3_tile_decode(p, tile, j, w, t0, mt, nt);
            int ulo = 0;
            int plo[PW3_TG], phi[PW3_TG];
            int steps_per_tile;
            if (p.jobs.school) {
                steps_per_tile = pw3_school_pairs(p.jobs, t0, w, ulo) * p.kblocks;
            } else {
                pw3_point_ranges(p.jobs, j, t0, plo, phi);
                int live = 0;
                for (int cp = 0; cp < cps_per_kb; ++cp) {
                    uint32_t needA, needF;
                    pw3_stage_need(plo, phi, cp * PW3_CPS, needA, needF);
                    live += needA != 0;
                }
                steps_per_tile = pw_class_pairs(p.jobs, w) * live * p.kblocks;
            }
            if (steps_per_tile == 0) continue;  // tile without terms
            if (!mbar_wait_bounded(bar_tempty, acc_phase ^ 1, abort_flag, global_timer_ns() + tmo))
                break;
            tc_fence_after();
            if (p.jobs.school) {
                int rlo[PW3_TG], rhi[PW3_TG];
#pragma unroll
                for (int tt = 0; tt < PW3_TG; ++tt) pw_school_range(p.jobs, t0 + tt, w, rlo[tt], rhi[tt]);
                uint32_t started = 0;
                for (int it = 0; it < steps_per_tile; ++it) {
                    if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag,
                                           global_timer_ns() + tmo))
                        goto mma_done;
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + stage * PW3_STAGE_BYTES);
                    const int c = ulo + 2 * (it / p.kblocks);
#pragma unroll
                    for (int cc = 0; cc < PW3_CPS; ++cc) {
#pragma unroll
                        for (int tt = 0; tt < PW3_TG; ++tt) {
                            const int u = c + cc;
                            if (u < rlo[tt] || u > rhi[tt]) continue;  // zero or foreign term
                            const int fi = PW3_TG - 1 - tt + cc;       // B plane t0+tt-u
                            const uint32_t a0 = st + cc * PW3_A_BYTES;
                            const uint32_t b0 = st + PW3_CPS * PW3_A_BYTES + fi * PW3_F_BYTES;
                            const uint32_t acc_on = (started >> tt) & 1u;
#pragma unroll
                            for (int kk = 0; kk < PW_BK / 32; ++kk)
                                mma_i8_pair(tmem_base + (uint32_t)(tt * PW3_BN),
                                            sdesc_kmajor_sw128(a0 + kk * 32),
                                            sdesc_kmajor_sw128(b0 + kk * 32), idesc,
                                            (acc_on | (uint32_t)kk) != 0 ? 1u : 0u);
                            started |= 1u << tt;
                        }
                    }
                    mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
                    if (++stage == PW3_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                mma_commit_pair_mc(bar_tfull, 0x3);
                acc_phase ^= 1;
                continue;
            }
            {
            // same stage walk as the producer: class pairs, c1 pairs with a
            // possibly non-zero term, contraction blocks
            const int npr = pw_class_pairs(p.jobs, w);
            uint32_t started = 0;
            for (int pi = 0; pi < npr; ++pi)
            for (int cp = 0; cp < cps_per_kb; ++cp) {
                const int c = cp * PW3_CPS;
                uint32_t needA, needF;
                pw3_stage_need(plo, phi, c, needA, needF);
                if (needA == 0) continue;
                for (int kb = 0; kb < p.kblocks; ++kb) {
                    if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag,
                                           global_timer_ns() + tmo))
                        goto mma_done;
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + stage * PW3_STAGE_BYTES);
#pragma unroll
                    for (int cc = 0; cc < PW3_CPS; ++cc) {
#pragma unroll
                        for (int tt = 0; tt < PW3_TG; ++tt) {
                            if (c + cc < plo[tt] || c + cc > phi[tt]) continue;  // zero term
                            const int fi = PW3_TG - 1 - tt + cc;  // F plane K-1-(t0+tt)+(c+cc) - p_lo
                            const uint32_t a0 = st + cc * PW3_A_BYTES;
                            const uint32_t b0 = st + PW3_CPS * PW3_A_BYTES + fi * PW3_F_BYTES;
                            const uint32_t acc_on = (started >> tt) & 1u;
#pragma unroll
                            for (int kk = 0; kk < PW_BK / 32; ++kk)
                                mma_i8_pair(tmem_base + (uint32_t)(tt * PW3_BN),
                                            sdesc_kmajor_sw128(a0 + kk * 32),
                                            sdesc_kmajor_sw128(b0 + kk * 32), idesc,
                                            (acc_on | (uint32_t)kk) != 0 ? 1u : 0u);
                            started |= 1u << tt;
                        }
                    }
                    mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
                    if (++stage == PW3_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            }
            mma_commit_pair_mc(bar_tfull, 0x3);
            acc_phase ^= 1;
        }
    mma_done:
        mma_commit_pair(bar_drain);
        if (!mbar_wait_deadline(bar_drain, 0, global_timer_ns() + tmo)) *abort_flag = 1;
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles; tile += npairs) {
            int j, w, t0, mt, nt;
            pw3_tile_decode(p, tile, j, w, t0, mt, nt);
            int plo[PW3_TG], phi[PW3_TG];
            bool any = true;  // the MMA thread accumulated something for this tile
            if (p.jobs.school) {
                int ulo;
                if (pw3_school_pairs(p.jobs, t0, w, ulo) == 0) continue;
            } else {
                pw3_point_ranges(p.jobs, j, t0, plo, phi);
                any = false;
#pragma unroll
                for (int tt = 0; tt < PW3_TG; ++tt) any |= plo[tt] <= phi[tt];
            }
            if (any) {
                if (!mbar_wait_bounded(bar_tfull, acc_phase, abort_flag, global_timer_ns() + tmo))
                    break;
                tc_fence_after();
            }
            const int row = mt * 256 + (int)rank * 128 + quarter * 32 + lane;
            const int col0 = nt * PW3_BN;
            const int colmax = p.cols - col0;
            for (int tt = 0; tt < PW3_TG; ++tt) {
                int q = (j * K + t0 + tt) * p.jobs.nW + w;  // job (j, t, w), one chunk
                if (p.jobs.school) {
                    int lo, hi;
                    pw_school_range(p.jobs, t0 + tt, w, lo, hi);
                    if (lo > hi) continue;  // no term: the plane is never read
                    q = (t0 + tt) * p.jobs.nchunk + w;
                }
                // an MFFT job without terms (t > K - 2 at a half point) is a zero plane
                const bool zero = !p.jobs.school && plo[tt] > phi[tt];
                int32_t* orow = p.out + (long long)q * p.out_plane + (long long)row * p.ldo + col0;
                for (int c = 0; c < PW3_BN / 32; ++c) {
                    uint32_t v[32];
                    if (zero) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = 0u;
                    } else {
                        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                               (uint32_t)(tt * PW3_BN + c * 32),
                                           v);
                        tmem_ld_wait();
                    }
                    if (row < p.rows) {
#pragma unroll
                        for (int e = 0; e < 32; e += 4) {
                            const int col = c * 32 + e;
                            if (col < colmax) {
                                int4 o;
                                o.x = (int)v[e];
                                o.y = (int)v[e + 1];
                                o.z = (int)v[e + 2];
                                o.w = (int)v[e + 3];
                                *reinterpret_cast<int4*>(orow + col) = o;
                            }
                        }
                    }
                }
            }
            if (any) {
                tc_fence_before();
                mbar_arrive_cluster(mapa_shared(bar_tempty, 0));
                acc_phase ^= 1;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    tc_fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicCAS(p.err, 0, MFFTB_ERR_TIMEOUT);
    if (warp == 1) tmem_dealloc_pair(tmem_base, PW_TMEM_COLS);
}

// ---------------------------------------------------------------- Karatsuba CTA-pair variant
// Karatsuba mode (PwJobs::kara): the ring product of point j is three full
// convolutions of length 4 (P0 = a0*b0, P1 = a1*b1, P2 = (a0+a1)*(b0+b1);
// half points P0 only), 16 plane products each, instead of the 64 of the
// negacyclic product.  A tile group is (j, p, half): the "lo" half computes
// output coefficients s = 0..3 of product p (the 10 terms u + v <= 3), the
// "hi" half s = 4..6 (the 6 terms u + v >= 4, u, v in 1..3), so every
// multiply of a stage holds a term: a stage loads the 4 (lo) or 3 (hi) A
// planes and as many B planes of the product and issues all of its terms,
// one 256 x 128 accumulator per output coefficient.
constexpr int PWK_BN = 128;           // output columns per pair tile (MMA N)
// warp 0 TMA producer, warp 1 MMA issuer, warps 2-9 epilogue: two warps per
// 32-lane TMEM quarter, each draining 64 of an accumulator's 128 columns, so
// the tensor pipe waits half as long between tiles
constexpr int PWK_EPI_WARPS = 8;
constexpr int PWK_THREADS = 32 * (2 + PWK_EPI_WARPS);
// 192 KB of stages per CTA: two of 4 A plane tiles (128 rows) and 4 B
// half-tiles (64 columns) of 128 contraction bytes, or, for tiles of
// length-2 convolutions only, four of 2 + 2.  (Four 48 KB stages of 64
// contraction bytes with 64-byte swizzling were measured slower for the
// mixed tile kinds.)
constexpr int PWK_A_BYTES = 128 * PW_BK;
constexpr int PWK_B_BYTES = (PWK_BN / 2) * PW_BK;
constexpr int PWK_SMEM_BYTES = 1024 + 8 * (PWK_A_BYTES + PWK_B_BYTES) + 256;

// A tile group of the Karatsuba kernel: kind 0 ("lo", 4 + 4 planes, output
// coefficients 0..3 of a length-4 convolution), 1 ("hi", 3 + 3 planes,
// coefficients 4..6) or 2 (a length-2 convolution of kara = 2: 2 + 2 planes,
// coefficients 0..2, two k-blocks per stage); abase is its first operand
// plane, qbase its first job plane.
__device__ __forceinline__ void pwk_tile_decode(const PwParams& p, long long tile, int& kind,
                                                int& abase, int& qbase, int& mt, int& nt) {
    const long long per_sj = (long long)p.tiles_m * p.tiles_n;
    int sj = (int)(tile / per_sj);
    const int r = (int)(tile % per_sj);
    const int GM = p.group_m;
    const int group = GM * p.tiles_n;
    const int g = r / group;
    const int first_m = g * GM;
    const int gm = p.tiles_m - first_m < GM ? p.tiles_m - first_m : GM;
    const int local = r % group;
    mt = first_m + local % gm;
    nt = local / gm;
    int j;
    for (j = 0; j < p.jobs.NB; ++j) {
        const int ng = pw_kara_point_groups(p.jobs, pw_kara_half(p.jobs, j));
        if (sj < ng) break;
        sj -= ng;
    }
    if (p.jobs.kara >= 2) {
        const int ops = pw_kara_ops(p.jobs), nq = pw_kara_jobs(p.jobs);
        if (sj < 6 || p.jobs.kara == 3) {
            kind = 2;
            abase = j * ops + pw_kara2_qplane(sj);
            qbase = j * nq + 3 * sj;
        } else {
            kind = sj - 6;
            abase = j * ops + 8 + kind;
            qbase = j * nq + 18 + 4 * kind;
        }
    } else {
        kind = sj & 1;
        abase = j * PWK_OPS + 4 * (sj >> 1) + kind;
        qbase = j * PWK_JOBS + 7 * (sj >> 1) + 4 * kind;
    }
}

// NSTAGE = 2: stages of 4 + 4 plane slots (96 KB), every tile kind (the
// default); NSTAGE = 4: stages of 2 + 2 slots (48 KB, one k-block), length-2
// convolution tiles only (kara = 3): three stages in flight while one is
// multiplied, but half the MMAs per barrier round trip.
template <int NSTAGE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PWK_THREADS, 1)
    pointwise_kara_i8_kernel(const __grid_constant__ CUtensorMap tmA,
                             const __grid_constant__ CUtensorMap tmB, const PwParams p) {
    constexpr int NS = 8 / NSTAGE;                                // slots per side and stage
    constexpr int STAGE_BYTES = NS * (PWK_A_BYTES + PWK_B_BYTES);
    constexpr int QK = NS / 2;  // k-blocks per stage of a length-2 convolution tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE_BYTES);
    const uint32_t bar_full = smem_u32(bars);
    const uint32_t bar_empty = smem_u32(bars + NSTAGE);
    const uint32_t bar_tfull = smem_u32(bars + 2 * NSTAGE);
    const uint32_t bar_tempty = smem_u32(bars + 2 * NSTAGE + 1);
    const uint32_t bar_drain = smem_u32(bars + 2 * NSTAGE + 2);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NSTAGE + 3);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const long long pair = blockIdx.x >> 1;
    const long long npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSTAGE; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_tfull, 1);
        mbar_init(bar_tempty, 2 * 32 * PWK_EPI_WARPS);
        mbar_init(bar_drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), PW_TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const unsigned long long tmo = p.timeout_ns;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------ TMA producer (both CTAs)
        int stage = 0;
        uint32_t phase = 0;
        int issued_parity[NSTAGE];
        for (int s = 0; s < NSTAGE; ++s) issued_parity[s] = -1;
        const long long first_tile = p.stall_producer ? p.num_tiles : pair;
        bool align = p.wave_counter != nullptr;
        long long wave = 0;
        for (long long tile = first_tile; tile < p.num_tiles && !*abort_flag;
             tile += npairs, ++wave) {
            if (align && (wave + 1) * npairs <= p.num_tiles) {
                atomicAdd(p.wave_counter, 1u);
                const unsigned target = gridDim.x * (unsigned)(wave + 1);
                const uint64_t dl = global_timer_ns() + 2000000ull;  // 2 ms
                while (*reinterpret_cast<volatile unsigned*>(p.wave_counter) < target) {
                    if (global_timer_ns() > dl) {
                        align = false;  // give up aligning; never wait again
                        break;
                    }
                }
            }
            int kind, abase, qbase, mt, nt;
            pwk_tile_decode(p, tile, kind, abase, qbase, mt, nt);
            // planes per side and k-blocks per stage: lo u, v in [0, 3];
            // hi u, v in [1, 3]; a length-2 convolution, u, v in [0, 1] for
            // two consecutive k-blocks
            const int nsl = kind == 2 ? 2 : (kind ? 3 : 4);
            const int ksub = kind == 2 ? QK : 1;
            for (int kb = 0; kb < p.kblocks; kb += ksub) {
                const int nk = kb + ksub <= p.kblocks ? ksub : 1;
                const uint32_t stage_tx =
                    2u * (uint32_t)(nk * nsl) * (PWK_A_BYTES + PWK_B_BYTES);
                if (!mbar_wait_bounded(bar_empty + 8 * stage, phase ^ 1, abort_flag,
                                       global_timer_ns() + tmo))
                    goto producer_done;
                const uint32_t full_leader = mapa_shared(bar_full + 8 * stage, 0);
                if (leader) mbar_arrive_expect_tx(bar_full + 8 * stage, stage_tx);
                uint8_t* st = smem + stage * STAGE_BYTES;
                for (int h = 0; h < nk; ++h)
                    for (int i = 0; i < nsl; ++i) {
                        const int slot = h * nsl + i;
                        tma_load_3d_pair(smem_u32(st + slot * PWK_A_BYTES), &tmA, full_leader,
                                         (kb + h) * PW_BK, mt * 256 + (int)rank * 128, abase + i);
                        tma_load_3d_pair(smem_u32(st + NS * PWK_A_BYTES + slot * PWK_B_BYTES),
                                         &tmB, full_leader, (kb + h) * PW_BK,
                                         nt * PWK_BN + (int)rank * (PWK_BN / 2), abase + i);
                    }
                issued_parity[stage] = (int)phase;
                if (++stage == NSTAGE) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
    producer_done:
        for (int s = 0; s < NSTAGE; ++s)
            if (issued_parity[s] >= 0)
                if (!mbar_wait_deadline(bar_empty + 8 * s, (uint32_t)issued_parity[s],
                                        global_timer_ns() + tmo))
                    *abort_flag = 1;
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------ MMA issuer (leader only)
        const uint32_t idesc = idesc_i8(256, PWK_BN);
        int stage = 0;
        uint32_t phase = 0;
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles && !*abort_flag; tile += npairs) {
            int kind, abase, qbase, mt, nt;
            pwk_tile_decode(p, tile, kind, abase, qbase, mt, nt);
            const int hi = kind & 1;
            const int ksub = kind == 2 ? QK : 1;
            if (!mbar_wait_bounded(bar_tempty, acc_phase ^ 1, abort_flag, global_timer_ns() + tmo))
                break;
            tc_fence_after();
            for (int kb = 0; kb < p.kblocks; kb += ksub) {
                if (!mbar_wait_bounded(bar_full + 8 * stage, phase, abort_flag,
                                       global_timer_ns() + tmo))
                    goto mma_done;
                tc_fence_after();
                const uint32_t st = smem_u32(smem + stage * STAGE_BYTES);
                if (kind == 2) {
                    // slots 2h + u (A) / 2h + v (B) hold k-block kb + h; the
                    // term (u, v) belongs to accumulator u + v, started by
                    // its first term in loop order -- (0,0), (0,1), (1,1) --
                    // in k-block 0
                    const int nk = kb + QK <= p.kblocks ? QK : 1;
                    for (int h = 0; h < nk; ++h) {
                        const uint32_t acc0 = kb + h != 0 ? 1u : 0u;
#pragma unroll
                        for (int ia = 0; ia < 2; ++ia) {
#pragma unroll
                            for (int ib = 0; ib < 2; ++ib) {
                                const int accn = ia + ib;
                                const bool init = ia == 0 || accn == 2;
                                const uint32_t a0 = st + (2 * h + ia) * PWK_A_BYTES;
                                const uint32_t b0 =
                                    st + NS * PWK_A_BYTES + (2 * h + ib) * PWK_B_BYTES;
#pragma unroll
                                for (int kk = 0; kk < PW_BK / 32; ++kk)
                                    mma_i8_pair(tmem_base + (uint32_t)(accn * PWK_BN),
                                                sdesc_kmajor_sw128(a0 + kk * 32),
                                                sdesc_kmajor_sw128(b0 + kk * 32), idesc,
                                                (acc0 | (uint32_t)kk | (init ? 0u : 1u)) != 0
                                                    ? 1u
                                                    : 0u);
                            }
                        }
                    }
                    mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
                    if (++stage == NSTAGE) {
                        stage = 0;
                        phase ^= 1;
                    }
                    continue;
                }
                if constexpr (NS == 4) {
                    const uint32_t acc0 = kb != 0 ? 1u : 0u;  // the first k-block starts every sum
                    // slot i holds plane u = hi + i (A) / v = hi + i (B); the
                    // term (u, v) belongs to output s = u + v, accumulator
                    // s - 4 hi
#pragma unroll
                    for (int ia = 0; ia < NS; ++ia) {
#pragma unroll
                        for (int ib = 0; ib < NS; ++ib) {
                            const int s = ia + ib + 2 * hi;  // u + v
                            if (hi ? (ia == 3 || ib == 3 || s < 4) : s > 3) continue;
                            const int accn = hi ? s - 4 : s;
                            // the first term of each accumulator in loop order
                            // -- ia = 0 (lo), ia = accn (hi) -- starts it in
                            // k-block 0
                            const bool init = ia == (hi ? accn : 0);
                            const uint32_t a0 = st + ia * PWK_A_BYTES;
                            const uint32_t b0 = st + NS * PWK_A_BYTES + ib * PWK_B_BYTES;
#pragma unroll
                            for (int kk = 0; kk < PW_BK / 32; ++kk)
                                mma_i8_pair(tmem_base + (uint32_t)(accn * PWK_BN),
                                            sdesc_kmajor_sw128(a0 + kk * 32),
                                            sdesc_kmajor_sw128(b0 + kk * 32), idesc,
                                            (acc0 | (uint32_t)kk | (init ? 0u : 1u)) != 0 ? 1u
                                                                                          : 0u);
                        }
                    }
                }
                mma_commit_pair_mc(bar_empty + 8 * stage, 0x3);
                if (++stage == NSTAGE) {
                    stage = 0;
                    phase ^= 1;
                }
            }
            mma_commit_pair_mc(bar_tfull, 0x3);
            acc_phase ^= 1;
        }
    mma_done:
        mma_commit_pair(bar_drain);
        if (!mbar_wait_deadline(bar_drain, 0, global_timer_ns() + tmo)) *abort_flag = 1;
    } else if (warp >= 2) {
        // ------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;               // TMEM lanes this warp may access
        const int half = (warp - 2) / 4;            // columns [64 half, 64 half + 64)
        uint32_t acc_phase = 0;
        for (long long tile = pair; tile < p.num_tiles; tile += npairs) {
            int kind, abase, qbase, mt, nt;
            pwk_tile_decode(p, tile, kind, abase, qbase, mt, nt);
            if (!mbar_wait_bounded(bar_tfull, acc_phase, abort_flag, global_timer_ns() + tmo))
                break;
            tc_fence_after();
            const int row = mt * 256 + (int)rank * 128 + quarter * 32 + lane;
            const int col0 = nt * PWK_BN;
            const int colmax = p.cols - col0;
            const int nout = kind == 0 ? 4 : 3;
            for (int a = 0; a < nout; ++a) {
                const int q = qbase + a;
                int32_t* orow = p.out + (long long)q * p.out_plane + (long long)row * p.ldo + col0;
                {
                    const int c = half;
                    uint32_t v[64];  // this warp's 64 columns, one wait
                    tmem_ld_32x32b_x64_wait(tmem_base + ((uint32_t)(quarter * 32) << 16) +
                                                (uint32_t)(a * PWK_BN + c * 64),
                                            v);
                    if (row < p.rows) {
#pragma unroll
                        for (int e = 0; e < 64; e += 4) {
                            const int col = c * 64 + e;
                            if (col < colmax) {
                                int4 o;
                                o.x = (int)v[e];
                                o.y = (int)v[e + 1];
                                o.z = (int)v[e + 2];
                                o.w = (int)v[e + 3];
                                *reinterpret_cast<int4*>(orow + col) = o;
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive_cluster(mapa_shared(bar_tempty, 0));
            acc_phase ^= 1;
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();
    tc_fence_after();
    if (threadIdx.x == 0 && *abort_flag) atomicCAS(p.err, 0, MFFTB_ERR_TIMEOUT);
    if (warp == 1) tmem_dealloc_pair(tmem_base, PW_TMEM_COLS);
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) !=
                cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return nullptr;
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// 3-D int8 tensor [planes][rows][kdim] with row stride ld bytes and plane
// stride plane_bytes; box = box_rows x 128 bytes of one plane, 128B swizzle.
static int make_map(CUtensorMap* m, const void* base, int kdim, int rows, int planes, long long ld,
                    long long plane_bytes, int box_rows) {
    auto enc = get_encode_fn();
    if (!enc) return MFFTB_ERR_CUDA;
    cuuint64_t dims[3] = {(cuuint64_t)kdim, (cuuint64_t)rows, (cuuint64_t)planes};
    cuuint64_t strides[2] = {(cuuint64_t)ld, (cuuint64_t)plane_bytes};
    cuuint32_t box[3] = {(cuuint32_t)PW_BK, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MFFTB_OK : MFFTB_ERR_CUDA;
}

static int launch_kara(const PwLaunch& L, cudaStream_t stream) {
    // one digit class and chunk, K = 8 (S = 4), CTA pairs over 256-row tiles
    // (map_rows >= 256: rows past L.rows are read from the plane's padding and
    // their outputs are not stored)
    if (L.jobs.K != 8 || L.jobs.dA != 1 || L.jobs.dB != 1 || L.jobs.nchunk != 1 ||
        L.num_sms < 2 || L.cols < 128 || L.map_rows < 256 || L.map_rows < L.rows ||
        L.a_planes != L.jobs.NB * pw_kara_ops(L.jobs) ||
        L.f_planes != L.jobs.NB * pw_kara_ops(L.jobs))
        return MFFTB_ERR_ARG;
    if (L.chosen) *L.chosen = 4;
    PwParams p;
    p.jobs = L.jobs;
    p.rows = L.rows;
    p.cols = L.cols;
    p.kdim = L.kdim;
    p.kblocks = (L.kdim + PW_BK - 1) / PW_BK;
    p.block_n = PWK_BN;
    p.tiles_m = (L.rows + 255) / 256;
    p.tiles_n = (L.cols + PWK_BN - 1) / PWK_BN;
    p.num_tiles = (long long)p.tiles_m * p.tiles_n * pw_kara_groups(L.jobs);
    p.out = L.out;
    p.out_plane = L.out_plane;
    p.ldo = L.ldo;
    p.err = L.err;
    p.timeout_ns = L.timeout_ns;
    p.stall_producer = L.stall_producer;
    p.raster = L.raster;
    p.group_m = L.group_m > 0 ? L.group_m : PW_GROUP_M / 2;
    p.wave_counter = L.wave_counter;
    if (p.wave_counter &&
        cudaMemsetAsync(p.wave_counter, 0, sizeof(unsigned int), stream) != cudaSuccess)
        return MFFTB_ERR_CUDA;
    CUtensorMap tmA, tmB;
    int rc = make_map(&tmA, L.A, L.kdim, L.map_rows, L.a_planes, L.lda, L.a_plane_bytes, PW_BM);
    if (rc) return rc;
    rc = make_map(&tmB, L.F, L.kdim, L.cols, L.f_planes, L.ldf, L.f_plane_bytes, PWK_BN / 2);
    if (rc) return rc;
    // four 48 KB stages only on request (kara_stages = 4, level 3): at c5
    // they ran 10 % slower per clock than two 96 KB stages (half the MMAs
    // per barrier round trip)
    const bool four = L.jobs.kara == 3 && L.kara_stages == 4;
    static int attr_dev[2] = {-1, -1};
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev[four] != dev) {
        if (cudaFuncSetAttribute(four ? pointwise_kara_i8_kernel<4> : pointwise_kara_i8_kernel<2>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PWK_SMEM_BYTES) != cudaSuccess)
            return MFFTB_ERR_CUDA;
        attr_dev[four] = dev;
    }
    long long pairs = L.num_sms / 2;
    if (pairs > p.num_tiles) pairs = p.num_tiles;
    if (pairs <= 0) return MFFTB_OK;
    if (four)
        pointwise_kara_i8_kernel<4>
            <<<(unsigned)(2 * pairs), PWK_THREADS, PWK_SMEM_BYTES, stream>>>(tmA, tmB, p);
    else
        pointwise_kara_i8_kernel<2>
            <<<(unsigned)(2 * pairs), PWK_THREADS, PWK_SMEM_BYTES, stream>>>(tmA, tmB, p);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

int pointwise_launch(const PwLaunch& L, cudaStream_t stream) {
    if (L.kdim <= 0 || L.rows <= 0 || L.cols <= 0) return MFFTB_ERR_ARG;
    if ((L.lda % 16) || (L.ldf % 16) || (L.ldo % 4) || (L.a_plane_bytes % 16) ||
        (L.f_plane_bytes % 16) || (L.cols % 16))
        return MFFTB_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(L.A) % 16 || reinterpret_cast<uintptr_t>(L.F) % 16 ||
        reinterpret_cast<uintptr_t>(L.out) % 16)
        return MFFTB_ERR_ARG;
    if (L.jobs.kara) return launch_kara(L, stream);
    // t-grouped CTA pairs for one-chunk plans, CTA pairs when both dimensions
    // fill at least one 256 x 256 pair tile, single CTAs otherwise.  The
    // schoolbook job table runs on the t-grouped kernel only, at any size
    // (tiles past the operand edges load zeros).
    const bool grouped_ok =
        L.jobs.K % PW3_TG == 0 && L.num_sms >= 2 &&
        (L.jobs.school ? (L.jobs.dA == 1 && L.jobs.dB == 1 && L.jobs.nW == 1 && L.jobs.U >= 1)
                       : (L.jobs.nchunk == 1 && L.rows >= 256 && L.cols >= 128));
    if (L.jobs.school && (!grouped_ok || (L.variant != 0 && L.variant != 3))) return MFFTB_ERR_ARG;
    const bool grouped = L.variant == 3 ? grouped_ok : (L.variant == 0 && grouped_ok);
    if (L.variant == 3 && !grouped_ok) return MFFTB_ERR_ARG;
    const bool pair = !grouped && (L.variant == 2 || (L.variant == 0 && L.block_n == 256 &&
                                                      L.rows >= 256 && L.cols >= 256 &&
                                                      L.num_sms >= 2));
    if (L.chosen) *L.chosen = grouped ? 3 : (pair ? 2 : 1);
    PwParams p;
    p.jobs = L.jobs;
    p.rows = L.rows;
    p.cols = L.cols;
    p.kdim = L.kdim;
    p.kblocks = (L.kdim + PW_BK - 1) / PW_BK;
    p.block_n = grouped ? PW3_BN : (pair ? PW2_BN : L.block_n);
    if (p.block_n != 64 && p.block_n != 128 && p.block_n != 256) return MFFTB_ERR_ARG;
    p.tiles_m = (pair || grouped) ? (L.rows + 255) / 256 : (L.rows + PW_BM - 1) / PW_BM;
    p.tiles_n = (L.cols + p.block_n - 1) / p.block_n;
    p.num_tiles = (long long)p.tiles_m * p.tiles_n *
                  (grouped ? (long long)(L.jobs.njobs / PW3_TG) : (long long)L.jobs.njobs);
    p.out = L.out;
    p.out_plane = L.out_plane;
    p.ldo = L.ldo;
    p.err = L.err;
    p.timeout_ns = L.timeout_ns;
    p.stall_producer = L.stall_producer;
    p.raster = L.raster;
    p.group_m = L.group_m > 0 ? L.group_m : ((pair || grouped) ? PW_GROUP_M / 2 : PW_GROUP_M);
    p.wave_counter = grouped ? L.wave_counter : nullptr;
    if (p.wave_counter &&
        cudaMemsetAsync(p.wave_counter, 0, sizeof(unsigned int), stream) != cudaSuccess)
        return MFFTB_ERR_CUDA;

    CUtensorMap tmA, tmF;
    int rc = make_map(&tmA, L.A, L.kdim, L.rows, L.a_planes, L.lda, L.a_plane_bytes, PW_BM);
    if (rc) return rc;
    rc = make_map(&tmF, L.F, L.kdim, L.cols, L.f_planes, L.ldf, L.f_plane_bytes,
                  grouped ? PW3_BN / 2 : (pair ? PW2_BN / 2 : p.block_n));
    if (rc) return rc;

    if (grouped) {
        static int attr_dev3 = -1;
        int dev = 0;
        cudaGetDevice(&dev);
        if (attr_dev3 != dev) {
            if (cudaFuncSetAttribute(pointwise3_i8_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     PW3_SMEM_BYTES) != cudaSuccess)
                return MFFTB_ERR_CUDA;
            attr_dev3 = dev;
        }
        long long pairs = L.num_sms / 2;
        if (pairs > p.num_tiles) pairs = p.num_tiles;
        if (pairs <= 0) return MFFTB_OK;
        pointwise3_i8_kernel<<<(unsigned)(2 * pairs), PW_THREADS, PW3_SMEM_BYTES, stream>>>(tmA,
                                                                                         tmF, p);
        return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
    }

    if (pair) {
        static int attr_dev = -1;
        int dev = 0;
        cudaGetDevice(&dev);
        if (attr_dev != dev) {
            if (cudaFuncSetAttribute(pointwise2_i8_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     PW2_SMEM_BYTES) != cudaSuccess)
                return MFFTB_ERR_CUDA;
            attr_dev = dev;
        }
        long long pairs = L.num_sms / 2;
        if (pairs > p.num_tiles) pairs = p.num_tiles;
        if (pairs <= 0) return MFFTB_OK;
        pointwise2_i8_kernel<<<(unsigned)(2 * pairs), PW_THREADS, PW2_SMEM_BYTES, stream>>>(tmA, tmF,
                                                                                         p);
        return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
    }
    static int attr_dev1 = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (attr_dev1 != dev) {
        if (cudaFuncSetAttribute(pointwise_i8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PW_SMEM_BYTES) != cudaSuccess)
            return MFFTB_ERR_CUDA;
        attr_dev1 = dev;
    }
    long long grid = L.num_sms;
    if (grid > p.num_tiles) grid = p.num_tiles;
    if (grid <= 0) return MFFTB_OK;
    pointwise_i8_kernel<<<(unsigned)grid, PW_THREADS, PW_SMEM_BYTES, stream>>>(tmA, tmF, p);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

}  // namespace mfftb

// ---------------------------------------------------------------- checker
// Plain CUDA-core evaluation of the same job table, one thread per output
// element with an int64 accumulator.  Used only by the unit tests of the
// tcgen05 kernel (never on the product path).
namespace mfftb {

__global__ void pointwise_simt_check_kernel(const int8_t* A, long long lda, long long a_plane,
                                            const int8_t* F, long long ldf, long long f_plane,
                                            int rows, int cols, int kdim, PwJobs J, int32_t* out,
                                            long long out_plane, int ldo, int* mismatch,
                                            long long* first_bad) {
    long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    long long per_job = (long long)rows * cols;
    if (idx >= per_job * J.njobs) return;
    int q = (int)(idx / per_job);
    int r = (int)((idx % per_job) / cols);
    int c = (int)(idx % cols);
    long long acc = 0;
    if (J.kara) {
        // kara = 1: q = j*21 + p*7 + s, the sum over u + v = s (u, v < 4) of
        // A(base + u) * B(base + v), base = j*12 + 4p.  kara = 2: q = j*25 +
        // 3g + s (g < 6) sums u + v = s (u, v < 2) from the first plane of
        // length-2 convolution g; q = j*25 + 18 + s is P2 (base j*16 + 8).
        // kara = 3: q = j*27 + 3g + s for all nine g.
        const int nq = pw_kara_jobs(J), ops = pw_kara_ops(J);
        const int j = q / nq, off = q % nq;
        int base, s, w;
        if ((J.kara == 2 && off < 18) || J.kara == 3) {
            base = j * ops + pw_kara2_qplane(off / 3);
            s = off % 3;
            w = 2;
            if (off >= 9 && pw_kara_half(J, j)) return;  // P1, P2: not at a half point
        } else {
            const int pr = J.kara == 2 ? 2 : off / 7;
            base = j * ops + 4 * pr;
            s = J.kara == 2 ? off - 18 : off % 7;
            w = 4;
            if (pr > 0 && pw_kara_half(J, j)) return;  // not computed at a half point
        }
        for (int u = s > w - 1 ? s - (w - 1) : 0; u <= (s < w - 1 ? s : w - 1); ++u) {
            const int8_t* a = A + (base + u) * a_plane + r * lda;
            const int8_t* f = F + (base + (s - u)) * f_plane + c * ldf;
            for (int k = 0; k < kdim; ++k) acc += (long long)a[k] * (long long)f[k];
        }
        int32_t got = out[q * out_plane + (long long)r * ldo + c];
        if ((long long)got != acc) {
            if (atomicAdd(mismatch, 1) == 0) *first_bad = idx;
        }
        return;
    }
    if (J.school) {
        const int t = q / J.nchunk, ch = q % J.nchunk;
        int lo, hi;
        pw_school_range(J, t, ch, lo, hi);
        if (lo > hi) return;  // a job without terms is never written
        for (int u = lo; u <= hi; ++u) {
            const int8_t* a = A + u * a_plane + r * lda;
            const int8_t* f = F + (t - u) * f_plane + c * ldf;
            for (int k = 0; k < kdim; ++k) acc += (long long)a[k] * (long long)f[k];
        }
        int32_t got = out[q * out_plane + (long long)r * ldo + c];
        if ((long long)got != acc) {
            if (atomicAdd(mismatch, 1) == 0) *first_bad = idx;
        }
        return;
    }
    int j, t, w, ch, s0, s1;
    pw_job_decode(J, q, j, t, w, ch);
    pw_chunk_range(J, w, ch, s0, s1);
    for (int s = s0; s < s1; ++s) {
        int pa, pf;
        pw_segment_planes(J, j, t, w, s, pa, pf);
        const int8_t* a = A + pa * a_plane + r * lda;
        const int8_t* f = F + pf * f_plane + c * ldf;
        for (int k = 0; k < kdim; ++k) acc += (long long)a[k] * (long long)f[k];
    }
    int32_t got = out[q * out_plane + (long long)r * ldo + c];
    if ((long long)got != acc) {
        if (atomicAdd(mismatch, 1) == 0) *first_bad = idx;
    }
}

int pointwise_check_launch(const PwLaunch& L, int* d_mismatch, long long* d_first_bad,
                           cudaStream_t stream) {
    long long total = (long long)L.rows * L.cols * L.jobs.njobs;
    int threads = 256;
    long long blocks = (total + threads - 1) / threads;
    pointwise_simt_check_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        L.A, L.lda, L.a_plane_bytes, L.F, L.ldf, L.f_plane_bytes, L.rows, L.cols, L.kdim, L.jobs,
        L.out, L.out_plane, L.ldo, d_mismatch, d_first_bad);
    return cudaGetLastError() == cudaSuccess ? MFFTB_OK : MFFTB_ERR_CUDA;
}

}  // namespace mfftb
