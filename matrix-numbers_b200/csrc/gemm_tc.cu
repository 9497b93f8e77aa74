// Stage 3b: the N per-modulus INT8 products, on the 5th-generation tensor cores, with the modular reduction fused
// into the epilogue (the reference runs one cuBLASLt INT8 GEMM per modulus and a separate reduce_k pass,
// code/ozaki_engine.py:1333-1341, :952-967, so its INT32 products make a round trip through HBM).
//
// Design (sm_100a):
//   - persistent grid, one CTA per SM, looping over work units (modulus t, 128 x 256 output tile); tiles of one
//     modulus are visited in groups of 16 tile-rows so that the A row-blocks and B column-blocks of a wave stay in L2;
//   - warp 0 (one lane): TMA producer, 4-stage ring of {A 128x128, B 256x128} int8 tiles, 128-byte swizzle;
//   - warp 1 (one lane): tcgen05.mma.cta_group::1.kind::i8 issuer, M=128 N=256 K=32, accumulating in TMEM;
//     warp 1 also allocates / frees the 512 TMEM columns (two 256-column accumulators, double-buffered so the
//     epilogue of one tile overlaps the main loop of the next);
//   - warps 2..9: epilogue, tcgen05.ld 32 lanes x 32 columns, INT32 -> residue mod m_t in [0, m_t) -> uint8 X.
//   - the contraction is cut into segments of 65536 (OZK_KSEG): each segment is accumulated in a fresh TMEM buffer
//     (|sum| <= 65536 * 128 * 128 = 2^30, exact), and segment residues are added modulo m_t, so any k is exact.
//   - every mbarrier wait is bounded (wall clock); on a timeout the CTA records a flag in *err, stops, waits
//     (bounded) for its own TMA loads and MMAs in flight, frees TMEM and exits.  No cluster multicast is used.
#include <cuda.h>

#include "ozk_common.cuh"
#include "tc_ptx.cuh"

using namespace ozk_ptx;

namespace {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr uint32_t A_BYTES = BM * BK;
constexpr uint32_t B_BYTES = BN * BK;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int SEG_KB = OZK_KSEG / BK;
constexpr int GROUP_M = 16;
constexpr uint32_t IDESC = umma_idesc_i8(BM, BN);
constexpr int NUM_BARS = 2 * STAGES + 5;   // full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;   // 4 s of wall time per wait

static_assert(NUM_BARS * 8 + 16 <= 256, "barrier area");

enum { MODE_RESIDUE = 0, MODE_I32 = 1 };

// Reduction of a signed INT32 accumulator v (|v| <= 2^30) modulo P, exact for every P <= 256:
//   u = v + OFF (OFF = P ceil(2^30 / P), a multiple of P; 0 <= u < 2^32), s = (u >> 16) R + (u & 0xffff) with
//   R = 2^16 mod P (s < 2^24 and s = u mod P), then s - P umulhi(s, MG) with MG = ceil(2^32 / P), exact for s < 2^24.
struct ModParams {
    uint32_t P[OZK_NMAX], R16[OZK_NMAX], MG[OZK_NMAX], OFF[OZK_NMAX];
};

__device__ __forceinline__ void decode_unit(int u, int tiles, int tiles_m, int tiles_n, int& t, int& tm, int& tn) {
    t = u / tiles;
    const int tile = u - t * tiles;
    const int per_group = GROUP_M * tiles_n;
    const int g = tile / per_group;
    const int first_m = g * GROUP_M;
    const int gm = min(tiles_m - first_m, GROUP_M);
    const int in = tile - g * per_group;
    tm = first_m + in % gm;
    tn = in / gm;
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int32_t* err, int code) {
    *abort_flag = 1;
    atomicOr(err, code);
}

// One thread's 32 consecutive accumulator columns of a row: stored as INT32 (MODE_I32) or reduced modulo m_t to a
// residue byte, added modulo m_t to the residues of earlier k segments (seg > 0)
template <int MODE>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&v)[32], int row, int col, int t, int seg, int m, int n,
                                               const ModParams& mp, void* __restrict__ out) {
    if (MODE == MODE_I32) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<int32_t*>(out) + (size_t)row * n + col);
#pragma unroll
        for (int q = 0; q < 8; q++) dst[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
        const uint32_t P = mp.P[t], R = mp.R16[t], MG = mp.MG[t], OFF = mp.OFF[t];
        uint32_t rs[32];
#pragma unroll
        for (int e = 0; e < 32; e++) {
            const uint32_t uu = v[e] + OFF;
            const uint32_t s = (uu >> 16) * R + (uu & 0xffffu);
            rs[e] = s - __umulhi(s, MG) * P;
        }
        uint8_t* xrow = static_cast<uint8_t*>(out) + ((size_t)t * m + row) * (size_t)n + col;
        uint4* dst = reinterpret_cast<uint4*>(xrow);
        if (seg > 0) {
            // add this segment's residues to the ones stored by this thread for earlier segments
            const uint4 p0 = dst[0], p1 = dst[1];
            const uint32_t pw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int e = 0; e < 32; e++) {
                uint32_t a = rs[e] + ((pw[e >> 2] >> (8 * (e & 3))) & 0xffu);
                rs[e] = a >= P ? a - P : a;
            }
        }
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; q++)
            w[q] = rs[4 * q] | (rs[4 * q + 1] << 8) | (rs[4 * q + 2] << 16) | (rs[4 * q + 3] << 24);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, void* __restrict__ out,
                   int m, int n, int k, int N, const __grid_constant__ ModParams mp, int32_t* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (uint32_t)(STAGES + s); };
    auto accf_bar = [&](int b) { return bar0 + 8u * (uint32_t)(2 * STAGES + b); };
    auto acce_bar = [&](int b) { return bar0 + 8u * (uint32_t)(2 * STAGES + 2 + b); };
    const uint32_t drain_bar = bar0 + 8u * (uint32_t)(2 * STAGES + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) { mbar_init(full_bar(s), 1); mbar_init(empty_bar(s), 1); }
        for (int b = 0; b < 2; b++) { mbar_init(accf_bar(b), 1); mbar_init(acce_bar(b), EPI_WARPS); }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int tiles_m = (m + BM - 1) / BM, tiles_n = (n + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int units = N * tiles;
    const int kblocks = (k + BK - 1) / BK;
    const int nseg = (kblocks + SEG_KB - 1) / SEG_KB;

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ TMA producer
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
                int t, tm, tn;
                decode_unit(u, tiles, tiles_m, tiles_n, t, tm, tn);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
                    tma_load_3d(smem_addr(sA + stage * A_BYTES), &tmA, kb * BK, tm * BM, t, full_bar(stage));
                    tma_load_3d(smem_addr(sB + stage * B_BYTES), &tmB, kb * BK, tn * BN, t, full_bar(stage));
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // let the loads already issued land before the CTA exits (bounded)
                const long long first = issued > STAGES ? issued - STAGES : 0;
                for (long long j = first; j < issued; j++) {
                    const int s = (int)(j % STAGES);
                    const uint32_t par = (uint32_t)((j / STAGES) & 1);
                    int dummy = 0;
                    mbar_wait_bounded(full_bar(s), par, &dummy, WAIT_LIMIT_NS);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ------------------------------------------------------------ MMA issuer
            int stage = 0;
            uint32_t phase = 0, acc_it = 0;
            bool ok = true, issued_any = false;
            for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
                for (int seg = 0; ok && seg < nseg; seg++) {
                    const int b = (int)(acc_it & 1u);
                    const uint32_t aph = (acc_it >> 1) & 1u;
                    if (!mbar_wait_bounded(acce_bar(b), aph ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
                    const int kb0 = seg * SEG_KB, kb1 = min(kblocks, kb0 + SEG_KB);
                    for (int kb = kb0; kb < kb1; kb++) {
                        if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, WAIT_LIMIT_NS)) {
                            if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t adesc = umma_desc_sw128(smem_addr(sA + stage * A_BYTES));
                        const uint64_t bdesc = umma_desc_sw128(smem_addr(sB + stage * B_BYTES));
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++) {
                            // advance 32 bytes along K inside the 128-byte swizzle atom: +2 in the >>4 address field
                            umma_i8(d_tmem, adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), IDESC,
                                    (kb > kb0 || kk > 0) ? 1u : 0u);
                        }
                        issued_any = true;
                        umma_commit(empty_bar(stage));
                        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    umma_commit(accf_bar(b));
                    acc_it++;
                }
            }
            if (!ok && issued_any) {
                // all MMAs issued by this thread must finish before TMEM is released
                umma_commit(drain_bar);
                int dummy = 0;
                mbar_wait_bounded(drain_bar, 0u, &dummy, WAIT_LIMIT_NS);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue warps
        const int ew = warp - 2;
        const int quarter = warp & 3;          // TMEM lanes this warp may access: [32 quarter, 32 quarter + 32)
        const int half = ew >> 2;              // column half of the 256-column accumulator
        uint32_t acc_it = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
            int t, tm, tn;
            decode_unit(u, tiles, tiles_m, tiles_n, t, tm, tn);
            const int row = tm * BM + quarter * 32 + lane;
            for (int seg = 0; seg < nseg; seg++) {
                const int b = (int)(acc_it & 1u);
                const uint32_t aph = (acc_it >> 1) & 1u;
                if (!mbar_wait_bounded(accf_bar(b), aph, abort_flag, WAIT_LIMIT_NS)) {
                    if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_EPILOGUE);
                    ok = false;
                    break;
                }
                __syncwarp();
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < 4; cc++) {
                    const int col_local = half * 128 + cc * 32;
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN + col_local), v);
                    tmem_wait_ld();
                    const int col = tn * BN + col_local;
                    if (row < m && col < n) epilogue_chunk<MODE>(v, row, col, t, seg, m, n, mp, out);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce_bar(b));
                acc_it++;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- the two-SM tile (tcgen05 cta_group::2) -------------------------------------------------------------------
// A cluster of two CTAs on a pair of SMs computes a 256 x 256 tile of one modulus: CTA r holds rows 128 r .. 128 r +
// 127 of the A tile and columns 128 r .. 128 r + 127 of the B tile (K-major, 128-byte swizzle, at the same shared
// memory offsets in both CTAs), so each SM streams 32 KB per 128-deep k block instead of 48 KB, and six stages fit.
//   - both CTAs' warp 0 load their halves with TMA; every load completes on CTA 0's full barrier, which CTA 0's
//     producer arms with the bytes of both halves (no multicast: each CTA loads only its own data);
//   - CTA 0's warp 1 issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32): it reads A and B from both CTAs'
//     shared memory and writes each CTA's TMEM with its own 128 rows; its commits arrive on the stage's empty barrier
//     and on the accumulator-full barrier of both CTAs (one commit per barrier);
//   - the epilogue warps of both CTAs drain their own TMEM as in the one-SM kernel and arrive on CTA 0's
//     accumulator-empty barrier (the follower's arrivals are remote, at cluster scope);
//   - the CTAs meet at a cluster barrier after initialisation and before TMEM is freed, so no CTA leaves while its
//     peer can still write its TMEM or its barriers; every other wait is bounded, as in the one-SM kernel.
constexpr int HALF = 128;                    // rows of A and of B held by each CTA of the pair
constexpr int BM2 = 2 * HALF, BN2 = 2 * HALF;
constexpr int STAGES2 = 6;
constexpr uint32_t A2_BYTES = HALF * BK, B2_BYTES = HALF * BK;
constexpr uint32_t STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int GROUP_M2 = 8;                  // 8 tile-rows of 256 = the 16 tile-rows of 128 of the one-SM kernel
constexpr uint32_t IDESC2 = umma_idesc_i8(BM2, BN2);
constexpr int NUM_BARS2 = 2 * STAGES2 + 5;   // full[S], empty[S], acc_full[2], acc_empty[2], drain
constexpr size_t SMEM2_BYTES = (size_t)STAGES2 * STAGE2_BYTES + 1024 + 256;
static_assert(NUM_BARS2 * 8 + 16 <= 256, "barrier area");
static_assert(BN2 == BN, "the epilogue covers the 256 accumulator columns of the one-SM kernel");

__device__ __forceinline__ void decode_unit2(int u, int tiles, int tiles_m, int tiles_n, int& t, int& tm, int& tn) {
    t = u / tiles;
    const int tile = u - t * tiles;
    const int per_group = GROUP_M2 * tiles_n;
    const int g = tile / per_group;
    const int first_m = g * GROUP_M2;
    const int gm = min(tiles_m - first_m, GROUP_M2);
    const int in = tile - g * per_group;
    tm = first_m + in % gm;
    tn = in / gm;
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    void* __restrict__ out, int m, int n, int k, int N, const __grid_constant__ ModParams mp,
                    int32_t* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES2 * A2_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();           // 0: issues the MMAs; 1: its peer
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (uint32_t)(STAGES2 + s); };
    auto accf_bar = [&](int b) { return bar0 + 8u * (uint32_t)(2 * STAGES2 + b); };
    auto acce_bar = [&](int b) { return bar0 + 8u * (uint32_t)(2 * STAGES2 + 2 + b); };
    const uint32_t drain_bar = bar0 + 8u * (uint32_t)(2 * STAGES2 + 4);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES2; s++) { mbar_init(full_bar(s), 1); mbar_init(empty_bar(s), 1); }
        for (int b = 0; b < 2; b++) { mbar_init(accf_bar(b), 1); mbar_init(acce_bar(b), 2 * EPI_WARPS); }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_addr(tmem_slot), TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();                                    // the peer's barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int tiles_m = (m + BM2 - 1) / BM2, tiles_n = (n + BN2 - 1) / BN2;
    const int tiles = tiles_m * tiles_n;
    const int units = N * tiles;
    const int kblocks = (k + BK - 1) / BK;
    const int nseg = (kblocks + SEG_KB - 1) / SEG_KB;
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);

    if (warp == 0) {
        if (lane == 0) {
            // ------------------------------------------------------------ TMA producer (both CTAs)
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int u = pair; ok && u < units; u += npairs) {
                int t, tm, tn;
                decode_unit2(u, tiles, tiles_m, tiles_n, t, tm, tn);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    const uint32_t full0 = map_to_rank(full_bar(stage), 0u);
                    if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2u * STAGE2_BYTES);
                    tma_load_3d_pair(smem_addr(sA + stage * A2_BYTES), &tmA, kb * BK, tm * BM2 + (int)rank * HALF, t,
                                     full0);
                    tma_load_3d_pair(smem_addr(sB + stage * B2_BYTES), &tmB, kb * BK, tn * BN2 + (int)rank * HALF, t,
                                     full0);
                    issued++;
                    if (++stage == STAGES2) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok && rank == 0) {
                // let the loads already armed land before the pair exits (bounded)
                const long long first = issued > STAGES2 ? issued - STAGES2 : 0;
                for (long long j = first; j < issued; j++) {
                    const int s = (int)(j % STAGES2);
                    const uint32_t par = (uint32_t)((j / STAGES2) & 1);
                    int dummy = 0;
                    mbar_wait_bounded(full_bar(s), par, &dummy, WAIT_LIMIT_NS);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ------------------------------------------------------------ MMA issuer (CTA 0 of the pair)
            int stage = 0;
            uint32_t phase = 0, acc_it = 0;
            bool ok = true, issued_any = false;
            for (int u = pair; ok && u < units; u += npairs) {
                for (int seg = 0; ok && seg < nseg; seg++) {
                    const int b = (int)(acc_it & 1u);
                    const uint32_t aph = (acc_it >> 1) & 1u;
                    if (!mbar_wait_bounded(acce_bar(b), aph ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN2);
                    const int kb0 = seg * SEG_KB, kb1 = min(kblocks, kb0 + SEG_KB);
                    for (int kb = kb0; kb < kb1; kb++) {
                        if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, WAIT_LIMIT_NS)) {
                            if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t adesc = umma_desc_sw128(smem_addr(sA + stage * A2_BYTES));
                        const uint64_t bdesc = umma_desc_sw128(smem_addr(sB + stage * B2_BYTES));
#pragma unroll
                        for (int kk = 0; kk < BK / 32; kk++)
                            umma_i8_pair(d_tmem, adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), IDESC2,
                                         (kb > kb0 || kk > 0) ? 1u : 0u);
                        issued_any = true;
                        umma_commit_pair(empty_bar(stage));
                        umma_commit_pair(map_to_rank(empty_bar(stage), 1u));
                        if (++stage == STAGES2) { stage = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    umma_commit_pair(accf_bar(b));
                    umma_commit_pair(map_to_rank(accf_bar(b), 1u));
                    acc_it++;
                }
            }
            if (!ok && issued_any) {
                // every MMA issued by this thread finishes before the pair's TMEM is released
                umma_commit_pair(drain_bar);
                int dummy = 0;
                mbar_wait_bounded(drain_bar, 0u, &dummy, WAIT_LIMIT_NS);
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue warps (both CTAs)
        const int ew = warp - 2;
        const int quarter = warp & 3;          // TMEM lanes this warp may access: [32 quarter, 32 quarter + 32)
        const int half = ew >> 2;              // column half of the 256-column accumulator
        uint32_t acc_it = 0;
        bool ok = true;
        for (int u = pair; ok && u < units; u += npairs) {
            int t, tm, tn;
            decode_unit2(u, tiles, tiles_m, tiles_n, t, tm, tn);
            const int row = tm * BM2 + (int)rank * HALF + quarter * 32 + lane;
            for (int seg = 0; seg < nseg; seg++) {
                const int b = (int)(acc_it & 1u);
                const uint32_t aph = (acc_it >> 1) & 1u;
                bool w = mbar_wait_bounded(accf_bar(b), aph, abort_flag, WAIT_LIMIT_NS);
                if (!w && !*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_EPILOGUE);
                if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < 4; cc++) {
                    const int col_local = half * 128 + cc * 32;
                    uint32_t v[32];
                    tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN2 + col_local), v);
                    tmem_wait_ld();
                    const int col = tn * BN2 + col_local;
                    if (row < m && col < n) epilogue_chunk<MODE>(v, row, col, t, seg, m, n, mp, out);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(map_to_rank(acce_bar(b), 0u));
                acc_it++;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();                                    // neither CTA leaves while its peer may still reach it
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
    }
}

// ---- bounded-wait self-test ----------------------------------------------------------------------------------
// gemm_tc_kernel's failure path in miniature, on one CTA: warp 0 (the producer's role) and warp 2 (an epilogue
// role) each wait on an mbarrier that nothing arrives on, while warp 1 holds 32 TMEM columns as the GEMM's warp 1
// holds the accumulators.  The role named by `role` (0 = producer, 1 = epilogue) waits with `limit_ns`; the other
// waits with WAIT_LIMIT_NS and the abort flag, so it leaves through the flag that the timed-out role raises, not
// through its own limit.  Each role records how long it waited; TMEM is freed after both have returned, as at the
// end of gemm_tc_kernel.
__global__ void __launch_bounds__(96, 1)
    wait_selftest_kernel(int role, uint64_t limit_ns, int32_t* __restrict__ err, long long* __restrict__ waited_ns) {
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        mbar_init(smem_addr(&bars[0]), 1);
        mbar_init(smem_addr(&bars[1]), 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_addr(&tmem_slot), 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;
    if ((warp == 0 || warp == 2) && lane == 0) {
        const int me = warp == 0 ? 0 : 1;
        const uint64_t t0 = global_timer_ns();
        // phase 0 of a fresh barrier completes only after one arrival, and none comes
        const bool ok = mbar_wait_bounded(smem_addr(&bars[me]), 0u, &abort_flag, me == role ? limit_ns : WAIT_LIMIT_NS);
        waited_ns[me] = (long long)(global_timer_ns() - t0);
        if (!ok && !abort_flag)
            raise_abort(&abort_flag, err, me == 0 ? OZK_DEVERR_TIMEOUT_PRODUCER : OZK_DEVERR_TIMEOUT_EPILOGUE);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, 32);
    }
}

// ---- host side ------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// int8 planes [planes][rows][k] (K contiguous), box {BK, box_rows, 1}, 128-byte swizzle, zero fill out of bounds
int make_plane_map(CUtensorMap* map, const void* base, int k, int rows, int planes, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return OZK_ERR_DRIVER;
    const cuuint64_t dims[3] = {(cuuint64_t)k, (cuuint64_t)rows, (cuuint64_t)planes};
    const cuuint64_t strides[2] = {(cuuint64_t)k, (cuuint64_t)k * (cuuint64_t)rows};
    const cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)box_rows, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? OZK_OK : OZK_ERR_DRIVER;
}

ModParams make_mod_params() {
    ModParams mp{};
    for (int t = 0; t < OZK_NMAX; t++) {
        const uint32_t P = (uint32_t)ozk_mod(t);
        mp.P[t] = P;
        mp.R16[t] = (uint32_t)(65536u % P);
        mp.MG[t] = (uint32_t)((0x100000000ULL + P - 1) / P);
        mp.OFF[t] = (uint32_t)(P * (((1ULL << 30) + P - 1) / P));
    }
    return mp;
}

struct DeviceInfo {
    int sms = 0;
    bool attr_res = false, attr_i32 = false;
    bool attr2_res = false, attr2_i32 = false;
    int pairs = 0;                           // CTA pairs of the two-SM kernel that fit on the device at once
};
DeviceInfo g_dev[64];

int device_info(DeviceInfo** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OZK_ERR_DEVICE;
    DeviceInfo& d = g_dev[dev];
    if (d.sms == 0) {
        int major = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return OZK_ERR_DEVICE;
        if (major != 10) return OZK_ERR_DEVICE;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return OZK_ERR_DEVICE;
        d.sms = sms;
    }
    *out = &d;
    return OZK_OK;
}

template <int MODE>
int launch_gemm(const int8_t* Ares, const int8_t* Bres, int m, int n, int k, int N, void* out, int32_t* err,
                cudaStream_t st) {
    DeviceInfo* d = nullptr;
    int rc = device_info(&d);
    if (rc != OZK_OK) return rc;
    bool& attr = MODE == MODE_I32 ? d->attr_i32 : d->attr_res;
    if (!attr) {
        if (cudaFuncSetAttribute(gemm_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) !=
            cudaSuccess)
            return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
        attr = true;
    }
    CUtensorMap ta, tb;
    if ((rc = make_plane_map(&ta, Ares, k, m, N, BM)) != OZK_OK) return rc;
    if ((rc = make_plane_map(&tb, Bres, k, n, N, BN)) != OZK_OK) return rc;
    const long long units = (long long)N * ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
    if (units > 0x7fffffffLL) return OZK_ERR_ARG;
    const int grid = (int)(units < d->sms ? units : d->sms);
    static const ModParams mp = make_mod_params();
    gemm_tc_kernel<MODE><<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, out, m, n, k, N, mp, err);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

// The two-SM kernel: one cluster of two CTAs per pair of SMs, persistent over 256 x 256 tiles
template <int MODE>
int launch_gemm2(const int8_t* Ares, const int8_t* Bres, int m, int n, int k, int N, void* out, int32_t* err,
                 cudaStream_t st) {
    DeviceInfo* d = nullptr;
    int rc = device_info(&d);
    if (rc != OZK_OK) return rc;
    bool& attr = MODE == MODE_I32 ? d->attr2_i32 : d->attr2_res;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute cluster[1];
    cluster[0].id = cudaLaunchAttributeClusterDimension;
    cluster[0].val.clusterDim.x = 2;
    cluster[0].val.clusterDim.y = 1;
    cluster[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = SMEM2_BYTES;
    cfg.stream = st;
    cfg.attrs = cluster;
    cfg.numAttrs = 1;
    if (!attr) {
        if (cudaFuncSetAttribute(gemm_tc2_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)SMEM2_BYTES) != cudaSuccess)
            return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
        if (d->pairs == 0) {
            cfg.gridDim = dim3(2 * (d->sms / 2), 1, 1);
            int pairs = 0;
            if (cudaOccupancyMaxActiveClusters(&pairs, gemm_tc2_kernel<MODE>, &cfg) != cudaSuccess || pairs < 1)
                return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
            d->pairs = pairs;
        }
        attr = true;
    }
    CUtensorMap ta, tb;
    if ((rc = make_plane_map(&ta, Ares, k, m, N, HALF)) != OZK_OK) return rc;
    if ((rc = make_plane_map(&tb, Bres, k, n, N, HALF)) != OZK_OK) return rc;
    const long long units = (long long)N * ((m + BM2 - 1) / BM2) * ((n + BN2 - 1) / BN2);
    if (units > 0x7fffffffLL) return OZK_ERR_ARG;
    const int pairs = (int)(units < d->pairs ? units : d->pairs);
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    static const ModParams mp = make_mod_params();
    if (cudaLaunchKernelEx(&cfg, gemm_tc2_kernel<MODE>, ta, tb, out, m, n, k, N, mp, err) != cudaSuccess)
        return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

// Which tile: the two-SM kernel reads half the operand bytes per SM and is faster where a plane's operands stay in
// L2 (c2 +2 %, c5 (2048 x 2048, k = 262144) +14 % on one B200); on larger planes that stream from DRAM the one-SM
// kernel was faster under the 1 kW power cap (c3 -12 %, c4 -30 % for the two-SM kernel, same GPU, alternating runs)
bool use_pair_tiles(int m, int n) { return m > HALF && (long long)m * n <= 4096LL * 4096LL; }

bool shapes_ok(const void* a, const void* b, const void* out, const void* err, int m, int n, int k) {
    if (!a || !b || !out || !err) return false;
    if (m <= 0 || n <= 0 || k <= 0 || (m & 3) || (n & 31) || (k & 31)) return false;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) return false;
    if (reinterpret_cast<uintptr_t>(out) & 15) return false;
    return true;
}

}  // namespace

extern "C" int ozk_gemm_residues(const int8_t* Ares, const int8_t* Bres, int m, int n, int k, int N, uint8_t* X,
                                 int32_t* err, ozk_stream_t stream) {
    if (!shapes_ok(Ares, Bres, X, err, m, n, k) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (use_pair_tiles(m, n)) return launch_gemm2<MODE_RESIDUE>(Ares, Bres, m, n, k, N, X, err, st);
    return launch_gemm<MODE_RESIDUE>(Ares, Bres, m, n, k, N, X, err, st);
}

extern "C" int ozk_gemm_i32(const int8_t* A_plane, const int8_t* B_plane, int m, int n, int k, int32_t* C32,
                            int32_t* err, ozk_stream_t stream) {
    if (!shapes_ok(A_plane, B_plane, C32, err, m, n, k) || k > OZK_KSEG) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (use_pair_tiles(m, n)) return launch_gemm2<MODE_I32>(A_plane, B_plane, m, n, k, 1, C32, err, st);
    return launch_gemm<MODE_I32>(A_plane, B_plane, m, n, k, 1, C32, err, st);
}

extern "C" int ozk_wait_selftest(int role, int64_t limit_ns, int32_t* err, int64_t* waited_ns, ozk_stream_t stream) {
    if (!err || !waited_ns || (reinterpret_cast<uintptr_t>(waited_ns) & 7) || role < 0 || role > 1 ||
        limit_ns < 1000 || limit_ns > (int64_t)WAIT_LIMIT_NS)
        return OZK_ERR_ARG;
    DeviceInfo* d = nullptr;
    const int rc = device_info(&d);
    if (rc != OZK_OK) return rc;
    wait_selftest_kernel<<<1, 96, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        role, (uint64_t)limit_ns, err, reinterpret_cast<long long*>(waited_ns));
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_device_sm_count(int* out) {
    if (!out) return OZK_ERR_ARG;
    DeviceInfo* d = nullptr;
    const int rc = device_info(&d);
    if (rc != OZK_OK) return rc;
    *out = d->sms;
    return OZK_OK;
}
