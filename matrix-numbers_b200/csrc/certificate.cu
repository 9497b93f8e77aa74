// Full-matrix certificate of the plane count (the reference's full_certificate, code/ozaki_engine.py:1542-1583):
// a lower bound of D_ij = sum_l |A_il||B_lj| on EVERY entry from one FP16 tensor-core product of the scaled
// magnitudes, and from it the smallest p for which the error bound E_ij(p) <= tau D_ij / safety holds on all (i, j).
//
// Reference arithmetic, kept operation for operation (each step rounded once, in this order):
//   As_il = fp16(fp32((|A_il| (2^gamma_l 2^-r_i)) (1 - 2^-10)))      (torch: fp64 products, then .to(float16), which
//   Bs_lj = fp16(fp32((|B_lj| (2^-c_j / 2^gamma_l)) (1 - 2^-10)))     converts through float32)
//   Dl_ij = sum_l As_il Bs_lj with FP32 accumulation (the reference's torch.mm(..., out_dtype=float32))
//   D = ((Dl (1 - 8 k 2^-24)) 2^r_i) 2^c_j;  thr = (tau D) / safety;  F1 = 0.5 (2^r_i sB_j + 2^c_j sA_i);
//   F2 = ((0.25 k) 2^r_i) 2^c_j;  xmax = (2 thr) / (F1 + sqrt(F1 F1 + (4 F2) thr))
//   need = max over D > 0 of -log2(xmax) = -log2(min xmax)  (log2 is monotone), uncertified = #(not D > 0).
// The accumulation order of the FP32 sums differs from cuBLAS's (both are covered by the 8 k 2^-24 derating).
//
// Design (sm_100a): prep kernels write the FP16 operands K-major (A16[m][k], B16t[n][k], B transposed through
// shared memory); the product is a persistent tcgen05.mma kind::f16 kernel (128 x 256 tiles, 4-stage TMA ring with
// 128-byte swizzle, FP32 accumulators double-buffered in TMEM), whose 8 epilogue warps evaluate the bound for every
// entry straight out of TMEM and reduce min xmax / the uncertified count per warp, so the m x n matrix D never
// reaches HBM (an optional debug output writes D).  Only the minimum matters, so an entry is skipped once a lower
// bound of its xmax cannot beat the running minimum (published across CTAs after every tile): a lower bound of the
// formula in which the row and column scalings cancel, evaluated in FP32 without branches for 32 entries at a time
// (fast_term); the exact reference formula runs only for the entries near the minimum and for rows or columns
// outside that bound's range.  Waits are bounded; no cluster multicast.
#include <cuda.h>
#include <cuda_fp16.h>

#include "ozk_common.cuh"
#include "tc_ptx.cuh"

using namespace ozk_ptx;

namespace {

constexpr int BM = 128, BN = 256, BKB = 128;       // BKB: bytes of K per stage (64 fp16)
constexpr int STAGES = 4;
constexpr uint32_t A_BYTES = BM * BKB;
constexpr uint32_t B_BYTES = BN * BKB;
constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr int GROUP_M = 16;
constexpr uint32_t IDESC = umma_idesc_f16_f32(BM, BN);
constexpr int NUM_BARS = 2 * STAGES + 5;
constexpr int COLSTAGE_DOUBLES = 2 * 32 + 16;     // per epilogue warp: 2^c_j, sB_j (f64) and sB_j / 2^c_j (f32)
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + 1024 + 256 + (size_t)EPI_WARPS * COLSTAGE_DOUBLES * 8;
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;
constexpr unsigned long long kEmpty = 0xFFFFFFFFFFFFFFFFull;   // "no certified entry" (above every double's bits)

static_assert(NUM_BARS * 8 + 16 <= 256, "barrier area");

struct CertParams {
    const double* rowscale;   // 2^r_i
    const double* colscale;   // 2^c_j
    const double* sA;
    const double* sB;
    double derate, tau, safety, f2k;   // 1 - 8 k 2^-24, tau, safety, 0.25 k
    double inv_safety;                 // 1 / safety when safety is a power of two (then x / safety == x * inv_safety)
    int safety_pow2;
    float c8, k4;                      // the fast bound's constants (fast_term); c8 NaN: no fast bound
    int m, n, k;
    unsigned long long* xmin;          // bit pattern of min xmax over certified entries (atomicMin)
    unsigned long long* uncertified;
    double* dbg_D;                     // optional m x n output of D
};

__device__ __forceinline__ double pow2i(int e) { return ldexp(1.0, e); }

// g[l] = 2^gamma_l and ig[l] = 2^-gamma_l (torch.exp2 of the integer gamma, exact; ig is only used where it is a
// finite power of two, so that x * ig[l] and x / g[l] are the same correctly rounded value)
__global__ void cert_pow2_kernel(const int32_t* __restrict__ gam, int k, double* __restrict__ g, double* __restrict__ ig) {
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= k) return;
    g[l] = pow2i(gam[l]);
    ig[l] = pow2i(-gam[l]);
}

// As = fp16(fp32((|A| (2^gamma 2^-r)) (1 - 2^-10))), 2 elements per thread; row scales 2^r_i as a by-product
__global__ void cert_prep_a_kernel(const double* __restrict__ A, const double* __restrict__ g,
                                   const int32_t* __restrict__ r, int m, int k, __half2* __restrict__ A16,
                                   double* __restrict__ rowscale) {
    const double2* g2 = reinterpret_cast<const double2*>(g);
    for (int i = blockIdx.y; i < m; i += gridDim.y) {
        const double sr = pow2i(-r[i]);
        if (blockIdx.x == 0 && threadIdx.x == 0) rowscale[i] = pow2i(r[i]);
        const double2* row = reinterpret_cast<const double2*>(A + (size_t)i * k);
        for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < k / 2; h += gridDim.x * blockDim.x) {
            const double2 v = __ldg(row + h);
            const double2 gg = __ldg(g2 + h);
            const double f0 = __dmul_rn(gg.x, sr), f1 = __dmul_rn(gg.y, sr);
            const double x0 = __dmul_rn(__dmul_rn(fabs(v.x), f0), 1.0 - 0x1p-10);
            const double x1 = __dmul_rn(__dmul_rn(fabs(v.y), f1), 1.0 - 0x1p-10);
            A16[(size_t)i * (k / 2) + h] = __halves2half2(__float2half_rn(__double2float_rn(x0)),
                                                          __float2half_rn(__double2float_rn(x1)));
        }
    }
}

// Bs^T[j][l] = fp16(fp32((|B_lj| (2^-c_j / 2^gamma_l)) (1 - 2^-10))), through a 64 x 64 shared tile; the division
// by the power of two 2^gamma_l is a multiplication by 2^-gamma_l (the same rounded value) where that is finite
constexpr int kT = 64;
__global__ void __launch_bounds__(256) cert_prep_b_kernel(const double* __restrict__ B, const double* __restrict__ g,
                                                          const double* __restrict__ ig, const int32_t* __restrict__ c,
                                                          int k, int n, __half* __restrict__ B16t,
                                                          double* __restrict__ colscale) {
    __shared__ __half tile[kT][kT + 2];
    const int l0 = blockIdx.y * kT, j0 = blockIdx.x * kT;
    const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;   // 64 x 4
    const int j = j0 + tx;
    const double scj = j < n ? pow2i(-c[j]) : 0.0;
    if (blockIdx.y == 0 && ty == 0 && j < n) colscale[j] = pow2i(c[j]);
    for (int yy = ty; yy < kT; yy += 4) {
        const int l = l0 + yy;
        __half h = __float2half_rn(0.0f);
        if (l < k && j < n) {
            const double igl = __ldg(ig + l);
            const double f = igl < INFINITY ? __dmul_rn(scj, igl) : __ddiv_rn(scj, __ldg(g + l));
            const double x = __dmul_rn(__dmul_rn(fabs(__ldg(B + (size_t)l * n + j)), f), 1.0 - 0x1p-10);
            h = __float2half_rn(__double2float_rn(x));
        }
        tile[yy][tx] = h;
    }
    __syncthreads();
    for (int yy = ty; yy < kT; yy += 4) {
        const int jj = j0 + yy, l = l0 + tx;
        if (jj < n && l < k) B16t[(size_t)jj * k + l] = tile[tx][yy];
    }
}

__device__ __forceinline__ void decode_tile(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
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

// fast approximations (hardware reciprocal / reciprocal square root, errors far below 2^-8), used only to skip entries
__device__ __forceinline__ float rcp_approx_f32(float x) {   // at most 1 ulp from 1 / x
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

// The fast lower bound.  With R = 2^r_i 2^c_j, D = v derate R, thr = kap v R (kap = tau derate / safety),
// F1 = 0.5 R s and F2 = 0.25 k R, where s = sA_i / 2^r_i + sB_j / 2^c_j, the scalings cancel from the formula:
//   xmax = 4 kap v / (s + sqrt(s^2 + 4 k kap v)),
// and sqrt(s^2 + t) <= s + t / (2 s) gives  xmax >= 8 kap v s / (4 s^2 + 4 k kap v).
// Evaluated in FP32 with c8 = 8 kap (1 - 2^-8) and k4 = 4 k kap, its error is a few 2^-23, far inside the 2^-8
// margin, provided the reference's FP64 chain stays in the normal range, where it is within a few 2^-53 of the
// exact formula.  That holds when 2^r_i and 2^c_j lie in [2^-200, 2^200], the row and column terms in
// [2^-59, 2^60], v in {0} U [2^-48, 2^31] (sums of FP16 products of magnitudes below 1, k < 2^31) and tau and
// safety in [2^-100, 2^100]; outside, fast_term returns NaN (or the host sets c8 to NaN) and every entry of that
// row or column goes to the exact evaluation.  Inside, v = 0 gives D = 0 (uncertified); an entry with v > 0 is
// either skipped by the bound or classified by the exact evaluation.
__device__ __forceinline__ float fast_term(double s, double scale) {
    const bool ok = scale >= 0x1p-200 && scale <= 0x1p200;
    const double t = ok ? s / scale : 0.0;                       // exact scaling by a power of two
    return (ok && t >= 0x1p-59 && t <= 0x1p60) ? __double2float_rn(t) : __int_as_float(0x7fffffff);
}

// xmax of one entry, in the reference's operation order: thr = (tau D) / safety, F1 = 0.5 (rI sB + cJ sA),
// F2 = ((0.25 k) rI) cJ, xmax = (2 thr) / (F1 + sqrt(F1 F1 + (4 F2) thr))
__device__ __forceinline__ double entry_xmax(double thr, double F1, double F2) {
    const double disc = __dadd_rn(__dmul_rn(F1, F1), __dmul_rn(__dmul_rn(4.0, F2), thr));
    return __ddiv_rn(__dmul_rn(2.0, thr), __dadd_rn(F1, __dsqrt_rn(disc)));
}

__global__ void __launch_bounds__(THREADS, 1)
    cert_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CertParams cp, int32_t* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    double* colstage = reinterpret_cast<double*>(smem + STAGES * STAGE_BYTES + 256);

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

    const int m = cp.m, n = cp.n;
    const int tiles_m = (m + BM - 1) / BM, tiles_n = (n + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int kblocks = (2 * cp.k + BKB - 1) / BKB;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < tiles; u += gridDim.x) {
                int tm, tn;
                decode_tile(u, tiles_m, tiles_n, tm, tn);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_PRODUCER);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), STAGE_BYTES);
                    tma_load_3d(smem_addr(sA + stage * A_BYTES), &tmA, kb * BKB, tm * BM, 0, full_bar(stage));
                    tma_load_3d(smem_addr(sB + stage * B_BYTES), &tmB, kb * BKB, tn * BN, 0, full_bar(stage));
                    issued++;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                const long long first = issued > STAGES ? issued - STAGES : 0;
                for (long long j = first; j < issued; j++) {
                    int dummy = 0;
                    mbar_wait_bounded(full_bar((int)(j % STAGES)), (uint32_t)((j / STAGES) & 1), &dummy, WAIT_LIMIT_NS);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, acc_it = 0;
            bool ok = true, issued_any = false;
            for (int u = blockIdx.x; ok && u < tiles; u += gridDim.x) {
                const int b = (int)(acc_it & 1u);
                const uint32_t aph = (acc_it >> 1) & 1u;
                if (!mbar_wait_bounded(acce_bar(b), aph ^ 1u, abort_flag, WAIT_LIMIT_NS)) {
                    if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, WAIT_LIMIT_NS)) {
                        if (!*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_MMA);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t adesc = umma_desc_sw128(smem_addr(sA + stage * A_BYTES));
                    const uint64_t bdesc = umma_desc_sw128(smem_addr(sB + stage * B_BYTES));
#pragma unroll
                    for (int kk = 0; kk < BKB / 32; kk++)   // K = 16 fp16 = 32 bytes per instruction
                        umma_f16(d_tmem, adesc + (uint64_t)(2 * kk), bdesc + (uint64_t)(2 * kk), IDESC,
                                 (kb > 0 || kk > 0) ? 1u : 0u);
                    issued_any = true;
                    umma_commit(empty_bar(stage));
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                umma_commit(accf_bar(b));
                acc_it++;
            }
            if (!ok && issued_any) {
                umma_commit(drain_bar);
                int dummy = 0;
                mbar_wait_bounded(drain_bar, 0u, &dummy, WAIT_LIMIT_NS);
            }
        }
    } else {
        const int ew = warp - 2;
        const int quarter = warp & 3;
        const int half = ew >> 2;
        uint32_t acc_it = 0;
        unsigned long long best = kEmpty, unc = 0;
        for (int u = blockIdx.x; u < tiles; u += gridDim.x) {
            int tm, tn;
            decode_tile(u, tiles_m, tiles_n, tm, tn);
            const int row = tm * BM + quarter * 32 + lane;
            const int b = (int)(acc_it & 1u);
            const uint32_t aph = (acc_it >> 1) & 1u;
            // every lane waits; the warp proceeds only if all of them saw the accumulator (warp-uniform exit)
            const bool got = mbar_wait_bounded(accf_bar(b), aph, abort_flag, WAIT_LIMIT_NS);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0 && !*abort_flag) raise_abort(abort_flag, err, OZK_DEVERR_TIMEOUT_EPILOGUE);
                break;
            }
            __syncwarp();
            tc_fence_after();
            const bool rv = row < m;
            const double rI = rv ? cp.rowscale[row] : 0.0, sAi = rv ? cp.sA[row] : 0.0;
            const double f2r = __dmul_rn(cp.f2k, rI);                // (0.25 k) 2^r_i
            const float aI = fast_term(sAi, rI);                       // sA_i / 2^r_i, or NaN: no fast bound
            // the smallest xmax found so far by any CTA: entries whose lower bound is above it are skipped
            {
                const unsigned long long gb = *reinterpret_cast<volatile unsigned long long*>(cp.xmin);
                best = gb < best ? gb : best;
            }
#pragma unroll 1
            for (int cc = 0; cc < 4; cc++) {
                const int col_local = half * 128 + cc * 32;
                uint32_t v[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN + col_local), v);
                tmem_wait_ld();
                const int col0 = tn * BN + col_local;
                // the chunk's column terms, loaded once (lane = column) into the warp's slot and read as broadcasts
                double* cs = colstage + ew * COLSTAGE_DOUBLES;
                float* bs = reinterpret_cast<float*>(cs + 64);
                if (col0 < n) {                  // warp-uniform (n % 32 == 0)
                    __syncwarp();
                    const double cj = cp.colscale[col0 + lane], sbj = cp.sB[col0 + lane];
                    cs[lane] = cj;
                    cs[32 + lane] = sbj;
                    bs[lane] = fast_term(sbj, cj);                       // sB_j / 2^c_j, or NaN
                    __syncwarp();
                }
                if (rv && col0 < n) {            // n % 32 == 0: the 32 columns are all in range or all out
                    // Pass 1, branch-free over the chunk (the 32 entries' dependency chains interleave), in FP32:
                    // L = c8 v s / (4 s^2 + k4 v) <= xmax (1 - 2^-8) (see fast_term).  An entry with L >= the
                    // current minimum (rounded up to FP32) cannot lower it and is skipped; an entry of a row and
                    // column inside the fast bound's range with v = 0 has D = 0 and is uncertified.  Pass 2
                    // evaluates every other entry exactly, in the reference's operation order; after the first
                    // tiles of a run it is rarely taken.
                    const double bestd = best == kEmpty ? INFINITY : __longlong_as_double((long long)best);
                    const float best_up = __double2float_ru(bestd);
                    if (cp.dbg_D) {                  // optional debug output of D
#pragma unroll
                        for (int e = 0; e < 32; e++)
                            cp.dbg_D[(size_t)row * n + col0 + e] =
                                __dmul_rn(__dmul_rn(__dmul_rn((double)__uint_as_float(v[e]), cp.derate), rI), cs[e]);
                    }
                    uint32_t keep = 0, zero = 0;
#pragma unroll
                    for (int e = 0; e < 32; e++) {   // fully unrolled: v[] stays in registers
                        const float vf = __uint_as_float(v[e]);
                        const float sf = aI + bs[e];
                        const float den = __fmaf_rn(__fmul_rn(sf, sf), 4.0f, __fmul_rn(cp.k4, vf));
                        const float q = __fmul_rn(__fmul_rn(vf, sf), rcp_approx_f32(den));
                        const float L = __fmul_rn(q, cp.c8);
                        const bool in_range = sf == sf;
                        const bool pos = vf > 0.0f;
                        // q must be a normal FP32 number: a subnormal q carries only a few bits and may be rounded
                        // up by far more than the 2^-8 margin (in the proven range that only happens where L is
                        // far below xmax, but the check keeps the argument local)
                        const bool above = L >= best_up && L >= 0x1p-100f && L < INFINITY && q >= 0x1p-126f;
                        zero |= (in_range && !pos) ? (1u << e) : 0u;
                        keep |= (in_range && (!pos || above)) ? 0u : (1u << e);
                    }
                    unc += (unsigned long long)__popc(zero);
                    if (keep) {
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            if (!(keep & (1u << e))) continue;
                            const double cJ = cs[e];
                            const double vd = (double)__uint_as_float(v[e]);
                            const double D = __dmul_rn(__dmul_rn(__dmul_rn(vd, cp.derate), rI), cJ);
                            if (!(D > 0.0)) { unc++; continue; }                  // uncertified
                            const double tD = __dmul_rn(cp.tau, D);
                            const double thr = cp.safety_pow2 ? __dmul_rn(tD, cp.inv_safety) : __ddiv_rn(tD, cp.safety);
                            const double F1 = __dmul_rn(0.5, __dadd_rn(__dmul_rn(rI, cs[32 + e]), __dmul_rn(cJ, sAi)));
                            const double F2 = __dmul_rn(f2r, cJ);
                            const double x = entry_xmax(thr, F1, F2);
                            const unsigned long long xb = (unsigned long long)__double_as_longlong(x);
                            if (!(x != x) && xb < best) best = xb;           // NaN bounds are not minima
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce_bar(b));
            acc_it++;
            // publish the warp's minimum after every tile, so that the other CTAs can skip against it
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
                best = ob < best ? ob : best;
            }
            if (lane == 0 && best != kEmpty) atomicMin(cp.xmin, best);
        }
        for (int o = 16; o > 0; o >>= 1) unc += __shfl_down_sync(0xffffffffu, unc, o);
        if (lane == 0 && unc) atomicAdd(cp.uncertified, unc);
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

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

// fp16 rows [rows][k] addressed as bytes (2k per row), box {128 bytes, box_rows, 1}, 128-byte swizzle, zero fill
int make_half_map(CUtensorMap* map, const void* base, int k, int rows, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return OZK_ERR_DRIVER;
    const cuuint64_t dims[3] = {(cuuint64_t)(2 * (size_t)k), (cuuint64_t)rows, 1};
    const cuuint64_t strides[2] = {(cuuint64_t)(2 * (size_t)k), (cuuint64_t)(2 * (size_t)k) * (cuuint64_t)rows};
    const cuuint32_t box[3] = {(cuuint32_t)BKB, (cuuint32_t)box_rows, 1u};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? OZK_OK : OZK_ERR_DRIVER;
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int g_sms[64];
bool g_attr[64];

}  // namespace

extern "C" size_t ozk_certificate_workspace_bytes(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return align256((size_t)m * k * 2) + align256((size_t)n * k * 2) + align256((size_t)m * 8) +
           align256((size_t)n * 8) + 2 * align256((size_t)k * 8) + 256;
}

extern "C" int ozk_certificate(const double* A, const double* B, int m, int n, int k, const int32_t* gam,
                               const int32_t* r, const int32_t* c, const double* sA, const double* sB, double tau,
                               double safety, double* xmin, uint64_t* uncertified, double* D_out, int32_t* err,
                               void* workspace, size_t workspace_bytes, ozk_stream_t stream_) {
    if (!A || !B || !gam || !r || !c || !sA || !sB || !xmin || !uncertified || !err || !workspace) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0 || (m & 3) || (n & 31) || (k & 31)) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 255)) return OZK_ERR_ARG;
    if (workspace_bytes < ozk_certificate_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OZK_ERR_DEVICE;
    if (g_sms[dev] == 0) {
        int major = 0, sms = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10)
            return OZK_ERR_DEVICE;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return OZK_ERR_DEVICE;
        g_sms[dev] = sms;
    }
    if (!g_attr[dev]) {
        if (cudaFuncSetAttribute(cert_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES) !=
            cudaSuccess)
            return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
        g_attr[dev] = true;
    }
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    char* ws = static_cast<char*>(workspace);
    __half* A16 = reinterpret_cast<__half*>(ws);
    __half* B16t = reinterpret_cast<__half*>(ws + align256((size_t)m * k * 2));
    double* rowscale = reinterpret_cast<double*>(ws + align256((size_t)m * k * 2) + align256((size_t)n * k * 2));
    double* colscale = rowscale + align256((size_t)m * 8) / 8;
    double* g = colscale + align256((size_t)n * 8) / 8;
    double* ig = g + align256((size_t)k * 8) / 8;

    if (cudaMemsetAsync(xmin, 0xFF, 8, st) != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    if (cudaMemsetAsync(uncertified, 0, 8, st) != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    const int bx = (k / 2 + 255) / 256 < 8 ? (k / 2 + 255) / 256 : 8;
    cert_pow2_kernel<<<(k + 255) / 256, 256, 0, st>>>(gam, k, g, ig);
    OZK_CHECK_LAUNCH();
    cert_prep_a_kernel<<<dim3(bx, m < 65535 ? m : 65535), 256, 0, st>>>(A, g, r, m, k, reinterpret_cast<__half2*>(A16), rowscale);
    OZK_CHECK_LAUNCH();
    cert_prep_b_kernel<<<dim3((n + kT - 1) / kT, (k + kT - 1) / kT), 256, 0, st>>>(B, g, ig, c, k, n, B16t, colscale);
    OZK_CHECK_LAUNCH();

    CUtensorMap ta, tb;
    int rc;
    if ((rc = make_half_map(&ta, A16, k, m, BM)) != OZK_OK) return rc;
    if ((rc = make_half_map(&tb, B16t, k, n, BN)) != OZK_OK) return rc;
    CertParams cp;
    cp.rowscale = rowscale;
    cp.colscale = colscale;
    cp.sA = sA;
    cp.sB = sB;
    cp.derate = 1.0 - 8.0 * (double)k * 0x1p-24;
    cp.tau = tau;
    cp.safety = safety;
    {
        int e2 = 0;
        const double fr = frexp(safety, &e2);
        cp.safety_pow2 = (fr == 0.5) ? 1 : 0;                  // safety = 2^(e2 - 1)
        cp.inv_safety = cp.safety_pow2 ? ldexp(1.0, 1 - e2) : 0.0;
    }
    cp.f2k = 0.25 * (double)k;
    {
        const double kap = tau * cp.derate / safety;
        const double c8 = 8.0 * kap * (1.0 - 0x1p-8), k4 = 4.0 * (double)k * kap;
        const bool ok = tau >= 0x1p-100 && tau <= 0x1p100 && safety >= 0x1p-100 && safety <= 0x1p100 &&
                        c8 >= 0x1p-110 && c8 <= 0x1p110 && k4 >= 0x1p-110 && k4 <= 0x1p110;
        cp.c8 = ok ? (float)c8 : nanf("");
        cp.k4 = ok ? (float)k4 : 0.0f;
    }
    cp.m = m;
    cp.n = n;
    cp.k = k;
    cp.xmin = reinterpret_cast<unsigned long long*>(xmin);
    cp.uncertified = reinterpret_cast<unsigned long long*>(uncertified);
    cp.dbg_D = D_out;
    const long long tiles = (long long)((m + BM - 1) / BM) * ((n + BN - 1) / BN);
    const int grid = (int)(tiles < g_sms[dev] ? tiles : g_sms[dev]);
    cert_gemm_kernel<<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, cp, err);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
