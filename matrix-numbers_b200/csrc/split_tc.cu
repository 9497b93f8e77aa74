// Stage 3a on the tensor cores: the residue split with its byte-string products issued as tcgen05.mma.
//
// Semantics as in split.cu (the reference's decomp / resid / resA_k / resB_k, code/ozaki_engine.py:971-1038):
// residue_t = X mod m_t in the symmetric int8 range [-floor(m_t / 2), ceil(m_t / 2) - 1], X = sign(v) x,
// x = round(|v| 2^ag) (round half away from zero), ag = p - r_i + gamma_l for A and p - c_j - gamma_l for B.
// This kernel covers |X| < 2^120 (p <= 119); split.cu's kernel takes larger p.
//
// Method (this build's own).
// * String.  y = |v| 2^ag is formed in FP64 by exponent arithmetic (exact), and x = floor(y + 1/2) is cut into
//   chunks by FP64 operations with directed rounding: A = floor(y / 2^104), B = floor((y mod 2^104) / 2^52),
//   C = floor((y mod 2^52) + 1/2), each read off the bit pattern of 2^52 + chunk (fma / add rounding toward zero;
//   the remainders y mod 2^104, y mod 2^52 are exact).  C reaches 2^52 only when A = B = 0.  The 128 bits of x are
//   stored as a little-endian 16-byte string, all 16 bytes one's complemented when v < 0.  With byte weights
//   w_q = 2^(8q) mod m (q < 15) and w_15 = -(sum_{q<15} 2^(8q)) mod m, the weighted byte sum s = sum_q b_q w_q is
//   congruent to X mod m for either sign (the complement adds 255 sum_q 2^(8q), which w_15 cancels) and lies in
//   [0, 16 * 255^2] < 2^20.
// * Products.  A tile is 1024 elements: 128 rows of 8 strings in a K-major, 128-byte-swizzled shared-memory tile
//   (row R = TMEM lane R).  MMA j (M = 128, K = 32, N = 4 CW) reads strings 2j and 2j + 1 of every row against the
//   constant weight operand, whose column (2h + sigma) CW + i carries modulus h TPH + i's weights in the K-half of
//   string slot sigma.  TMEM column j 4 CW + (2h + sigma) CW + i of lane R then holds s of string 2j + sigma of row
//   R for modulus h TPH + i.
// * Residues.  Warps w and w + 4 share TMEM lanes 32 (w % 4) ..; warp half h takes moduli h TPH .. h TPH + TPH - 1.
//   q = floor((s + h_t) / m_t) is the high word of s ceil(2^32 / m_t) + h_t ceil(2^32 / m_t) (exact for
//   s + h_t < 2^24), h_t = floor(m_t / 2), and the residue is the low byte of s - m_t q (for m_0 = 256, of s
//   itself).  The eight strings of a row
//   are eight consecutive elements of one vector, so each modulus leaves as one 8-byte store.
// * Vectors.  A: a tile is 1024 consecutive elements of row-major A (elements e0 + 8R .. e0 + 8R + 7 in row R),
//   loaded by TMA as 64 rows of 16 doubles (128-byte swizzle).  B: a tile is 16 columns x 64 contraction indices
//   (TMA box {16, 64} of row-major B); row R holds column R / 8, indices 8 (R % 8) .. 8 (R % 8) + 7.  Thread (R, h)
//   builds four strings of row R: A its indices 4h .. 4h + 3; B index (4h + step) XOR tau(R % 8), tau the
//   multiplication by x in GF(8) = GF(2)[x] / (x^3 + x + 1), so that both its shared-memory reads of B and its
//   string writes are free of bank conflicts (tau and tau + identity are both bijections).
// * Pipeline per CTA (8 warps, two CTAs per SM for TMEM's 2 x 256 columns): TMA loads run STAGES tiles ahead; in
//   iteration i all threads build tile i + 1's strings (second string buffer) while tile i's MMAs run, then read
//   tile i's sums from TMEM and store its residues, then arrive (one arrival per warp) on an mbarrier; thread 0 alone
//   waits for the eight arrivals and issues tile i + 1's MMAs and the next load, while the other warps go on.
//   Every wait is bounded (4 s); a wait that runs out ORs OZK_DEVERR_TIMEOUT_SPLIT into *err and the CTA drains
//   its loads and MMAs, frees TMEM and leaves.
#include <cuda.h>
#include <stdlib.h>
#include <string.h>

#include "ozk_common.cuh"
#include "tc_ptx.cuh"

namespace {

using namespace ozk_ptx;

namespace stc {
constexpr int THREADS = 256;                 // 8 warps
constexpr int ROWS = 128;                    // MMA M, TMEM lanes
constexpr int TILE = 1024;                   // elements per tile (8 per row)
constexpr int X_BYTES = TILE * 8;            // one FP64 tile: 64 rows of 128 bytes
constexpr int STAGES = 5;
constexpr int S_BYTES = ROWS * 128;          // one string tile
constexpr int W_BYTES = 64 * 128;            // weight operand: up to 64 columns
constexpr int TMEM_COLS = 256;
constexpr int NUM_BARS = STAGES + 3;         // full[s], mma, drain, done
// > 227 KB / 3: at most two CTAs per SM, as TMEM holds two allocations of 256 columns
constexpr int SMEM_BYTES = 1024 + STAGES * X_BYTES + 2 * S_BYTES + W_BYTES + NUM_BARS * 8 + 16;
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;
static_assert(3 * (SMEM_BYTES + 1024) > 228 * 1024, "more than two CTAs per SM would contend for TMEM");
}  // namespace stc

struct TcTables {
    uint32_t W[OZK_NMAX][4];          // the 16 byte weights of modulus t, four per word (little-endian)
    uint32_t M[OZK_NMAX];             // ceil(2^32 / m_t)
    uint32_t nP[OZK_NMAX];            // -m_t mod 2^32
    unsigned long long hM[OZK_NMAX];  // floor(m_t / 2) ceil(2^32 / m_t)
};

constexpr int pow2_mod_tc(int e, int P) {
    int w = 1 % P;
    for (int i = 0; i < e; i++) w = (w * 2) % P;
    return w;
}

constexpr TcTables make_tc_tables() {
    TcTables t{};
    for (int i = 0; i < OZK_NMAX; i++) {
        const int P = ozk_mod(i);
        int g15 = 0;
        for (int q = 0; q < 15; q++) {
            const int w = pow2_mod_tc(8 * q, P);
            g15 = (g15 + w) % P;
            t.W[i][q >> 2] |= (uint32_t)w << (8 * (q & 3));
        }
        t.W[i][3] |= (uint32_t)((P - g15) % P) << 24;
        const unsigned long long M = (0x100000000ULL + (unsigned long long)P - 1ULL) / (unsigned long long)P;
        t.M[i] = (uint32_t)M;
        t.nP[i] = 0u - (uint32_t)P;
        t.hM[i] = (unsigned long long)(P / 2) * M;
    }
    return t;
}

__constant__ TcTables c_tc = make_tc_tables();

struct TcArgs {
    const int32_t* vexp;              // r (A) or c (B)
    const int32_t* gam;
    const int32_t* p_dev;
    int8_t* out;
    int32_t* err;
    unsigned long long plane_bytes;   // V k
    unsigned long long kdiv;          // A: floor(2^64 / k) + 1 (row of a flat index by one multiply-high)
    unsigned E;                       // A: m k
    int k, N, ntiles, lblocks;        // lblocks (B): tiles along the contraction index
    unsigned long long ldiv;          // B: floor(2^64 / lblocks) + 1 for lblocks > 1 (column block by a multiply-high)
};

// B tile T -> (column block, contraction block): T / lblocks by a multiply-high, exact for T < 2^32 (lblocks = 1,
// where floor(2^64 / lblocks) + 1 does not fit 64 bits, is the identity)
__device__ __forceinline__ void b_tile(const TcArgs& a, int T, int& jb, int& lb) {
    jb = a.lblocks == 1 ? T : (int)__umul64hi((unsigned long long)(unsigned)T, a.ldiv);
    lb = T - jb * a.lblocks;
}

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int32_t* err) {
    *abort_flag = 1;
    atomicOr(err, OZK_DEVERR_TIMEOUT_SPLIT);
}

// y = |v| 2^ag for a normal v with the exponent field moved (0 when it falls below 2^-1022, where x rounds to 0);
// *sub flags a nonzero subnormal v, which scaled_subnormal handles
__device__ __forceinline__ double scaled_normal(double v, int ag, bool& sub) {
    const uint32_t hi = (uint32_t)__double2hiint(v), lo = (uint32_t)__double2loint(v);
    const uint32_t E = (hi >> 20) & 0x7FFu;
    sub = E == 0u && ((hi & 0xFFFFFu) | lo) != 0u;
    const double y = __hiloint2double((int)((hi & 0x7FFFFFFFu) + ((uint32_t)ag << 20)), (int)lo);
    return (E != 0u && (int)E + ag >= 1) ? y : 0.0;
}
__device__ __noinline__ double scaled_subnormal(double v, int ag) {
    const uint32_t mh = (uint32_t)__double2hiint(v) & 0xFFFFFu, lo = (uint32_t)__double2loint(v);
    return ldexp(__hiloint2double((int)(0x43300000u | mh), (int)lo) - 0x1p52, ag - 1074);
}

// The 16-byte string of x = floor(y + 1/2) (file comment), complemented by msk (all ones for v < 0).  WIDE: x may
// reach 2^104 (p > 100), so the top chunk is needed.
template <bool WIDE>
__device__ __forceinline__ uint4 string_of(double y, uint32_t msk) {
    uint32_t A = 0u;
    double y1 = y;
    if (WIDE) {
        const double a = __fma_rz(y, 0x1p-104, 0x1p52);     // 2^52 + floor(y / 2^104)
        A = (uint32_t)__double2loint(a);
        y1 = fma(-(a - 0x1p52), 0x1p104, y);                // y mod 2^104
    }
    const double b = __fma_rz(y1, 0x1p-52, 0x1p52);         // 2^52 + floor(y1 / 2^52)
    const double y2 = fma(-(b - 0x1p52), 0x1p52, y1);       // y mod 2^52
    const double c = __dadd_rz(__dadd_rz(y2, 0.5), 0x1p52); // 2^52 + floor(y2 + 1/2), at most 2^53
    const uint32_t Blo = (uint32_t)__double2loint(b), Bhi = (uint32_t)__double2hiint(b) & 0xFFFFFu;
    const uint32_t Clo = (uint32_t)__double2loint(c), Chi = (uint32_t)__double2hiint(c) - 0x43300000u;
    return make_uint4(Clo ^ msk, (Chi | (Blo << 20)) ^ msk, __funnelshift_r(Blo, Bhi, 12) ^ msk,
                      ((Bhi >> 12) | (A << 8)) ^ msk);
}

// low byte of s - m_t floor((s + h_t) / m_t): the symmetric residue, as an int in [-128, 127]; for m_0 = 256 it is
// the low byte of s itself, sign-extended
__device__ __forceinline__ int residue_tc(uint32_t s, int t) {
    if (t == 0) return (int)(int8_t)(uint8_t)s;
    const unsigned long long prod = (unsigned long long)s * c_tc.M[t] + c_tc.hM[t];
    return (int)(s + c_tc.nP[t] * (uint32_t)(prod >> 32));
}

// bytes 2, 3 of a packed word (r2, r3); then bytes 0, 1 (r0, r1) over it
__device__ __forceinline__ uint32_t pack_hi(int r2, int r3) {
    uint32_t w;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(w) : "r"(r3), "r"(r2));
    return w;
}
__device__ __forceinline__ uint32_t pack_lo(int r0, int r1, uint32_t hi) {
    uint32_t w;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(r1), "r"(r0), "r"(hi));
    return w;
}

// Residues of one tile for the moduli of warp half HALF: w[i] holds bytes of elements 8R .. 8R + 7 (two words).
// Reads MMAs 2 pr + 1 then 2 pr: strings 4 pr + 2, 4 pr + 3 give bytes 2, 3, strings 4 pr, 4 pr + 1 bytes 0, 1.
template <int TPH, int CW, int HALF>
__device__ __forceinline__ void tile_residues(uint32_t lanes, uint32_t (&w0)[TPH], uint32_t (&w1)[TPH]) {
    constexpr int NCOLS = 4 * CW;
#pragma unroll
    for (int pr = 0; pr < 2; pr++) {
        uint32_t v[4][TPH];   // (MMA 2 pr + 1: slot 0, slot 1), (MMA 2 pr: slot 0, slot 1)
        tmem_ld_cols<TPH>(lanes + (uint32_t)((2 * pr + 1) * NCOLS + (2 * HALF) * CW), v[0]);
        tmem_ld_cols<TPH>(lanes + (uint32_t)((2 * pr + 1) * NCOLS + (2 * HALF + 1) * CW), v[1]);
        tmem_ld_cols<TPH>(lanes + (uint32_t)((2 * pr) * NCOLS + (2 * HALF) * CW), v[2]);
        tmem_ld_cols<TPH>(lanes + (uint32_t)((2 * pr) * NCOLS + (2 * HALF + 1) * CW), v[3]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < TPH; i++) {
            constexpr int t0 = HALF * TPH;
            const uint32_t hw = pack_hi(residue_tc(v[0][i], t0 + i), residue_tc(v[1][i], t0 + i));
            const uint32_t w = pack_lo(residue_tc(v[2][i], t0 + i), residue_tc(v[3][i], t0 + i), hw);
            if (pr == 0) w0[i] = w;
            else w1[i] = w;
        }
    }
}

template <bool IS_B, int TPH>
__global__ void __launch_bounds__(stc::THREADS, 2)
    split_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ TcArgs a) {
    using namespace stc;
    constexpr int CW = TPH > 8 ? 16 : (TPH > 4 ? 8 : 4);
    constexpr int NCOLS = 4 * CW;                            // product columns of one MMA (multiple of 16)
    constexpr uint32_t IDESC = (2u << 4) | ((uint32_t)(NCOLS >> 3) << 17) | ((uint32_t)(ROWS >> 4) << 24);
    static_assert(4 * NCOLS <= TMEM_COLS && NCOLS * 128 <= W_BYTES, "tile sizes");

    const int p = *a.p_dev;
    if (p > 119) return;   // split.cu's kernel runs for these (the same decision in every thread)

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sX = smem;
    uint8_t* sS = sX + STAGES * X_BYTES;
    uint8_t* sW = sS + 2 * S_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sW + W_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int half = warp >> 2;
    const int R = 32 * (warp & 3) + lane;                    // string row = TMEM lane
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    const uint32_t mma_bar = bar0 + 8u * STAGES, drain_bar = mma_bar + 8u, done_bar = drain_bar + 8u;

    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) mbar_init(full_bar(s), 1);
        mbar_init(mma_bar, 1);
        mbar_init(drain_bar, 1);
        mbar_init(done_bar, THREADS / 32);      // one arrival per warp and tile
        *abort_flag = 0;
        mbar_fence_init();
        tma_prefetch_desc(&tmX);
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    // the weight operand: row n, logical 16-byte chunk c (K bytes 16c ..) stored at chunk c ^ (n & 7); the 32-byte
    // K-slice of every MMA holds the same two halves
    for (int idx = tid; idx < NCOLS * 8; idx += THREADS) {
        const int n = idx >> 3, pc = idx & 7, c = pc ^ (n & 7);
        const int blk = n / CW, i = n % CW, t = (blk >> 1) * TPH + i;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if ((c & 1) == (blk & 1) && i < TPH && t < a.N)
            w = make_uint4(c_tc.W[t][0], c_tc.W[t][1], c_tc.W[t][2], c_tc.W[t][3]);
        *reinterpret_cast<uint4*>(sW + n * 128 + pc * 16) = w;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint32_t wbase = smem_addr(sW);
    const bool wide = p > 100;

    const int G = (int)gridDim.x;
    const int nloc = (int)blockIdx.x < a.ntiles ? (a.ntiles - 1 - (int)blockIdx.x) / G + 1 : 0;
    // thread 0's bookkeeping, so that it can drain what is in flight if a wait runs out
    int loads_issued = 0, loads_seen = 0;
    bool mma_pending = false;

    auto issue_load = [&](int i) {
        const int s = i % STAGES, T = (int)blockIdx.x + i * G;
        mbar_arrive_expect_tx(full_bar(s), (uint32_t)X_BYTES);
        const uint32_t dst = smem_addr(sX + s * X_BYTES);
        if (IS_B) {
            int jb, lb;
            b_tile(a, T, jb, lb);
            tma_load_2d(dst, &tmX, jb * 16, lb * 64, full_bar(s));
        }
        else tma_load_2d(dst, &tmX, 0, T * 64, full_bar(s));
        loads_issued++;
    };
    auto issue_mma = [&](int i) {
        const uint32_t sbase = smem_addr(sS + (i & 1) * S_BYTES);
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; j++)
            umma_i8(tmem_base + (uint32_t)(j * NCOLS), umma_desc_sw128(sbase + 32u * j), umma_desc_sw128(wbase + 32u * j),
                    IDESC, 0u);
        umma_commit(mma_bar);
        mma_pending = true;
    };

    // logical string index in row R of this thread's four strings (the same in every tile)
    int rowsel[4];
    {
        const int g = R & 7, tau = ((g << 1) & 7) ^ ((g >> 2) * 3);
#pragma unroll
        for (int u = 0; u < 4; u++) rowsel[u] = IS_B ? (4 * half + u) ^ tau : 4 * half + u;
    }
    // the scaling exponents ag of this thread's four elements of local tile i (loaded one tile ahead of their use)
    auto fetch_ag = [&](int i, int (&ag)[4]) {
        const int T = (int)blockIdx.x + i * G;
        if (!IS_B) {
            const unsigned e = (unsigned)T * (unsigned)TILE + 8u * (unsigned)R + 4u * (unsigned)half;
            const bool in = e < a.E;
            const unsigned row = in ? (unsigned)__umul64hi((unsigned long long)e, a.kdiv) : 0u;
            const unsigned l = in ? e - row * (unsigned)a.k : 0u;
            const int base = p - __ldg(a.vexp + row);
#pragma unroll
            for (int u = 0; u < 4; u++) ag[u] = base + __ldg(a.gam + l + u);
        } else {
            int jb, lb;
            b_tile(a, T, jb, lb);
            const int base = p - __ldg(a.vexp + jb * 16 + (R >> 3));
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int l = lb * 64 + 8 * (R & 7) + rowsel[u];
                ag[u] = base - __ldg(a.gam + (l < a.k ? l : 0));
            }
        }
    };

    // this thread's four strings of local tile i, written to string buffer i & 1; false if the load wait ran out
    // (decided per warp)
    auto build_strings = [&](int i, const int (&ag)[4]) -> bool {
        const int s = i % STAGES;
        bool ok = mbar_wait_bounded(full_bar(s), (uint32_t)((i / STAGES) & 1), abort_flag, WAIT_LIMIT_NS);
        if (!ok && !*abort_flag) raise_abort(abort_flag, a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) return false;
        if (tid == 0) loads_seen = i + 1;
        const uint8_t* xs = sX + s * X_BYTES;
        double x[4];
        if (!IS_B) {
            // elements 8R + 4 half .. : tile row R / 2, chunks 4 (R & 1) + 2 half + {0, 1} (swizzled by row & 7)
            const int rho = R >> 1;
#pragma unroll
            for (int v2 = 0; v2 < 2; v2++) {
                const int ch = 4 * (R & 1) + 2 * half + v2;
                const double2 d = *reinterpret_cast<const double2*>(xs + rho * 128 + 16 * (ch ^ (rho & 7)));
                x[2 * v2] = d.x;
                x[2 * v2 + 1] = d.y;
            }
        } else {
            // column R / 8 of the tile, index 8 (R & 7) + rowsel: tile row l, chunk (column / 2) ^ (l & 7)
            const int j = R >> 3;
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int l = 8 * (R & 7) + rowsel[u];
                x[u] = *reinterpret_cast<const double*>(xs + l * 128 + 16 * ((j >> 1) ^ (l & 7)) + 8 * (j & 1));
            }
        }
        double y[4];
        bool any_sub = false;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            bool sub;
            y[u] = scaled_normal(x[u], ag[u], sub);
            any_sub |= sub;
        }
        if (__any_sync(0xffffffffu, any_sub)) {   // subnormal inputs: rare, off the common path
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint32_t hi = (uint32_t)__double2hiint(x[u]), lo = (uint32_t)__double2loint(x[u]);
                if (((hi >> 20) & 0x7FFu) == 0u && ((hi & 0xFFFFFu) | lo) != 0u) y[u] = scaled_subnormal(x[u], ag[u]);
            }
        }
        uint8_t* srow = sS + (i & 1) * S_BYTES + R * 128;
        if (wide) {
#pragma unroll
            for (int u = 0; u < 4; u++)
                *reinterpret_cast<uint4*>(srow + 16 * (rowsel[u] ^ (R & 7))) =
                    string_of<true>(y[u], (uint32_t)(__double2hiint(x[u]) >> 31));
        } else {
#pragma unroll
            for (int u = 0; u < 4; u++)
                *reinterpret_cast<uint4*>(srow + 16 * (rowsel[u] ^ (R & 7))) =
                    string_of<false>(y[u], (uint32_t)(__double2hiint(x[u]) >> 31));
        }
        fence_proxy_async_smem();
        return true;
    };

    // residues of local tile i from TMEM, stored; false if the MMA wait ran out (decided per warp)
    auto store_residues = [&](int i) -> bool {
        bool ok = mbar_wait_bounded(mma_bar, (uint32_t)(i & 1), abort_flag, WAIT_LIMIT_NS);
        if (!ok && !*abort_flag) raise_abort(abort_flag, a.err);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) return false;
        if (tid == 0) mma_pending = false;
        tc_fence_after();
        const uint32_t lanes = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16);
        uint32_t w0[TPH], w1[TPH];
        if (half == 0) tile_residues<TPH, CW, 0>(lanes, w0, w1);
        else tile_residues<TPH, CW, 1>(lanes, w0, w1);
        const int T = (int)blockIdx.x + i * G;
        unsigned long long off;
        bool in;
        if (!IS_B) {
            off = (unsigned long long)T * TILE + 8ull * (unsigned)R;
            in = off < a.E;
        } else {
            int jb, lb;
            b_tile(a, T, jb, lb);
            const int l = lb * 64 + 8 * (R & 7);
            off = (unsigned long long)(jb * 16 + (R >> 3)) * (unsigned)a.k + (unsigned)l;
            in = l < a.k;
        }
        if (in) {
            int8_t* o = a.out + off + (unsigned long long)(half * TPH) * a.plane_bytes;
#pragma unroll
            for (int t = 0; t < TPH; t++) {
                if (half * TPH + t < a.N) *reinterpret_cast<uint2*>(o) = make_uint2(w0[t], w1[t]);
                o += a.plane_bytes;
            }
        }
        return true;
    };

    if (tid == 0)
        for (int i = 0; i < STAGES && i < nloc; i++) issue_load(i);
    bool run = nloc > 0;
    int ag_next[4] = {0, 0, 0, 0};
    if (run) {
        fetch_ag(0, ag_next);
        const bool ok = build_strings(0, ag_next);
        if (nloc > 1) fetch_ag(1, ag_next);
        if (__syncthreads_or(ok ? 0 : 1)) run = false;
        else if (tid == 0) {
            if (STAGES < nloc) issue_load(STAGES);
            issue_mma(0);
        }
    }
    for (int i = 0; run && i < nloc; i++) {
        bool ok = true;
        if (i + 1 < nloc) {
            ok = build_strings(i + 1, ag_next);
            if (i + 2 < nloc) fetch_ag(i + 2, ag_next);
        }
        ok = store_residues(i) && ok;
        // this warp is done with tile i's TMEM and with tile i + 1's strings and input stage: one arrival; only the
        // issuing thread waits for all warps, the others go on to the next tile
        tc_fence_before();
        ok = __all_sync(0xffffffffu, ok);
        __syncwarp();
        if (lane == 0) mbar_arrive(done_bar);
        if (!ok) break;
        if (warp == 0 && i + 1 < nloc) {
            bool got = true;
            if (lane == 0) {
                got = mbar_wait_bounded(done_bar, (uint32_t)(i & 1), abort_flag, WAIT_LIMIT_NS);
                if (!got) {
                    if (!*abort_flag) raise_abort(abort_flag, a.err);
                } else {
                    if (i + 1 + STAGES < nloc) issue_load(i + 1 + STAGES);
                    issue_mma(i + 1);
                }
            }
            if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) break;   // warp 0 leaves as one
        }
    }

    // leave only when nothing of this CTA is in flight (only a wait that ran out can leave loads or MMAs behind)
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        int dummy = 0;
        if (mma_pending) {
            umma_commit(drain_bar);
            mbar_wait_bounded(drain_bar, 0u, &dummy, WAIT_LIMIT_NS);
        }
        for (; loads_seen < loads_issued; loads_seen++)
            mbar_wait_bounded(full_bar(loads_seen % STAGES), (uint32_t)((loads_seen / STAGES) & 1), &dummy,
                              WAIT_LIMIT_NS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        __syncwarp();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- host ----------------------------------------------------------------------------------------------------
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

struct StcDevice {
    int sms = 0;
    bool attr[2][17] = {};
};
StcDevice g_stc_dev[64];

template <bool IS_B, int TPH>
int launch_stc(const CUtensorMap& map, const TcArgs& args, cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OZK_ERR_DEVICE;
    StcDevice& d = g_stc_dev[dev];
    if (d.sms == 0 && cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return OZK_ERR_DEVICE;
    if (!d.attr[IS_B ? 1 : 0][TPH]) {
        if (cudaFuncSetAttribute(split_tc_kernel<IS_B, TPH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 stc::SMEM_BYTES) != cudaSuccess)
            return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
        d.attr[IS_B ? 1 : 0][TPH] = true;
    }
    const int grid = args.ntiles < 2 * d.sms ? args.ntiles : 2 * d.sms;
    split_tc_kernel<IS_B, TPH><<<grid, stc::THREADS, stc::SMEM_BYTES, st>>>(map, args);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

template <bool IS_B>
int dispatch_stc(int tph, const CUtensorMap& map, const TcArgs& args, cudaStream_t st) {
    switch (tph) {
        case 2: return launch_stc<IS_B, 2>(map, args, st);
        case 4: return launch_stc<IS_B, 4>(map, args, st);
        case 6: return launch_stc<IS_B, 6>(map, args, st);
        case 8: return launch_stc<IS_B, 8>(map, args, st);
        case 9: return launch_stc<IS_B, 9>(map, args, st);
        case 10: return launch_stc<IS_B, 10>(map, args, st);
        case 12: return launch_stc<IS_B, 12>(map, args, st);
        case 14: return launch_stc<IS_B, 14>(map, args, st);
        case 16: return launch_stc<IS_B, 16>(map, args, st);
        default: return OZK_ERR_ARG;
    }
}

bool tc_split_enabled() {
    static int enabled = -1;
    if (enabled < 0) {
        const char* s = getenv("OZK_SPLIT_TC");
        enabled = (s && s[0] == '0') ? 0 : 1;
    }
    return enabled == 1;
}

}  // namespace

// Launches the tensor-core split of A (is_b = 0: m x k row-major) or B (is_b = 1: k x n row-major) when its shape
// qualifies; *p_lo is then 120 (the general kernel only runs for p >= 120), else 0 and nothing was launched.
int ozk_split_tc_launch(int is_b, const double* src, const int32_t* vexp, const int32_t* gam, const int32_t* p_dev,
                        int V, int k, int N, int8_t* out, int32_t* err, cudaStream_t st, int* p_lo) {
    *p_lo = 0;
    if (!tc_split_enabled() || !err) return OZK_OK;
    const unsigned long long E = (unsigned long long)V * (unsigned long long)k;
    if (E >= (1ULL << 32) || (k & 31) || (reinterpret_cast<uintptr_t>(src) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 7))
        return OZK_OK;
    if (is_b && (V & 15)) return OZK_OK;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return OZK_OK;
    TcArgs args;
    memset(&args, 0, sizeof(args));
    args.vexp = vexp;
    args.gam = gam;
    args.p_dev = p_dev;
    args.out = out;
    args.err = err;
    args.plane_bytes = E;
    args.k = k;
    args.N = N;
    CUtensorMap map;
    const cuuint32_t box[2] = {16u, 64u};
    const cuuint32_t estr[2] = {1u, 1u};
    if (!is_b) {
        // the flat elements as rows of 16 doubles; rows past the end are zero-filled
        const cuuint64_t dims[2] = {16u, (cuuint64_t)(E / 16)};
        const cuuint64_t strides[1] = {128u};
        if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double*>(src), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return OZK_OK;
        args.E = (unsigned)E;
        args.kdiv = ~0ULL / (unsigned long long)k + 1ULL;
        args.ntiles = (int)((E + stc::TILE - 1) / stc::TILE);
        args.lblocks = 1;
    } else {
        // B (k rows x V columns), box of 16 columns x 64 contraction indices; indices past k are zero-filled
        const cuuint64_t dims[2] = {(cuuint64_t)V, (cuuint64_t)k};
        const cuuint64_t strides[1] = {(cuuint64_t)V * 8u};
        if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double*>(src), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return OZK_OK;
        args.E = (unsigned)E;
        args.lblocks = (k + 63) / 64;
        args.ldiv = ~0ULL / (unsigned long long)args.lblocks + 1ULL;
        args.ntiles = (V / 16) * args.lblocks;
    }
    const int half = (N + 1) / 2;
    const int tph = half <= 2 ? 2 : half <= 4 ? 4 : half <= 6 ? 6 : half <= 8 ? 8 : half <= 9 ? 9 : half <= 10 ? 10
                  : half <= 12 ? 12 : half <= 14 ? 14 : 16;
    const int rc = is_b ? dispatch_stc<true>(tph, map, args, st) : dispatch_stc<false>(tph, map, args, st);
    if (rc == OZK_OK) *p_lo = 120;
    return rc;
}
