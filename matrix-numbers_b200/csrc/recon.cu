// Stage 3c: CRT reconstruction, correct rounding and unscale (replaces recon_k, code/ozaki_engine.py:1040-1101).
//
// Result semantics (identical to the reference): X = the symmetric lift of the residues x_t = X[t][i][j] modulo
// M = m_0 ... m_{N-1}, i.e. the X' in [0, M) with X' = x_t mod m_t, minus M when X' > (M - 1)/2 (:1065-1072);
// |X| is rounded to 53 bits with round-to-nearest-even using a 64-bit window and a sticky bit (__ull2double_rn,
// :1073-1097), then C_ij = +-ldexp(that, 2^(r_i + c_j - 2p)) (:1098-1099) -- so the subnormal range rounds twice,
// exactly as the reference does.
//
// Method (this build's own, not Garner): with W_t = M / m_t, y_t = W_t^-1 mod m_t and V_t = (y_t W_t) mod M,
// S = sum_t x_t V_t = X (mod M) and S < 8160 M.  Every V_t is split into 40-bit chunks held as doubles; the chunk
// sums sum_t x_t V_t[c] stay below 32 * 255 * 2^40 < 2^53, so they are exact in FP64 (DFMA).  The quotient
// q = rint(S / M) comes from the chunk sums times 2^(40c) / M (its error, ~1e-11, is far below the distance of S/M
// from a half-integer, at least 2.5e-10 for every p <= pmax_bits); X = S - q M chunk by chunk, carries are
// propagated with floor(), and a rare exact check keeps X in [-M/2, M/2 - 1] for inputs outside the bound.
//
// Where the chunk sums come from.  sum_t x_t V_t[c] is a matrix product: [entries x planes] times [planes x bytes
// of V_t], with byte sums T_b = sum_t x_t byte_b(V_t) < 32 * 255 * 255 < 2^21, from which the 40-bit chunk sums are
// a[c] = sum_{j<5} T_{5c+j} 2^(8j) (exact integers below 2^53).  recon_tc_kernel runs that product on the tensor
// cores: TMA loads a tile of 128 entries x 32 planes of X straight from its plane-major layout (an MN-major UMMA
// operand, 128-byte swizzle; planes >= N are zero-filled by TMA), one tcgen05.mma kind::i8 (u8 x u8 -> s32,
// M = 128 entries, N = 32 byte columns, K = 32 planes) against the constant table of V's bytes puts T in TMEM, and
// each thread reads its entry's row (tcgen05.ld) and finishes it with the FP64 steps above.  That replaces the
// byte-to-double conversions and the N C chunk DFMAs per entry (most of the FP64 work) by one MMA per 128 entries.
// recon_kernel (all FP64) remains for problems of 2^32 entries or more, beyond the TMA path's 32-bit entry index.
#include <cuda.h>

#include "ozk_common.cuh"
#include "tc_ptx.cuh"

#include <string.h>

using namespace ozk_ptx;

namespace {

constexpr int kCMax = 7;   // 40-bit chunks of M for N = 32 (M < 2^246)

struct ReconParams {
    double V[OZK_NMAX][kCMax];   // 40-bit chunks of V_t
    double Mc[kCMax + 1];        // chunks of M
    double Mh[kCMax + 1];        // chunks of M / 2
    double invM[kCMax + 1];      // 2^(40 c) / M
    double P40[kCMax + 1];       // 2^(40 c)
    double Mf;                   // float(M)
    int N, C;
};

constexpr double kTwo40 = 1099511627776.0;
constexpr double kInvTwo40 = 1.0 / 1099511627776.0;

template <int C>
__device__ __forceinline__ void normalize(double (&a)[C]) {
#pragma unroll
    for (int c = 0; c < C - 1; c++) {
        const double carry = floor(a[c] * kInvTwo40);
        a[c] = fma(-carry, kTwo40, a[c]);
        a[c + 1] += carry;
    }
}

template <int C>
__device__ __forceinline__ bool is_negative(const double (&a)[C]) {   // a normalised
    return a[C - 1] < 0.0;
}

// a -= s * b (chunkwise, exact) then normalise
template <int C>
__device__ __forceinline__ void sub_scaled(double (&a)[C], const double* b, double s) {
#pragma unroll
    for (int c = 0; c < C; c++) a[c] = fma(-s, b[c], a[c]);
    normalize<C>(a);
}

// integer value of a chunk (an exact double in [0, 2^40)): the low mantissa bits of chunk + 2^52
__device__ __forceinline__ unsigned long long chunk_bits(double v) {
    return (unsigned long long)__double_as_longlong(v + 4503599627370496.0) & 0xfffffffffffffULL;
}

template <int C>
__device__ __forceinline__ double to_double_unscaled(const double (&a)[C], int scale_exp) {
    // a: normalised, non-negative; returns RN(a) * 2^scale_exp with the reference's two-step rounding
    unsigned long long h = 0, md = 0, lo = 0;
    int ct = -1;
    bool sticky = false;
#pragma unroll
    for (int c = C - 1; c >= 0; c--) {
        const unsigned long long v = chunk_bits(a[c]);
        if (ct < 0) {
            if (v != 0ULL) { ct = c; h = v; }
        } else if (c == ct - 1) md = v;
        else if (c == ct - 2) lo = v;
        else sticky |= v != 0ULL;
    }
    if (ct < 0) return 0.0;
    // value = (h 2^80 + md 2^40 + lo) 2^(40 (ct - 2)); t1 = its bits above the lowest 56 of the 120-bit window,
    // nxt = those 56 bits left-aligned; normalise t1 (>= 2^24, so 0 <= sh <= 39) and keep a sticky bit
    const unsigned long long t1 = (h << 24) | (md >> 16);
    const unsigned long long nxt = (md << 48) | (lo << 8);
    const int sh = __clzll((long long)t1);
    unsigned long long qv = t1, lost = nxt;
    if (sh) { qv = (t1 << sh) | (nxt >> (64 - sh)); lost = nxt << sh; }
    if (sticky || lost != 0ULL) qv |= 1ULL;
    const double d = __ull2double_rn(qv);
    const int e = 40 * ct - 24 - sh + scale_exp;
    // one multiplication by an exact 2^e rounds d 2^e once, exactly as ldexp does; ldexp covers the rest
    if (e >= -1022 && e <= 1023) return d * __longlong_as_double((long long)(e + 1023) << 52);
    return ldexp(d, e);
}

// chunks of 40 bits of M = m_0 ... m_{N-1} (at least 2), per N
__host__ __device__ constexpr int chunks_for(int N) {
    constexpr int c[OZK_NMAX + 1] = {2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 3, 3, 3, 3, 3, 4,
                                     4, 4, 4, 4, 5, 5, 5, 5, 5, 5, 6, 6, 6, 6, 6, 7};
    return c[N];
}

template <int N>
__global__ void __launch_bounds__(256) recon_kernel(const uint8_t* __restrict__ X, const int32_t* __restrict__ r,
                                                    const int32_t* __restrict__ cexp, const int32_t* __restrict__ p_dev,
                                                    int m, int n, const __grid_constant__ ReconParams rp,
                                                    double* __restrict__ Cout) {
    constexpr int C = chunks_for(N);
    const long long quads = (long long)m * (n >> 2);
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= quads) return;
    const int n4 = n >> 2;
    const int i = (int)(g / n4), j4 = (int)(g - (long long)i * n4);
    const size_t mn = (size_t)m * n;
    const size_t idx = (size_t)i * n + 4 * (size_t)j4;
    unsigned w[N];
#pragma unroll
    for (int t = 0; t < N; t++) w[t] = __ldg(reinterpret_cast<const unsigned*>(X + (size_t)t * mn + idx));
    double acc[4][C];
#pragma unroll
    for (int e = 0; e < 4; e++)
#pragma unroll
        for (int c = 0; c < C; c++) acc[e][c] = 0.0;
#pragma unroll
    for (int t = 0; t < N; t++) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            // exact double of the byte: 2^52 + b, minus 2^52
            const double xd = __hiloint2double(0x43300000, (int)__byte_perm(w[t], 0u, 0x4440u | (unsigned)e)) -
                              4503599627370496.0;
#pragma unroll
            for (int c = 0; c < C; c++) acc[e][c] = fma(xd, rp.V[t][c], acc[e][c]);
        }
    }
    const int p = *p_dev;
    const int base = r[i] - 2 * p;
    const int4 cc = __ldg(reinterpret_cast<const int4*>(cexp) + j4);
    const int cj[4] = {cc.x, cc.y, cc.z, cc.w};
    double outv[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        double a[C];
        double f = 0.0;
#pragma unroll
        for (int c = 0; c < C; c++) { a[c] = acc[e][c]; f = fma(a[c], rp.invM[c], f); }
        const double q = rint(f);
        sub_scaled<C>(a, rp.Mc, q);
        // X must lie in [-M/2, M/2 - 1]; outside the bound of pmax_bits only, checked exactly when close
        double approx = 0.0;
#pragma unroll
        for (int c = 0; c < C; c++) approx = fma(a[c], rp.P40[c], approx);
        if (fabs(approx) > 0.4999 * rp.Mf) {
            double tmp[C];
#pragma unroll
            for (int c = 0; c < C; c++) tmp[c] = a[c];
            sub_scaled<C>(tmp, rp.Mh, 1.0);                 // X - M/2
            if (!is_negative<C>(tmp)) sub_scaled<C>(a, rp.Mc, 1.0);
            else {
#pragma unroll
                for (int c = 0; c < C; c++) tmp[c] = a[c];
                sub_scaled<C>(tmp, rp.Mh, -1.0);            // X + M/2
                if (is_negative<C>(tmp)) sub_scaled<C>(a, rp.Mc, -1.0);
            }
        }
        // magnitude, without a divergent branch: multiply by the sign and normalise again
        const bool neg = is_negative<C>(a);
        const double sg = neg ? -1.0 : 1.0;
#pragma unroll
        for (int c = 0; c < C; c++) a[c] *= sg;
        normalize<C>(a);
        const double v = to_double_unscaled<C>(a, base + cj[e]);
        outv[e] = neg ? -v : v;
    }
    double2* dst = reinterpret_cast<double2*>(Cout + idx);
    dst[0] = make_double2(outv[0], outv[1]);
    dst[1] = make_double2(outv[2], outv[3]);
}

// ---- tensor-core chunk sums ------------------------------------------------------------------------------------
namespace tcr {

#ifndef OZK_RECON_G
#define OZK_RECON_G 4        // tiles per CTA iteration
#endif
#ifndef OZK_RECON_LOCKSTEP
#define OZK_RECON_LOCKSTEP 2 // entries finished together (their dependency chains interleave)
#endif
#ifndef OZK_RECON_CTAS
#define OZK_RECON_CTAS 4     // CTAs per SM (shared memory is sized so that no more fit, TMEM then always does)
#endif
constexpr int THREADS = 128;                 // 4 warps; warp w reads TMEM lanes [32 w, 32 w + 32)
constexpr int BM = 128;                      // entries per tile = MMA M = TMEM lanes
constexpr int G = OZK_RECON_G;               // tiles per CTA iteration: each thread finishes G independent entries
constexpr int CTAS = OZK_RECON_CTAS;
constexpr int KP = 32;                       // planes per MMA (K); planes >= N arrive as zeros
constexpr int NC = 32;                       // byte columns of the CRT weights (MMA N)
constexpr uint32_t TILE_BYTES = BM * KP;     // one tile of X: 32 rows (planes) of 128 bytes (entries)
constexpr uint32_t STAGE_BYTES = G * TILE_BYTES;
constexpr uint32_t B_BYTES = NC * 128;       // the weight bytes, K-major rows padded to 128 bytes
constexpr int STAGES = 2;
constexpr uint32_t TMEM_COLS = G * NC;       // G accumulators of 32 columns, read out before the next MMAs
constexpr uint32_t IDESC = umma_idesc_u8_amn(BM, NC);
constexpr uint64_t WAIT_LIMIT_NS = 4000000000ull;
// shared memory per CTA such that at most CTAS fit on an SM (228 KB), so their TMEM (CTAS x G x 32 columns) fits
constexpr size_t SMEM_BYTES = ((228 * 1024) / (CTAS + 1) + 1024) & ~(size_t)1023;
constexpr int NUM_BARS = STAGES + 2;         // full[STAGES], mma, drain
constexpr int kLimbsMax = 9;                 // 32-bit limbs of the CRT sum S < 8160 M for N <= 32
static_assert(1024 + STAGES * STAGE_BYTES + B_BYTES + NUM_BARS * 8 + 16 <= SMEM_BYTES, "shared memory layout");
static_assert(CTAS * (SMEM_BYTES + 1024) <= 228 * 1024 && (CTAS + 1) * SMEM_BYTES > 228 * 1024 &&
                  CTAS * TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0 && G % OZK_RECON_LOCKSTEP == 0,
              "at most CTAS CTAs per SM, and their TMEM fits");

struct alignas(16) Params {
    uint8_t vb[NC][KP];                      // vb[b][t] = byte b of V_t for t < N, else 0
    uint32_t ML[kLimbsMax];                  // 32-bit limbs of M
    uint32_t NM[kLimbsMax];                  // limbs of 2^(32 LIMBS) - M (two's complement of M)
    uint32_t MH[kLimbsMax];                  // limbs of M / 2 (M is even)
    double K3[3];                            // 2^(32 (LIMBS - 3 + j)) / M: S / M from the top three limbs of S
    unsigned long long ndiv;                 // floor(2^64 / n) + 1: row = high 64 bits of e * ndiv (e < 2^32)
    int n;
};

__device__ __forceinline__ void raise_abort(volatile int* abort_flag, int32_t* err) {
    *abort_flag = 1;
    atomicOr(err, OZK_DEVERR_TIMEOUT_RECON);
}

// exact double of a 32-bit unsigned integer without a conversion instruction: 2^52 + v, minus 2^52
__device__ __forceinline__ double u32_to_f64(uint32_t v) {
    return __hiloint2double(0x43300000, (int)v) - 4503599627370496.0;
}

// Y = S - M, S + M or the comparison sign of S - M/2, on LIMBS limbs (two's complement); rarely used
template <int LIMBS>
__device__ __forceinline__ void limbs_add(uint32_t (&y)[LIMBS], const uint32_t* b, bool subtract) {
    unsigned long long acc = subtract ? 1ULL : 0ULL;
#pragma unroll
    for (int w = 0; w < LIMBS; w++) {
        acc += (unsigned long long)y[w] + (subtract ? (uint32_t)~b[w] : b[w]);
        y[w] = (uint32_t)acc;
        acc >>= 32;
    }
}

}  // namespace tcr

// The exact end of the CRT for one entry, from its byte sums T[b] = sum_t x_t byte_b(V_t) (b < NL):
//   S = sum_b T_b 2^(8b) on LIMBS 32-bit limbs (integer multiply-adds; S < 8160 M);
//   q = rint(S / M) from the top three limbs in FP64 (error ~1e-11, far below the distance of S / M from a
//   half-integer within the plane count's bound; outside it, |S / M - q| > 0.4999 triggers an exact correction);
//   Y = S - q M = S + q (2^(32 LIMBS) - M) modulo 2^(32 LIMBS), in [-M/2, M/2 - 1];
//   |Y| rounded to 53 bits (round to nearest even over its leading 64 bits plus a sticky bit), times 2^scale_exp,
//   with the sign of Y -- exactly the reference's result (ldexp of the rounded integer, so the subnormal range
//   rounds twice as there).  Integer and FP64 arithmetic only: no conversion instructions on the slow XU pipe
//   except one count of leading zeros.
template <int NL, int LIMBS>
__device__ __forceinline__ double crt_finish(const uint32_t (&T)[NL], int scale_exp, const tcr::Params& rp) {
    uint32_t S[LIMBS];
    uint32_t cy = 0u;
#pragma unroll
    for (int w = 0; w < LIMBS; w++) {
        const uint32_t t0 = 4 * w < NL ? T[4 * w] : 0u, t1 = 4 * w + 1 < NL ? T[4 * w + 1] : 0u;
        const uint32_t t2 = 4 * w + 2 < NL ? T[4 * w + 2] : 0u, t3 = 4 * w + 3 < NL ? T[4 * w + 3] : 0u;
        const uint32_t x = t1 * 256u + t0 + cy;                   // < 2^30
        const uint32_t y = t3 * 256u + t2;                        // < 2^30
        const unsigned long long acc = (unsigned long long)y * 65536ull + x;
        S[w] = (uint32_t)acc;
        cy = (uint32_t)(acc >> 32);
    }
    double f = 0.0;
#pragma unroll
    for (int j = 0; j < 3; j++) f = fma(tcr::u32_to_f64(S[LIMBS - 3 + j]), rp.K3[j], f);
    const double fq = f + 6755399441055744.0;                     // 1.5 2^52: the low mantissa bits hold rint(f)
    const uint32_t q = (uint32_t)__double2loint(fq);
    uint32_t Y[LIMBS];
    {
        unsigned long long acc = 0ULL;
#pragma unroll
        for (int w = 0; w < LIMBS; w++) {
            acc += (unsigned long long)q * rp.NM[w] + S[w];
            Y[w] = (uint32_t)acc;
            acc >>= 32;
        }
    }
    if (fabs(f - (fq - 6755399441055744.0)) > 0.4999) {
        // |Y| is close to M/2: place it in [-M/2, M/2 - 1] exactly (only for data outside the plane count's bound)
        uint32_t t[LIMBS];
#pragma unroll
        for (int w = 0; w < LIMBS; w++) t[w] = Y[w];
        tcr::limbs_add<LIMBS>(t, rp.MH, true);                    // Y - M/2
        if ((int)t[LIMBS - 1] >= 0) tcr::limbs_add<LIMBS>(Y, rp.ML, true);
        else {
#pragma unroll
            for (int w = 0; w < LIMBS; w++) t[w] = Y[w];
            tcr::limbs_add<LIMBS>(t, rp.MH, false);               // Y + M/2
            if ((int)t[LIMBS - 1] < 0) tcr::limbs_add<LIMBS>(Y, rp.ML, false);
        }
    }
    // sign and magnitude
    const uint32_t mask = (uint32_t)((int)Y[LIMBS - 1] >> 31);
    {
        unsigned long long acc = mask & 1u;
#pragma unroll
        for (int w = 0; w < LIMBS; w++) {
            acc += Y[w] ^ mask;
            Y[w] = (uint32_t)acc;
            acc >>= 32;
        }
    }
    // the leading limb k and the two below it; sticky = any bit further down
    uint32_t w0 = 0u, w1 = 0u, w2 = 0u, below = 0u, prefix = 0u;
    int k = -1;
#pragma unroll
    for (int w = 0; w < LIMBS; w++) {
        const bool nz = Y[w] != 0u;
        w0 = nz ? Y[w] : w0;
        w1 = nz ? (w >= 1 ? Y[w - 1] : 0u) : w1;
        w2 = nz ? (w >= 2 ? Y[w - 2] : 0u) : w2;
        below = nz ? prefix : below;                              // OR of limbs 0 .. w - 3
        k = nz ? w : k;
        if (w >= 2) prefix |= Y[w - 2];
    }
    if (k < 0) return 0.0;                                        // Y = 0
    const int sh = __clz((int)w0);
    const uint32_t hi = __funnelshift_l(w1, w0, sh), lo = __funnelshift_l(w2, w1, sh);
    const bool sticky = ((w2 << sh) | below) != 0u;
    // round the 64-bit window hi:lo (bit 63 set) to 53 bits, nearest even
    const uint32_t guard = (lo >> 10) & 1u, low10 = lo & 0x3FFu;
    const uint32_t mlo = (lo >> 11) | (hi << 21), mhi = hi >> 11;
    const uint32_t up = guard & (uint32_t)((low10 != 0u) | sticky | (mlo & 1u));
    const unsigned long long mant = (((unsigned long long)mhi << 32) | mlo) + up;   // in [2^52, 2^53]
    // |Y| = mant 2^(32 k - 21 - sh) (before rounding: the window's bit 63 is bit 32 k + 31 - sh of |Y|)
    const int e2 = 32 * k - 21 - sh;
    const int biased = e2 + scale_exp + 52 + 1023;                // exponent field of the result (mant < 2^53)
    unsigned long long bits;
    if (biased >= 1 && biased + (int)(mant >> 53) <= 2046) {
        bits = ((unsigned long long)biased << 52) + mant - (1ULL << 52);   // mant = 2^53 carries into the exponent
    } else {
        // subnormal or overflowing result: round the integer first, then scale (the reference's ldexp)
        const double d = __longlong_as_double((long long)(((unsigned long long)(52 + 1023) << 52) + mant - (1ULL << 52)));
        bits = (unsigned long long)__double_as_longlong(ldexp(d, e2 + scale_exp));
    }
    return __longlong_as_double((long long)(bits | ((unsigned long long)(mask & 1u) << 63)));
}

// The same result for N <= 20 (|Y| < 2^155) with the rounding done in FP64, two entries at a time (their chains
// interleave).  Differences from crt_finish:
//   S is kept as LIMBS partial sums R_w = sum_{j<4} T_{4w+j} 2^(8j) < 2^46 (S = sum_w R_w 2^(32w), no carries yet);
//   q = rint(S / M) comes from the top three R_w (exact doubles) times 2^(32w) / M -- the lower ones contribute
//   less than 2^-60 of M -- so Y = S + q (2^(32 LIMBS) - M) is one carry chain of multiply-adds;
//   |Y| is cut into three 52-bit chunks c0, c1, c2, converted exactly (c1 2^52 and c2 2^104 by the exponent of the
//   2^52 + c bit pattern); s = RN(c2 2^104 + c1 2^52) and its exact error e come from Fast2Sum (|c2 2^104| >= the
//   other term, or c2 = 0); e is a multiple of 2^52 and c0 < 2^52, so RN(|Y|) = RN(s + c0) when e = 0, the next
//   double above s when e is exactly half its spacing and c0 > 0, and s otherwise (the first rounding already broke
//   the tie to even, or |e + c0| stays below half a spacing -- also at a power of two, where the spacing below s
//   is half the one above);
//   the scaling adds to the exponent field when the result stays normal (ldexp otherwise, as the reference).
template <int G, int LIMBS>
__device__ __forceinline__ void crt_finish_fp(const unsigned long long (*R)[LIMBS], const int* scale_exp,
                                              const tcr::Params& rp, double* out) {
    // R[g][w] = sum_{j<4} T_{4w+j} 2^(8j): the limb-w contribution to S before carries (< 2^46); S = sum R_w 2^(32w)
    double f[G];
    uint32_t Q[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        double acc = 0.0;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const unsigned long long v = R[g][LIMBS - 3 + j];         // exact double of v < 2^52 by its bit pattern
            const double dv = __hiloint2double((int)(0x43300000u | (uint32_t)(v >> 32)), (int)(uint32_t)v) - 0x1p52;
            acc = fma(dv, rp.K3[j], acc);
        }
        f[g] = acc;
        Q[g] = (uint32_t)__double2loint(acc + 6755399441055744.0);
    }
    uint32_t Y[G][LIMBS];
#pragma unroll
    for (int g = 0; g < G; g++) {
        unsigned long long cy = 0ull;
#pragma unroll
        for (int w = 0; w < LIMBS; w++) {
            const unsigned long long acc = (unsigned long long)Q[g] * rp.NM[w] + R[g][w] + cy;
            Y[g][w] = (uint32_t)acc;
            cy = acc >> 32;
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        const double fr = f[g] - (__longlong_as_double(__double_as_longlong(f[g] + 6755399441055744.0)) -
                                  6755399441055744.0);
        if (fabs(fr) > 0.4999) {
            // |Y| is close to M/2: place it in [-M/2, M/2 - 1] exactly (data outside the plane count's bound)
            uint32_t t[LIMBS];
#pragma unroll
            for (int w = 0; w < LIMBS; w++) t[w] = Y[g][w];
            tcr::limbs_add<LIMBS>(t, rp.MH, true);
            if ((int)t[LIMBS - 1] >= 0) tcr::limbs_add<LIMBS>(Y[g], rp.ML, true);
            else {
#pragma unroll
                for (int w = 0; w < LIMBS; w++) t[w] = Y[g][w];
                tcr::limbs_add<LIMBS>(t, rp.MH, false);
                if ((int)t[LIMBS - 1] < 0) tcr::limbs_add<LIMBS>(Y[g], rp.ML, false);
            }
        }
    }
    uint32_t sign[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const uint32_t mask = (uint32_t)((int)Y[g][LIMBS - 1] >> 31);
        sign[g] = mask & 0x80000000u;
        unsigned long long acc = mask & 1u;
#pragma unroll
        for (int w = 0; w < LIMBS; w++) {
            acc += Y[g][w] ^ mask;
            Y[g][w] = (uint32_t)acc;
            acc >>= 32;
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        const uint32_t y0 = Y[g][0], y1 = LIMBS > 1 ? Y[g][1] : 0u, y2 = LIMBS > 2 ? Y[g][2] : 0u;
        const uint32_t y3 = LIMBS > 3 ? Y[g][3] : 0u, y4 = LIMBS > 4 ? Y[g][4] : 0u;
        // chunks of 52 bits, each as the exact double (2^52 + c) 2^(52 j) minus 2^52 2^(52 j)
        const double d0 = __hiloint2double((int)(0x43300000u | (y1 & 0xFFFFFu)), (int)y0) - 0x1p52;
        const double d1 = __hiloint2double((int)(0x46700000u | (__funnelshift_r(y2, y3, 20) & 0xFFFFFu)),
                                           (int)__funnelshift_r(y1, y2, 20)) - 0x1p104;
        const double d2 = __hiloint2double((int)(0x49B00000u | (y4 >> 8)), (int)__funnelshift_r(y3, y4, 8)) - 0x1p156;
        const double sm = d2 + d1;
        const double e = d1 - (sm - d2);
        const double near = sm + d0;
        const double up = __longlong_as_double(__double_as_longlong(sm) + 1);
        const bool tie_up = e == 0.5 * (up - sm) && d0 > 0.0;
        const double rnd = e == 0.0 ? near : (tie_up ? up : sm);
        // times 2^scale_exp with the sign of Y
        const int ebits = (int)((unsigned long long)__double_as_longlong(rnd) >> 52);
        const int fin = ebits + scale_exp[g];
        double v;
        if (ebits != 0 && fin >= 1 && fin <= 2046)
            v = __longlong_as_double(__double_as_longlong(rnd) + ((long long)scale_exp[g] << 52));
        else
            v = ldexp(rnd, scale_exp[g]);
        out[g] = __longlong_as_double(__double_as_longlong(v) | ((long long)sign[g] << 32));
    }
}

// One iteration of a CTA covers G consecutive tiles of 128 entries (a "group"); thread t finishes entries
// group * 128 G + 128 g + t, g < G.
// FP: the FP64 rounding of crt_finish_fp (|Y| < 2^156, N <= 20); else crt_finish's integer rounding.
template <int NL, int LIMBS, bool FP>
__global__ void __launch_bounds__(tcr::THREADS, tcr::CTAS)
    recon_tc_kernel(const __grid_constant__ CUtensorMap tmX, const int32_t* __restrict__ r,
                    const int32_t* __restrict__ cexp, const int32_t* __restrict__ p_dev, unsigned e_begin, int E,
                    int ngroups, const __grid_constant__ tcr::Params rp, double* __restrict__ Cout,
                    int32_t* __restrict__ err) {
    using namespace tcr;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + B_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t bar0 = smem_addr(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * (uint32_t)s; };
    const uint32_t mma_bar = bar0 + 8u * STAGES, drain_bar = bar0 + 8u * (STAGES + 1);

    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) mbar_init(full_bar(s), 1);
        mbar_init(mma_bar, 1);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        mbar_fence_init();
        tma_prefetch_desc(&tmX);
    }
    if (warp == 0) {
        tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    {
        // the weight bytes as the K-major B operand with the 128-byte swizzle: logical 16-byte chunk q of row b is
        // stored at chunk q ^ (b & 7); only chunks 0 and 1 (planes 0..31) are non-zero
        const int b = tid >> 2;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int pc = 2 * (tid & 3) + h;
            const int lc = pc ^ (b & 7);
            uint32_t w[4] = {0u, 0u, 0u, 0u};
            if (lc < 2) {
                const uint32_t* src = reinterpret_cast<const uint32_t*>(&rp.vb[b][16 * lc]);   // 4-byte aligned
#pragma unroll
                for (int q = 0; q < 4; q++) w[q] = src[q];
            }
            *reinterpret_cast<uint4*>(sB + b * 128 + pc * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_proxy_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int p = *p_dev;
    const uint64_t bdesc = umma_desc_sw128(smem_addr(sB));

    // thread 0 drives the pipeline: loads two groups ahead, issues the next group's G MMAs as soon as the current
    // group has been read out of TMEM.  Its bookkeeping lets it drain what is in flight if a wait runs out.
    int loads_issued[STAGES] = {0, 0}, loads_done[STAGES] = {0, 0};
    bool mma_in_flight = false;
    auto issue_load = [&](int group, int s) {
        // tiles past the end of X are not loaded (their entries are not stored; E is a multiple of 128)
        const int count = min(G, E / BM - group * G);
        mbar_arrive_expect_tx(full_bar(s), (uint32_t)count * TILE_BYTES);
        for (int g = 0; g < count; g++)
            tma_load_2d(smem_addr(sA + s * STAGE_BYTES + g * TILE_BYTES), &tmX, (group * G + g) * BM, 0, full_bar(s));
        loads_issued[s]++;
    };
    auto issue_mma = [&](int s) -> bool {   // waits for stage s, then one MMA per tile of the group
        if (!mbar_wait_bounded(full_bar(s), (uint32_t)(loads_done[s] & 1), abort_flag, WAIT_LIMIT_NS)) {
            if (!*abort_flag) raise_abort(abort_flag, err);
            return false;
        }
        loads_done[s]++;
        tc_fence_after();
#pragma unroll
        for (int g = 0; g < G; g++)
            umma_i8(tmem_base + (uint32_t)(g * NC), umma_desc_sw128_mn(smem_addr(sA + s * STAGE_BYTES + g * TILE_BYTES), 0u),
                    bdesc, IDESC, 0u);
        umma_commit(mma_bar);
        mma_in_flight = true;
        return true;
    };
    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            const int group = blockIdx.x + s * gridDim.x;
            if (group < ngroups) issue_load(group, s);
        }
        if (blockIdx.x < ngroups) issue_mma(0);
    }

    int it = 0;
    for (int group = blockIdx.x; group < ngroups; group += gridDim.x, it++) {
        const int s = it & 1;
        // this thread's entries and their scalings, loaded before the wait: entry e + 128 g lies in the row of entry
        // e or in a later one (one division for the group, then steps of 128 columns)
        int el[G], ex[G];
        {
            const unsigned e0 = e_begin + (unsigned)((group * G) * BM + tid);
            unsigned row = (unsigned)__umul64hi((unsigned long long)e0, rp.ndiv);
            unsigned col = e0 - row * (unsigned)rp.n;
            const unsigned nrow = (unsigned)rp.n;
#pragma unroll
            for (int g = 0; g < G; g++) {
                el[g] = (group * G + g) * BM + tid;
                if (g > 0) {
                    col += BM;
                    while (col >= nrow) { col -= nrow; row++; }      // once at most when n >= 128
                }
                const bool in = el[g] < E;
                ex[g] = __ldg(r + (in ? row : 0u)) - 2 * p + __ldg(cexp + (in ? col : 0u));
            }
        }
        // the group's byte sums: wait for its MMAs, read this thread's rows of TMEM
        bool ok = mbar_wait_bounded(mma_bar, (uint32_t)(it & 1), abort_flag, WAIT_LIMIT_NS);
        if (!ok && !*abort_flag) raise_abort(abort_flag, err);
        ok = __all_sync(0xffffffffu, ok);
        constexpr bool kFp = FP;                                  // N <= 20: FP64 rounding on byte pairs
        uint32_t T[kFp ? 1 : G][NL];
        unsigned long long Rl[kFp ? G : 1][LIMBS];
        if (ok) {
            tc_fence_after();
            const uint32_t lanes = tmem_base + ((uint32_t)(warp * 32) << 16);
#pragma unroll
            for (int g = 0; g < G; g++) {
                const uint32_t taddr = lanes + (uint32_t)(g * NC);
                uint32_t* dst = T[kFp ? 0 : g];
                tmem_ld_32x32b_x16(taddr, dst);
                if (NL >= 24) tmem_ld_32x32b_x8(taddr + 16u, dst + 16);
                if (NL == 32) tmem_ld_32x32b_x8(taddr + 24u, dst + 24);
                if constexpr (kFp) {
                    tmem_wait_ld();
#pragma unroll
                    for (int w = 0; w < LIMBS; w++) {
                        const uint32_t t0 = 4 * w < NL ? dst[4 * w] : 0u, t1 = 4 * w + 1 < NL ? dst[4 * w + 1] : 0u;
                        const uint32_t t2 = 4 * w + 2 < NL ? dst[4 * w + 2] : 0u;
                        const uint32_t t3 = 4 * w + 3 < NL ? dst[4 * w + 3] : 0u;
                        Rl[g][w] = (unsigned long long)(t3 * 256u + t2) * 65536ull + (t1 * 256u + t0);
                    }
                }
            }
            tmem_wait_ld();
        }
        tc_fence_before();
        if (!__syncthreads_and(ok ? 1 : 0)) break;
        if (tid == 0) {
            mma_in_flight = false;
            // stage s and TMEM are free: the load two groups ahead, then the next group's MMAs
            const int ahead = group + STAGES * (int)gridDim.x;
            if (ahead < ngroups) issue_load(ahead, s);
            if (group + (int)gridDim.x < ngroups) issue_mma(s ^ 1);
        }
        double v[G];
        if constexpr (kFp) {
#pragma unroll
            for (int g = 0; g < G; g += OZK_RECON_LOCKSTEP) crt_finish_fp<OZK_RECON_LOCKSTEP, LIMBS>(Rl + g, ex + g, rp, v + g);
        } else {
#pragma unroll
            for (int g = 0; g < G; g++) v[g] = crt_finish<NL, LIMBS>(T[g], ex[g], rp);
        }
#pragma unroll
        for (int g = 0; g < G; g++)
            if (el[g] < E) Cout[el[g]] = v[g];
    }

    // leave only when nothing of this CTA is in flight (only a wait that ran out can leave loads or MMAs behind)
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        int dummy = 0;
        if (mma_in_flight) {
            umma_commit(drain_bar);
            mbar_wait_bounded(drain_bar, 0u, &dummy, WAIT_LIMIT_NS);
        }
        for (int s = 0; s < STAGES; s++)
            for (; loads_done[s] < loads_issued[s]; loads_done[s]++)
                mbar_wait_bounded(full_bar(s), (uint32_t)(loads_done[s] & 1), &dummy, WAIT_LIMIT_NS);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        __syncwarp();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---- host: exact parameters per N (small multi-precision integers, 32-bit limbs) ---------------------------------
struct Big {
    uint32_t w[10];
};
void big_set(Big& a, uint32_t v) { memset(a.w, 0, sizeof(a.w)); a.w[0] = v; }
void big_mul_small(Big& a, uint32_t s) {
    uint64_t carry = 0;
    for (int q = 0; q < 10; q++) { const uint64_t v = (uint64_t)a.w[q] * s + carry; a.w[q] = (uint32_t)v; carry = v >> 32; }
}
uint32_t big_divmod_small(Big& a, uint32_t s) {   // a /= s, returns remainder
    uint64_t rem = 0;
    for (int q = 9; q >= 0; q--) { const uint64_t v = (rem << 32) | a.w[q]; a.w[q] = (uint32_t)(v / s); rem = v % s; }
    return (uint32_t)rem;
}
uint32_t big_mod_small(const Big& a, uint32_t s) {
    Big t = a;
    return big_divmod_small(t, s);
}
int big_cmp(const Big& a, const Big& b) {
    for (int q = 9; q >= 0; q--) if (a.w[q] != b.w[q]) return a.w[q] < b.w[q] ? -1 : 1;
    return 0;
}
void big_sub(Big& a, const Big& b) {
    int64_t borrow = 0;
    for (int q = 0; q < 10; q++) {
        const int64_t v = (int64_t)a.w[q] - (int64_t)b.w[q] - borrow;
        a.w[q] = (uint32_t)v;
        borrow = v < 0;
    }
}
int big_bits(const Big& a) {
    for (int q = 9; q >= 0; q--) if (a.w[q]) return 32 * q + 32 - __builtin_clz(a.w[q]);
    return 0;
}
double big_chunk40(const Big& a, int c) {   // bits [40c, 40c + 40)
    uint64_t v = 0;
    for (int b = 0; b < 40; b++) {
        const int bit = 40 * c + b;
        if (bit < 320 && ((a.w[bit >> 5] >> (bit & 31)) & 1u)) v |= 1ULL << b;
    }
    return (double)v;
}
uint32_t inv_mod(uint32_t a, uint32_t P) {
    int64_t t0 = 0, t1 = 1, r0 = P, r1 = a % P;
    while (r1) { const int64_t q = r0 / r1; int64_t tmp = r0 - q * r1; r0 = r1; r1 = tmp; tmp = t0 - q * t1; t0 = t1; t1 = tmp; }
    return (uint32_t)(t0 < 0 ? t0 + P : t0);
}

uint8_t g_vbytes[OZK_NMAX + 1][tcr::NC][tcr::KP];   // per N: byte b of V_t at [N][b][t]
struct LimbTable {                                   // per N: the limb constants of the tensor-core path
    int limbs;                                       // 32-bit limbs of S < 8160 M (at least 3)
    int nl;                                          // byte columns read from TMEM: 16, 24 or 32
    int mbits;                                       // bits of M
    uint32_t ML[tcr::kLimbsMax], NM[tcr::kLimbsMax], MH[tcr::kLimbsMax];
};
LimbTable g_limbs[OZK_NMAX + 1];

ReconParams make_params(int N) {
    ReconParams rp;
    memset(&rp, 0, sizeof(rp));
    memset(g_vbytes[N], 0, sizeof(g_vbytes[N]));
    rp.N = N;
    Big M;
    big_set(M, 1);
    for (int t = 0; t < N; t++) big_mul_small(M, (uint32_t)ozk_mod(t));
    rp.C = (big_bits(M) + 39) / 40;
    for (int t = 0; t < N; t++) {
        const uint32_t P = (uint32_t)ozk_mod(t);
        Big W = M;
        big_divmod_small(W, P);
        const uint32_t y = inv_mod(big_mod_small(W, P), P);
        Big V = W;
        big_mul_small(V, y);
        while (big_cmp(V, M) >= 0) big_sub(V, M);
        for (int c = 0; c < kCMax; c++) rp.V[t][c] = big_chunk40(V, c);
        for (int b = 0; b < tcr::NC; b++) g_vbytes[N][b][t] = (uint8_t)(V.w[b >> 2] >> (8 * (b & 3)));
    }
    Big Mh = M;
    big_divmod_small(Mh, 2);
    {
        LimbTable& L = g_limbs[N];
        memset(&L, 0, sizeof(L));
        Big S = M;
        big_mul_small(S, 8160u);                     // bound of S = sum_t x_t V_t
        L.limbs = (big_bits(S) + 31) / 32;
        if (L.limbs < 3) L.limbs = 3;
        L.mbits = big_bits(M);
        const int nb = (L.mbits + 7) / 8;
        L.nl = nb <= 16 ? 16 : (nb <= 24 ? 24 : 32);
        uint64_t borrow = 1;                         // 2^(32 limbs) - M = ~M + 1 on `limbs` limbs
        for (int w = 0; w < L.limbs; w++) {
            L.ML[w] = M.w[w];
            L.MH[w] = Mh.w[w];
            const uint64_t v = (uint64_t)(uint32_t)~M.w[w] + borrow;
            L.NM[w] = (uint32_t)v;
            borrow = v >> 32;
        }
    }
    rp.Mf = ozk_modulus_product(N);
    for (int c = 0; c <= kCMax; c++) {
        rp.Mc[c] = big_chunk40(M, c);
        rp.Mh[c] = big_chunk40(Mh, c);
        rp.invM[c] = ldexp(1.0, 40 * c) / rp.Mf;
        rp.P40[c] = ldexp(1.0, 40 * c);
    }
    return rp;
}

const ReconParams& params_for(int N) {
    static ReconParams table[OZK_NMAX + 1];
    static bool init = false;
    if (!init) {
        for (int q = 1; q <= OZK_NMAX; q++) table[q] = make_params(q);
        init = true;
    }
    return table[N];
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

struct TcDevice { int sms = 0; bool attr[128] = {}; };
TcDevice g_tc_dev[64];

template <int NL, int LIMBS, bool FP>
int launch_tc(const uint8_t* X, const int32_t* r, const int32_t* c, const int32_t* p_dev, int m, int n, int N,
              double* Cout, int32_t* err, cudaStream_t st) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OZK_ERR_DEVICE;
    TcDevice& d = g_tc_dev[dev];
    if (d.sms == 0 && cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return OZK_ERR_DEVICE;
    const int slot = (NL / 8 * 16 + LIMBS) * 2 + (FP ? 1 : 0);   // distinct per instantiation, < 128
    if (!d.attr[slot]) {
        if (cudaFuncSetAttribute(recon_tc_kernel<NL, LIMBS, FP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)tcr::SMEM_BYTES) != cudaSuccess)
            return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
        d.attr[slot] = true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) return OZK_ERR_DRIVER;
    static tcr::Params tp[OZK_NMAX + 1];
    static bool tp_init[OZK_NMAX + 1] = {};
    if (!tp_init[N] || tp[N].n != n) {
        const ReconParams& rp = params_for(N);
        const LimbTable& L = g_limbs[N];
        tcr::Params& q = tp[N];
        memset(&q, 0, sizeof(q));
        memcpy(q.vb, g_vbytes[N], sizeof(q.vb));
        memcpy(q.ML, L.ML, sizeof(q.ML));
        memcpy(q.NM, L.NM, sizeof(q.NM));
        memcpy(q.MH, L.MH, sizeof(q.MH));
        for (int j = 0; j < 3; j++) q.K3[j] = ldexp(1.0, 32 * (L.limbs - 3 + j)) / rp.Mf;
        q.n = n;
        q.ndiv = ~0ULL / (unsigned long long)n + 1ULL;
        tp_init[N] = true;
    }
    const unsigned long long E = (unsigned long long)m * (unsigned long long)n;
    // launches of at most 2^30 entries (32-bit TMA coordinates, int tile counts); X as a 2-D map {entries, planes
    // (stride E bytes)}, box {128, 32}: one tile of 32 planes, planes >= N and entries past the end zero-filled
    const unsigned long long chunk = 1ULL << 30;
    for (unsigned long long e0 = 0; e0 < E; e0 += chunk) {
        const unsigned long long len = E - e0 < chunk ? E - e0 : chunk;
        const unsigned long long tiles = len / tcr::BM;
        CUtensorMap map;
        const cuuint64_t dims[2] = {(cuuint64_t)len, (cuuint64_t)N};
        const cuuint64_t strides[1] = {(cuuint64_t)E};
        const cuuint32_t box[2] = {(cuuint32_t)tcr::BM, (cuuint32_t)tcr::KP};
        const cuuint32_t estr[2] = {1u, 1u};
        if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(X + e0), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return OZK_ERR_DRIVER;
        const int ngroups = (int)((tiles + tcr::G - 1) / tcr::G);
        const int grid = ngroups < tcr::CTAS * d.sms ? ngroups : tcr::CTAS * d.sms;
        recon_tc_kernel<NL, LIMBS, FP><<<grid, tcr::THREADS, tcr::SMEM_BYTES, st>>>(
            map, r, c, p_dev, (unsigned)e0, (int)len, ngroups, tp[N], Cout + e0, err);
        OZK_CHECK_LAUNCH();
    }
    return OZK_OK;
}

}  // namespace

extern "C" int ozk_reconstruct(const uint8_t* X, const int32_t* r, const int32_t* c, const int32_t* p_dev, int m,
                               int n, int N, double* C, int32_t* err, ozk_stream_t stream_) {
    if (!X || !r || !c || !p_dev || !C || !err) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || (n & 3) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(c)) & 3) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(C) & 15) || (reinterpret_cast<uintptr_t>(c) & 15)) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    const unsigned long long E = (unsigned long long)m * (unsigned long long)n;
    if (E < (1ULL << 32) && E % tcr::BM == 0 && (reinterpret_cast<uintptr_t>(X) & 15) == 0) {
        params_for(N);                               // builds the limb tables on first use
        const LimbTable& L = g_limbs[N];
        // the FP64 rounding needs |Y| <= M/2 < 2^156 (three 52-bit chunks): N <= 20
        const int fp = L.mbits <= 157 ? 1 : 0;
        switch ((L.nl * 16 + L.limbs) * 2 + fp) {
#define OZK_TC(NL_, LI_, FP_) \
    case (NL_ * 16 + LI_) * 2 + FP_: return launch_tc<NL_, LI_, FP_ != 0>(X, r, c, p_dev, m, n, N, C, err, st);
            OZK_TC(16, 3, 1) OZK_TC(16, 4, 1) OZK_TC(16, 5, 1) OZK_TC(24, 5, 1) OZK_TC(24, 6, 1) OZK_TC(24, 6, 0)
            OZK_TC(24, 7, 0) OZK_TC(32, 7, 0) OZK_TC(32, 8, 0)
#undef OZK_TC
            default: return OZK_ERR_ARG;
        }
    }
    const ReconParams& rp = params_for(N);
    const long long quads = (long long)m * (n >> 2);
    const long long blocks = (quads + 255) / 256;
    if (blocks > 0x7fffffffLL) return OZK_ERR_ARG;
    switch (N) {
#define OZK_RC(NN) case NN: recon_kernel<NN><<<(unsigned)blocks, 256, 0, st>>>(X, r, c, p_dev, m, n, rp, C); break;
        OZK_RC(1) OZK_RC(2) OZK_RC(3) OZK_RC(4) OZK_RC(5) OZK_RC(6) OZK_RC(7) OZK_RC(8)
        OZK_RC(9) OZK_RC(10) OZK_RC(11) OZK_RC(12) OZK_RC(13) OZK_RC(14) OZK_RC(15) OZK_RC(16)
        OZK_RC(17) OZK_RC(18) OZK_RC(19) OZK_RC(20) OZK_RC(21) OZK_RC(22) OZK_RC(23) OZK_RC(24)
        OZK_RC(25) OZK_RC(26) OZK_RC(27) OZK_RC(28) OZK_RC(29) OZK_RC(30) OZK_RC(31) OZK_RC(32)
#undef OZK_RC
        default: return OZK_ERR_ARG;
    }
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
