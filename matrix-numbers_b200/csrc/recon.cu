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
#include "ozk_common.cuh"

#include <string.h>

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

ReconParams make_params(int N) {
    ReconParams rp;
    memset(&rp, 0, sizeof(rp));
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
    }
    Big Mh = M;
    big_divmod_small(Mh, 2);
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

}  // namespace

extern "C" int ozk_reconstruct(const uint8_t* X, const int32_t* r, const int32_t* c, const int32_t* p_dev, int m,
                               int n, int N, double* C, ozk_stream_t stream_) {
    if (!X || !r || !c || !p_dev || !C) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || (n & 3) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(c)) & 3) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(C) & 15) || (reinterpret_cast<uintptr_t>(c) & 15)) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
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
