// Stage 3a: residue split.  FP64 A and B are read once (16-byte and 8-byte coalesced loads) and all N symmetric
// INT8 residue planes are written in the same pass, both K-major (the operand layout of the tcgen05 GEMM).
//
// Semantics (the reference's decomp / resid / resA_k / resB_k, code/ozaki_engine.py:971-1038):
//   x = round(|v| 2^ag) (exact when the shift is to the left, round half away from zero otherwise),
//   X = sign(v) x, residue = X mod m_t mapped to the symmetric range [-floor(m_t/2), ceil(m_t/2) - 1] as int8,
//   with ag = p - r_i + gamma_l for A and ag = p - c_j - gamma_l for B.
//
// Method (this build's own): X < 2^(p+1) is cut into 10-bit digits d_q (at most 16 for p <= 159), computed with
// exact FP64 operations (make_digits).  For each modulus,
// s = sum_q d_q (2^(10q) mod m_t) is an integer below 2^22, so the sum, the quotient rint(s / m_t) and the
// remainder s - m_t rint(s / m_t) are all exact in FP32 (the quotient is exact because s / m_t, m_t odd, stays at
// least 1/(2 m_t) away from a half-integer while fl(1/m_t) errs by less than that over |s| < 2^22; m_t = 256 is
// exact).  The remainder is already the symmetric residue; its low byte is read from the float's bits after adding
// 1.5 * 2^23.  The sign is folded into the digits.  This replaces the reference's integer % chains (mod53, table
// products) with FP32 fused multiply-adds.
#include "ozk_common.cuh"

namespace {

struct SplitTables {
    float P[OZK_NMAX];          // m_t
    float inv[OZK_NMAX];        // fl(1 / m_t)
    float W[OZK_NMAX][16];      // 2^(10 q) mod m_t
};

constexpr SplitTables make_split_tables() {
    SplitTables t{};
    for (int i = 0; i < OZK_NMAX; i++) {
        const int P = ozk_mod(i);
        t.P[i] = (float)P;
        t.inv[i] = 1.0f / (float)P;
        int w = 1 % P;
        for (int q = 0; q < 16; q++) {
            t.W[i][q] = (float)w;
            w = (int)(((long long)w * 1024) % P);
        }
    }
    return t;
}

__constant__ SplitTables c_split = make_split_tables();

constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23: adding it rounds a |value| < 2^22 to an integer

// 10-bit digits of X = round(|v| 2^ag) as floats, negated when v < 0, computed with exact FP64 operations:
// t = |v| 2^ag is a power-of-two scaling (exact; a result below 2^-1022 can only give X = 0),
// X = floor(t) + [t - floor(t) >= 1/2] rounds half away from zero, F_0 = X, F_{q+1} = floor(F_q / 1024) (exact
// scalings and floors), and the digit d_q = F_q - 1024 F_{q+1} is exact (Sterbenz).  This keeps the integer
// pipe free: the whole decomposition runs on the FP64 pipe, the residues on the FP32 pipe.
template <int ND>
__device__ __forceinline__ void make_digits(double v, int ag, float (&d)[ND]) {
    const double av = fabs(v);
    const bool neg = (ozk_bits(v) >> 63) != 0ULL;
    double tv;
    if (ag >= -1022 && ag <= 1023) tv = av * __longlong_as_double((long long)(ag + 1023) << 52);
    else tv = ldexp(av, ag);
    const double fl = floor(tv);
    double F = fl + ((tv - fl >= 0.5) ? 1.0 : 0.0);   // X
#pragma unroll
    for (int q = 0; q < ND; q++) {
        const double Fn = floor(F * 0.0009765625);     // floor(X 2^-10(q+1)) = floor(floor(X 2^-10q) / 1024)
        const double dq = fma(-1024.0, Fn, F);
        F = Fn;
        // the low word of 2^52 + d is d; 2^23 + d as a float is exact, minus 2^23
        const unsigned di = (unsigned)__double2loint(dq + 4503599627370496.0);
        const float fd = __fsub_rn(__uint_as_float(0x4B000000u | di), 8388608.0f);
        d[q] = neg ? -fd : fd;
    }
}

// symmetric residue byte of the digit vector modulo m_t
template <int ND>
__device__ __forceinline__ unsigned residue_bits(const float (&d)[ND], int t) {
    float s = 0.0f;
#pragma unroll
    for (int q = 0; q < ND; q++) s = __fmaf_rn(d[q], c_split.W[t][q], s);
    const float qt = __fadd_rn(__fmaf_rn(s, c_split.inv[t], kMagic), -kMagic);
    const float r = __fmaf_rn(-qt, c_split.P[t], s);
    return __float_as_uint(__fadd_rn(r, kMagic));   // low byte = r mod 256
}

__device__ __forceinline__ unsigned pack4(unsigned b0, unsigned b1, unsigned b2, unsigned b3) {
    return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// residues of 4 values, all moduli t < N, handed to `emit(t, packed_word)`
template <int ND, typename Emit>
__device__ __forceinline__ void quad_residues(const double (&v)[4], const int (&ag)[4], int N, Emit emit) {
    float d0[ND], d1[ND], d2[ND], d3[ND];
    make_digits<ND>(v[0], ag[0], d0);
    make_digits<ND>(v[1], ag[1], d1);
    make_digits<ND>(v[2], ag[2], d2);
    make_digits<ND>(v[3], ag[3], d3);
#pragma unroll
    for (int t = 0; t < OZK_NMAX; t++) {
        if (t < N) emit(t, pack4(residue_bits<ND>(d0, t), residue_bits<ND>(d1, t), residue_bits<ND>(d2, t),
                                 residue_bits<ND>(d3, t)));
    }
}

template <typename Emit>
__device__ __forceinline__ void quad_dispatch(int p, const double (&v)[4], const int (&ag)[4], int N, Emit emit) {
    const int nd = (p + 1 + 9) / 10;   // X < 2^(p+1)
    if (nd <= 6) quad_residues<6>(v, ag, N, emit);
    else if (nd <= 7) quad_residues<7>(v, ag, N, emit);
    else if (nd <= 8) quad_residues<8>(v, ag, N, emit);
    else if (nd <= 10) quad_residues<10>(v, ag, N, emit);
    else if (nd <= 12) quad_residues<12>(v, ag, N, emit);
    else quad_residues<16>(v, ag, N, emit);
}

// A (m x k, row-major) -> Ares[t][i][l]: one thread per 4 consecutive l of a row; plane stores are coalesced
__global__ void __launch_bounds__(256) split_a_kernel(const double* __restrict__ A, const int32_t* __restrict__ r,
                                                      const int32_t* __restrict__ gam, const int32_t* __restrict__ p_dev,
                                                      int m, int k, int N, int8_t* __restrict__ Ares) {
    const long long quads = (long long)m * (k >> 2);
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= quads) return;
    const int k4 = k >> 2;
    const int i = (int)(g / k4), l4 = (int)(g - (long long)i * k4);
    const int p = *p_dev;
    const double2* rowp = reinterpret_cast<const double2*>(A + (size_t)i * k) + 2 * l4;
    const double2 a01 = __ldg(rowp), a23 = __ldg(rowp + 1);
    const int4 gg = __ldg(reinterpret_cast<const int4*>(gam) + l4);
    const int base = p - __ldg(r + i);
    const double v[4] = {a01.x, a01.y, a23.x, a23.y};
    const int ag[4] = {base + gg.x, base + gg.y, base + gg.z, base + gg.w};
    const size_t plane = (size_t)m * k;
    unsigned* out = reinterpret_cast<unsigned*>(Ares + (size_t)i * k) + l4;
    quad_dispatch(p, v, ag, N, [&](int t, unsigned w) { out[(size_t)t * (plane >> 2)] = w; });
}

// B (k x n, row-major) -> Bres[t][j][l] (transposed): a block owns 32 rows l x 32 columns j; thread (j, quad of l)
// computes 4 residues per plane into shared memory, then the block writes 32-byte K-contiguous runs per (t, j).
constexpr int kBRows = 32, kBCols = 32, kBPitch = 9;   // words per (t, j) row of the smem tile: 8 + 1 pad

__global__ void __launch_bounds__(256) split_b_kernel(const double* __restrict__ B, const int32_t* __restrict__ c,
                                                      const int32_t* __restrict__ gam, const int32_t* __restrict__ p_dev,
                                                      int k, int n, int N, int8_t* __restrict__ Bres) {
    __shared__ unsigned sm[OZK_NMAX * kBCols * kBPitch];
    const int j0 = blockIdx.x * kBCols, l0 = blockIdx.y * kBRows;
    const int jj = threadIdx.x & 31, lq = threadIdx.x >> 5;   // lq: quad 0..7 of the 32 rows
    const int j = j0 + jj;
    const int p = *p_dev;
    const int base = p - __ldg(c + j);
    double v[4];
    int ag[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int l = l0 + 4 * lq + q;
        v[q] = __ldg(B + (size_t)l * n + j);
        ag[q] = base - __ldg(gam + l);
    }
    quad_dispatch(p, v, ag, N, [&](int t, unsigned w) { sm[(t * kBCols + jj) * kBPitch + lq] = w; });
    __syncthreads();
    // N planes x 32 columns x 2 chunks of 16 bytes
    const int chunks = N * kBCols * 2;
    for (int cidx = threadIdx.x; cidx < chunks; cidx += blockDim.x) {
        const int t = cidx / (kBCols * 2), rem = cidx % (kBCols * 2), jr = rem >> 1, part = rem & 1;
        const unsigned* src = sm + (t * kBCols + jr) * kBPitch + 4 * part;
        const uint4 w = make_uint4(src[0], src[1], src[2], src[3]);
        int8_t* dst = Bres + ((size_t)t * n + (j0 + jr)) * (size_t)k + l0 + 16 * part;
        *reinterpret_cast<uint4*>(dst) = w;
    }
}

}  // namespace

extern "C" int ozk_split_a(const double* A, const int32_t* r, const int32_t* gam, const int32_t* p_dev, int m, int k,
                           int N, int8_t* Ares, ozk_stream_t stream_) {
    if (!A || !r || !gam || !p_dev || !Ares) return OZK_ERR_ARG;
    if (m <= 0 || k <= 0 || (k & 31) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Ares) | reinterpret_cast<uintptr_t>(gam)) & 15)
        return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    const long long quads = (long long)m * (k >> 2);
    const long long blocks = (quads + 255) / 256;
    if (blocks > 0x7fffffffLL) return OZK_ERR_ARG;
    split_a_kernel<<<(unsigned)blocks, 256, 0, st>>>(A, r, gam, p_dev, m, k, N, Ares);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_split_b(const double* B, const int32_t* c, const int32_t* gam, const int32_t* p_dev, int k, int n,
                           int N, int8_t* Bres, ozk_stream_t stream_) {
    if (!B || !c || !gam || !p_dev || !Bres) return OZK_ERR_ARG;
    if (n <= 0 || k <= 0 || (k & 31) || (n & 31) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(Bres) & 15) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    split_b_kernel<<<dim3(n / kBCols, k / kBRows), 256, 0, st>>>(B, c, gam, p_dev, k, n, N, Bres);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
