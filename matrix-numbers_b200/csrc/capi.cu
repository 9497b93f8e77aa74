// Library-level entry points of libozaki_b200.so: version, error strings, the host helpers of the reference engine
// (moduli, their float product, limb count, pmax_bits) and ozk_core, the stage-3 sequence of OzakiCRT.core.
#include <math.h>
#include <string.h>

#include "ozk_common.cuh"

#define OZK_VERSION 100

namespace {

// exact product of the first N moduli in 32-bit limbs (at most 246 bits)
void modulus_product_limbs(int N, uint32_t (&a)[10]) {
    memset(a, 0, sizeof(a));
    a[0] = 1u;
    for (int t = 0; t < N; t++) {
        uint64_t carry = 0;
        for (int q = 0; q < 10; q++) {
            const uint64_t v = (uint64_t)a[q] * (uint64_t)ozk_mod(t) + carry;
            a[q] = (uint32_t)v;
            carry = v >> 32;
        }
    }
}

bool fits_host(int p, double nuA, double nuB, double sk, double M) {
    const double tp = ldexp(1.0, p);
    volatile double x = tp * nuA;   // volatile: one rounding per operation, no contraction
    x = x + sk;
    volatile double y = tp * nuB;
    y = y + sk;
    volatile double v = 2.0 * x;
    v = v * y;
    v = v * (1.0 + 1e-9);
    v = v + 2.0;
    return v <= M;
}

}  // namespace

extern "C" int ozk_version(void) { return OZK_VERSION; }

extern "C" const char* ozk_error_string(int code) {
    switch (code) {
        case OZK_OK: return "ok";
        case OZK_ERR_ARG: return "invalid argument (shape, alignment, null pointer or count)";
        case OZK_ERR_P_RANGE: return "scaling bits p outside the supported range [0, 159]";
        case OZK_ERR_DEVICE: return "no CUDA device of compute capability 10.x (B200, sm_100) is current";
        case OZK_ERR_DRIVER: return "CUDA driver entry point or TMA tensor-map encoding failed";
        case OZK_ERR_WORKSPACE: return "workspace smaller than the size returned by the matching *_workspace_bytes query";
        case OZK_ERR_TOO_LARGE: return "problem needs more scratch than the static array of ozk_stats_noalloc (16 MiB)";
        default: break;
    }
    if (code >= OZK_ERR_CUDA_BASE) return cudaGetErrorString((cudaError_t)(code - OZK_ERR_CUDA_BASE));
    return "unknown error";
}

extern "C" int ozk_modulus(int t) { return (t >= 0 && t < OZK_NMAX) ? ozk_mod(t) : 0; }

extern "C" double ozk_modulus_product(int N) {
    if (N < 0 || N > OZK_NMAX) return 0.0;
    uint32_t a[10];
    modulus_product_limbs(N, a);
    int top = -1;
    for (int q = 9; q >= 0; q--)
        if (a[q]) { top = q; break; }
    if (top < 0) return 0.0;
    // top 64 bits with a sticky bit, rounded once (round to nearest even)
    const uint64_t w2 = a[top], w1 = top >= 1 ? a[top - 1] : 0u, w0 = top >= 2 ? a[top - 2] : 0u;
    uint32_t st = 0;
    for (int q = top - 3; q >= 0; q--) st |= a[q];
    const int lz = __builtin_clz((unsigned)w2);
    const uint64_t hi = (w2 << 32) | w1;
    uint64_t qv;
    uint32_t lost;
    if (lz == 0) { qv = hi; lost = (uint32_t)w0; }
    else { qv = (hi << lz) | (w0 >> (32 - lz)); lost = (uint32_t)(w0 << lz); }
    if ((lost | st) != 0u) qv |= 1ULL;
    return ldexp((double)qv, 32 * (top - 1) - lz);
}

extern "C" int ozk_limbs_for(int N) {
    if (N < 0 || N > OZK_NMAX) return 0;
    uint32_t a[10];
    modulus_product_limbs(N, a);
    int bits = 0;
    for (int q = 9; q >= 0; q--)
        if (a[q]) { bits = 32 * q + 32 - __builtin_clz(a[q]); break; }
    const int L = (bits + 31) / 32;
    return L < 2 ? 2 : L;
}

extern "C" int ozk_pmax_bits(int N, double nuA, double nuB, int k) {
    if (N < 1 || N > OZK_NMAX || k <= 0) return 0;
    const double M = ozk_modulus_product(N);
    const double sk = sqrt((double)k) / 2.0;
    if (!fits_host(0, nuA, nuB, sk, M)) return 0;
    const double a = nuA * nuB, bq = sk * (nuA + nuB), cq = sk * sk - (M - 2.0) / (2.0 * (1.0 + 1e-9));
    double y;
    if (a == 0.0) y = bq > 0.0 ? -cq / bq : ldexp(1.0, 249);
    else y = (-bq + sqrt(fmax(bq * bq - 4.0 * a * cq, 0.0))) / (2.0 * a);
    int p = 0;
    if (y > 0.0) { const double f = floor(log2(y)); p = f < 0.0 ? 0 : (f > 249.0 ? 249 : (int)f); }
    while (p > 0 && !fits_host(p, nuA, nuB, sk, M)) p--;
    while (p < 249 && fits_host(p + 1, nuA, nuB, sk, M)) p++;
    return p;
}

extern "C" int ozk_core(const double* A, const double* B, const int32_t* gam, const int32_t* r, const int32_t* c,
                        const int32_t* p_dev, int m, int n, int k, int N, int skip_a, int8_t* Ares, int8_t* Bres,
                        uint8_t* X, double* C, int32_t* err, ozk_stream_t stream) {
    int rc;
    if (!skip_a && (rc = ozk_split_a(A, r, gam, p_dev, m, k, N, Ares, err, stream)) != OZK_OK) return rc;
    if ((rc = ozk_split_b(B, c, gam, p_dev, k, n, N, Bres, err, stream)) != OZK_OK) return rc;
    if ((rc = ozk_gemm_residues(Ares, Bres, m, n, k, N, X, err, stream)) != OZK_OK) return rc;
    return ozk_reconstruct(X, r, c, p_dev, m, n, N, C, err, stream);
}
