// Shared definitions for the sm_100a kernels of the FP64-on-INT8 (Ozaki-II / CRT) GEMM engine.
//
// The moduli, the exponent convention and the residue semantics follow the reference engine
// dl1683/matrix-numbers code/ozaki_engine.py (moduli :824-829, fexp :838-843, residue range :989-995).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ozaki_b200.h"

#define OZK_NMAX 32
#define OZK_NEG (-1000000)
#define OZK_ABSMASK 0x7fffffffffffffffULL

// The 32 pairwise-coprime moduli <= 256; a product with N planes uses the first N (ozaki_engine.py:824-825).
__host__ __device__ constexpr int ozk_mod(int t) {
    constexpr int m[OZK_NMAX] = {256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193,
                                 191, 181, 179, 173, 167, 163, 157, 151, 149, 139, 137, 131, 127, 113, 109, 107};
    return m[t];
}

// frexp exponent of |x| from the |x| bit pattern; OZK_NEG for zero (ozaki_engine.py:838-843).
__device__ __forceinline__ int ozk_fexp(unsigned long long b) {
    if (b == 0ULL) return OZK_NEG;
    unsigned E = (unsigned)(b >> 52);
    if (E == 0u) return (63 - __clzll((long long)b)) - 1073;
    return (int)E - 1022;
}

__device__ __forceinline__ unsigned long long ozk_bits(double x) { return (unsigned long long)__double_as_longlong(x); }

// Upper bound of any p this build accepts: the split kernel's digit sums stay exact in FP32 up to here.
#define OZK_PMAX_SUPPORTED 159

// Segment of the contraction index over which one INT32 accumulator is exact: 65536 * 128 * 128 = 2^30.
#define OZK_KSEG 65536

#define OZK_CHECK_LAUNCH()                                        \
    do {                                                          \
        cudaError_t e_ = cudaGetLastError();                      \
        if (e_ != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)e_; \
    } while (0)
