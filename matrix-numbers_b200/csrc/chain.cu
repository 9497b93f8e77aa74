// Residue chains: the products of an exact integer chain A_1 A_2 ... A_q stay in INT8 residue form between products
// (the cost law of dl1683/matrix-numbers code/digit_gemm.py:1252-1291: one INT8 GEMM per modulus per product, the
// residues reduced after every product).  The GEMM kernel's residue epilogue already leaves X[t] = (A_t B_t^T) mod m_t
// in [0, m_t); this kernel maps those planes to the symmetric int8 range [-floor(m_t/2), ceil(m_t/2) - 1] of the
// split (code/ozaki_engine.py:989-995), so that X can be the left operand of the next product without leaving the
// device or the residue form.
//
// HBM-bound elementwise map: 16 bytes per thread and iteration, one byte-wise compare and one byte-wise subtraction
// per 4 residues (a byte r >= ceil(m/2) becomes r - m modulo 256, which is the int8 pattern of r - m; for m = 256 the
// byte is unchanged).
#include "ozk_common.cuh"

namespace {

__global__ void __launch_bounds__(256) residue_symmetric_kernel(const uint4* __restrict__ X, uint4* __restrict__ out,
                                                                int N, long long vecs_per_plane) {
    const long long total = (long long)N * vecs_per_plane;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += stride) {
        const int t = (int)(v / vecs_per_plane);
        const unsigned m = (unsigned)ozk_mod(t);
        const unsigned half4 = ((m + 1u) >> 1) * 0x01010101u;   // ceil(m / 2) in every byte (128 for m = 256)
        const unsigned m4 = (m & 0xFFu) * 0x01010101u;           // m modulo 256 in every byte
        uint4 w = __ldg(X + v);
        w.x = __vsub4(w.x, __vcmpgeu4(w.x, half4) & m4);
        w.y = __vsub4(w.y, __vcmpgeu4(w.y, half4) & m4);
        w.z = __vsub4(w.z, __vcmpgeu4(w.z, half4) & m4);
        w.w = __vsub4(w.w, __vcmpgeu4(w.w, half4) & m4);
        out[v] = w;
    }
}

}  // namespace

extern "C" int ozk_residue_symmetric(const uint8_t* X, int N, size_t plane_elems, int8_t* out, ozk_stream_t stream_) {
    if (!X || !out || N < 1 || N > OZK_NMAX || plane_elems == 0 || (plane_elems & 15)) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(out)) & 15) return OZK_ERR_ARG;
    const long long vecs = (long long)(plane_elems >> 4);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = ((long long)N * vecs + 255) / 256;
    const long long cap = 8LL * sms;
    const int blocks = (int)(want < cap ? want : cap);
    residue_symmetric_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(
        reinterpret_cast<const uint4*>(X), reinterpret_cast<uint4*>(out), N, vecs);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
