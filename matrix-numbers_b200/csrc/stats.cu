// Stage 1: per-index statistics of A and B (the reference's CU_STATS kernels, code/ozaki_engine.py:846-951,
// launched in the order of OzakiCRT.stats, :1229-1247).
//
// Differences from the reference, by design:
//   - every sum is reduced in a fixed order (per-thread strided sums, a fixed shuffle tree, then partial sums per
//     row chunk added in chunk order), so sB / nB are bitwise reproducible; the reference adds them with double
//     atomicAdd (:949-950), whose order varies from run to run;
//   - loads are 16-byte vectors, coalesced along the contiguous index of each matrix.
#include "ozk_common.cuh"
#include <atomic>

namespace {

constexpr int kThreads = 256;
constexpr int kColmaxRows = 64;     // rows of A folded by one block of colmax_a_kernel
// rows of B folded by one block of the column kernels: at most 512, fewer when B has few columns, so that the grid
// keeps about 600 blocks (a function of n and k only: the workspace size depends on it)
__host__ __device__ inline int col_chunk_rows(int n, int k) {
    const int colblocks = (n / 2 + 255) / 256;
    const int want = (600 + colblocks - 1) / colblocks;
    int rows = (k + want - 1) / want;
    rows = (rows + 7) & ~7;
    return rows < 8 ? 8 : (rows > 512 ? 512 : rows);
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T identity, T* sm, Op op) {
    // fixed-order tree: warp shuffle, then warp 0 over the per-warp results; the result is broadcast
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_down_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    __syncthreads();
    if (ln == 0) sm[w] = v;
    __syncthreads();
    if (w == 0) {
        v = ln < (int)(blockDim.x >> 5) ? sm[ln] : identity;
        for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_down_sync(0xffffffffu, v, o));
        if (ln == 0) sm[0] = v;
    }
    __syncthreads();
    T r = sm[0];
    __syncthreads();
    return r;
}

__device__ __forceinline__ double block_sum(double v, double* sm) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, ln = threadIdx.x & 31;
    __syncthreads();
    if (ln == 0) sm[w] = v;
    __syncthreads();
    if (w == 0) {
        v = ln < (int)(blockDim.x >> 5) ? sm[ln] : 0.0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
        if (ln == 0) sm[0] = v;
    }
    __syncthreads();
    double r = sm[0];
    __syncthreads();
    return r;
}

struct MaxU64 { __device__ unsigned long long operator()(unsigned long long a, unsigned long long b) const { return a > b ? a : b; } };
struct MaxI { __device__ int operator()(int a, int b) const { return a > b ? a : b; } };

// column max of |A| bit patterns (colmax_k, :847-854): 2 columns per thread, kColmaxRows rows per block
__global__ void __launch_bounds__(kThreads) colmax_a_kernel(const double* __restrict__ A, unsigned long long* __restrict__ colmax,
                                                            int m, int k) {
    const int l = 2 * (blockIdx.x * kThreads + threadIdx.x);
    if (l >= k) return;
    const int i0 = blockIdx.y * kColmaxRows, i1 = min(m, i0 + kColmaxRows);
    unsigned long long m0 = 0, m1 = 0;
    for (int i = i0; i < i1; i++) {
        const ulonglong2 v = __ldg(reinterpret_cast<const ulonglong2*>(A + (size_t)i * k + l));
        m0 = max(m0, v.x & OZK_ABSMASK);
        m1 = max(m1, v.y & OZK_ABSMASK);
    }
    atomicMax(colmax + l, m0);
    atomicMax(colmax + l + 1, m1);
}

// row max of |B| bit patterns (rowmax_k, :855-869): one block per row of B
__global__ void __launch_bounds__(kThreads) rowmax_b_kernel(const double* __restrict__ B, unsigned long long* __restrict__ rowmax, int n) {
    __shared__ unsigned long long sm[32];
    const int l = blockIdx.x;
    const ulonglong2* row = reinterpret_cast<const ulonglong2*>(B + (size_t)l * n);
    unsigned long long mx = 0;
    for (int j = threadIdx.x; j < n / 2; j += kThreads) {
        const ulonglong2 v = __ldg(row + j);
        mx = max(mx, max(v.x & OZK_ABSMASK, v.y & OZK_ABSMASK));
    }
    mx = block_reduce(mx, 0ULL, sm, MaxU64());
    if (threadIdx.x == 0) rowmax[l] = mx;
}

// gamma_l = (e_B - e_A) >> 1, 0 when disabled, when either side is zero or non-finite (gamma_k, :870-879)
__global__ void gamma_kernel(const unsigned long long* __restrict__ colmax, const unsigned long long* __restrict__ rowmax,
                             int32_t* __restrict__ gam, int32_t* __restrict__ flag, int k, int enable) {
    const int l = blockIdx.x * blockDim.x + threadIdx.x;
    if (l >= k) return;
    const unsigned long long a = colmax[l], b = rowmax[l];
    const bool bad = ((a >> 52) == 0x7ffULL) || ((b >> 52) == 0x7ffULL);
    if (bad) atomicOr(flag, 1);
    const int ea = ozk_fexp(a), eb = ozk_fexp(b);
    gam[l] = (!enable || bad || ea == OZK_NEG || eb == OZK_NEG) ? 0 : ((eb - ea) >> 1);
}

// x 2^e for |e| in the normal exponent range by one multiplication with an exact power of two (exact unless the
// result leaves the normal range, where ldexp takes over)
__device__ __forceinline__ double scale2(double x, int e) {
    if (e >= -1022 && e <= 1023) return x * __longlong_as_double((long long)(e + 1023) << 52);
    return ldexp(x, e);
}

// Running statistics of a set of values |x| 2^g (x != 0) with a running maximum exponent emax:
//   s = sum |x| 2^g,  q = sum (|x| 2^(g - emax))^2.
// When emax grows by d, q is rescaled by 2^-2d (an exact power-of-two scaling), so one pass gives the same sums as the
// reference's two passes (max first, then sums relative to it) up to the order of additions.
//
// add_abs is the per-element entry: z = |x| 2^g is formed by one multiplication with a power of two built from its
// bits, which is exact while z is normal; then e(z) = e(x) + g is read from z's exponent field, s += z, and
// y = z 2^-emax uses R = 2^-emax kept in a register.  Each of s, y and q is the same correctly rounded value as in the
// general path (add), so the results are bitwise the same; elements whose z is not normal or whose running maximum
// leaves [-1022, 1022] take the general path.
struct RunStats {
    int emax;
    double s, q, R;                 // R = 2^-emax while emax is in [-1022, 1022], else 0
    __device__ __forceinline__ void init() { emax = OZK_NEG; s = 0.0; q = 0.0; R = 0.0; }
    __device__ __forceinline__ void set_emax(int e) {
        emax = e;
        R = (e >= -1022 && e <= 1022) ? __hiloint2double((1023 - e) << 20, 0) : 0.0;
    }
    __device__ __forceinline__ void add(double x, int e_plus_g, int g) {   // x = |value| != 0
        if (e_plus_g > emax) {
            if (emax != OZK_NEG) q = scale2(q, -2 * (e_plus_g - emax));
            set_emax(e_plus_g);
        }
        s += scale2(x, g);
        const double y = scale2(x, g - emax);
        q = fma(y, y, q);
    }
    __device__ __forceinline__ void add_abs(double a, int g) {            // a = |value|, zero allowed
        const bool gok = g >= -1022 && g <= 1023;
        const double z = a * __hiloint2double((gok ? g + 1023 : 1023) << 20, 0);
        const int ez = (int)((unsigned)__double2hiint(z) >> 20);           // biased exponent (z >= 0)
        const int e = ez - 1022;                                            // frexp exponent of z
        if (gok && ez >= 1 && ez <= 2046 && (e > emax ? e <= 1022 : R != 0.0)) {
            if (e > emax) {
                if (emax != OZK_NEG) q = scale2(q, -2 * (e - emax));
                set_emax(e);
            }
            s += z;
            const double y = z * R;
            q = fma(y, y, q);
        } else if (a != 0.0) {
            add(a, ozk_fexp(ozk_bits(a)) + g, g);
        }
    }
};

// r_i = max_l (e(A_il) + gamma_l) over non-zeros (0 if none); sA_i = sum |A_il| 2^gamma_l;
// nA_i = sum (|A_il| 2^(gamma_l - r_i))^2   (rowstatsA_k, :904-925); one block per row, one pass over the row
__global__ void __launch_bounds__(kThreads) rowstats_a_kernel(const double* __restrict__ A, const int32_t* __restrict__ gam, int k,
                                                              int32_t* __restrict__ r_out, double* __restrict__ s_out,
                                                              double* __restrict__ n_out) {
    __shared__ int smi[32];
    __shared__ double smd[32];
    const int i = blockIdx.x;
    const double2* row = reinterpret_cast<const double2*>(A + (size_t)i * k);
    const int2* g2 = reinterpret_cast<const int2*>(gam);
    RunStats rs;
    rs.init();
    for (int h = threadIdx.x; h < k / 2; h += kThreads) {
        const double2 v = __ldg(row + h);
        const int2 g = __ldg(g2 + h);
        rs.add_abs(fabs(v.x), g.x);
        rs.add_abs(fabs(v.y), g.y);
    }
    const int mx = block_reduce(rs.emax, (int)OZK_NEG, smi, MaxI());
    const int rr = mx <= OZK_NEG / 2 ? 0 : mx;
    const double q = rs.emax == OZK_NEG ? 0.0 : scale2(rs.q, -2 * (mx - rs.emax));
    const double s = block_sum(rs.s, smd);
    const double qq = block_sum(q, smd);
    if (threadIdx.x == 0) { r_out[i] = rr; s_out[i] = s; n_out[i] = qq; }
}

// column statistics of B over one chunk of `chunk` rows, 2 columns per thread, one pass (colexpB_k and colsumsB_k,
// :926-951): per chunk the local maximum exponent, sB partial and nB partial relative to the local maximum
__global__ void __launch_bounds__(kThreads) colstats_b_kernel(const double* __restrict__ B, const int32_t* __restrict__ gam,
                                                              int k, int n, int chunk, int32_t* __restrict__ pc,
                                                              double* __restrict__ ps, double* __restrict__ pq) {
    const int j = 2 * (blockIdx.x * kThreads + threadIdx.x);
    if (j >= n) return;
    const int l0 = blockIdx.y * chunk, l1 = min(k, l0 + chunk);
    RunStats r0, r1;
    r0.init();
    r1.init();
    for (int l = l0; l < l1; l++) {
        const double2 v = __ldg(reinterpret_cast<const double2*>(B + (size_t)l * n + j));
        const int g = -__ldg(gam + l);
        r0.add_abs(fabs(v.x), g);
        r1.add_abs(fabs(v.y), g);
    }
    const size_t o = (size_t)blockIdx.y * n + j;
    pc[o] = r0.emax; pc[o + 1] = r1.emax;
    ps[o] = r0.s; ps[o + 1] = r1.s;
    pq[o] = r0.q; pq[o + 1] = r1.q;
}

// chunk partials combined: c_j = max of the local maxima (0 when the column has no non-zero, as the consumers of c do
// at :1257, :1060), sB_j = sum, nB_j = sum of the partials rescaled to c_j.  One block per 32 columns (lane = column,
// so every chunk row is read coalesced) and kFinWarps warps over the chunks (warp w: chunks w, w + kFinWarps, ...);
// the warps' results are combined in warp order, so the sums have a fixed order (bitwise reproducible).
constexpr int kFinWarps = 8;
__global__ void __launch_bounds__(kFinWarps * 32) colstats_final_kernel(const int32_t* __restrict__ pc,
                                                                        const double* __restrict__ ps,
                                                                        const double* __restrict__ pq, int nchunks,
                                                                        int n, int32_t* __restrict__ c,
                                                                        double* __restrict__ sB,
                                                                        double* __restrict__ nB) {
    __shared__ int smx[kFinWarps][32];
    __shared__ double sms[kFinWarps][32], smq[kFinWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int j = blockIdx.x * 32 + lane;
    const bool ok = j < n;
    int mx = OZK_NEG;
    if (ok)
        for (int h = w; h < nchunks; h += kFinWarps) mx = max(mx, __ldg(pc + (size_t)h * n + j));
    smx[w][lane] = mx;
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kFinWarps; u++) mx = max(mx, smx[u][lane]);
    double s = 0.0, q = 0.0;
    if (ok)
        for (int h = w; h < nchunks; h += kFinWarps) {
            const size_t o = (size_t)h * n + j;
            const int e = __ldg(pc + o);
            s += __ldg(ps + o);
            if (e != OZK_NEG) q += scale2(__ldg(pq + o), -2 * (mx - e));
        }
    sms[w][lane] = s;
    smq[w][lane] = q;
    __syncthreads();
    if (w == 0 && ok) {
        double S = 0.0, Q = 0.0;
#pragma unroll
        for (int u = 0; u < kFinWarps; u++) {
            S += sms[u][lane];
            Q += smq[u][lane];
        }
        sB[j] = S;
        nB[j] = Q;
        c[j] = mx <= OZK_NEG / 2 ? 0 : mx;
    }
}

}  // namespace

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

extern "C" size_t ozk_stats_workspace_bytes(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    const size_t nchunks = ((size_t)k + col_chunk_rows(n, k) - 1) / col_chunk_rows(n, k);
    return align256((size_t)k * 8) * 2 + align256(nchunks * (size_t)n * 8) * 2 + align256(nchunks * (size_t)n * 4);
}

extern "C" int ozk_stats_colmax(const double* A, int m, int k, uint64_t* colmax, ozk_stream_t stream_) {
    if (!A || !colmax) return OZK_ERR_ARG;
    if (m <= 0 || k <= 0 || (k & 1)) return OZK_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(A) & 15) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    if (cudaMemsetAsync(colmax, 0, (size_t)k * 8, st) != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    colmax_a_kernel<<<dim3((k / 2 + kThreads - 1) / kThreads, (m + kColmaxRows - 1) / kColmaxRows), kThreads, 0, st>>>(
        A, reinterpret_cast<unsigned long long*>(colmax), m, k);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_stats_finish(const double* A, const double* B, int m, int n, int k, int inside, const uint64_t* colmax,
                                int32_t* gam, int32_t* r, int32_t* c, double* sA, double* nA, double* sB, double* nB,
                                int32_t* flag, void* workspace, size_t workspace_bytes, ozk_stream_t stream_) {
    if (!A || !B || !colmax || !gam || !r || !c || !sA || !nA || !sB || !nB || !flag || !workspace) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0 || (k & 1) || (n & 1)) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return OZK_ERR_ARG;
    if (workspace_bytes < ozk_stats_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    const int chunk = col_chunk_rows(n, k);
    const int nchunks = (k + chunk - 1) / chunk;
    char* ws = static_cast<char*>(workspace);
    unsigned long long* rowmax = reinterpret_cast<unsigned long long*>(ws + align256((size_t)k * 8));
    double* ps = reinterpret_cast<double*>(ws + 2 * align256((size_t)k * 8));
    double* pq = reinterpret_cast<double*>(ws + 2 * align256((size_t)k * 8) + align256((size_t)nchunks * n * 8));
    if (cudaMemsetAsync(flag, 0, 4, st) != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    rowmax_b_kernel<<<k, kThreads, 0, st>>>(B, rowmax, n);
    OZK_CHECK_LAUNCH();
    gamma_kernel<<<(k + 255) / 256, 256, 0, st>>>(reinterpret_cast<const unsigned long long*>(colmax), rowmax, gam, flag,
                                                  k, inside ? 1 : 0);
    OZK_CHECK_LAUNCH();
    rowstats_a_kernel<<<m, kThreads, 0, st>>>(A, gam, k, r, sA, nA);
    OZK_CHECK_LAUNCH();
    int32_t* pc = reinterpret_cast<int32_t*>(ws + 2 * align256((size_t)k * 8) + 2 * align256((size_t)nchunks * n * 8));
    const dim3 g2((n / 2 + kThreads - 1) / kThreads, nchunks);
    colstats_b_kernel<<<g2, kThreads, 0, st>>>(B, gam, k, n, chunk, pc, ps, pq);
    OZK_CHECK_LAUNCH();
    colstats_final_kernel<<<(n + 31) / 32, kFinWarps * 32, 0, st>>>(pc, ps, pq, nchunks, n, c, sB, nB);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_stats_rowmax(const double* B, int k, int n, uint64_t* rowmax, ozk_stream_t stream_) {
    if (!B || !rowmax) return OZK_ERR_ARG;
    if (n <= 0 || k <= 0 || (n & 1)) return OZK_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(B) & 15) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    rowmax_b_kernel<<<k, kThreads, 0, st>>>(B, reinterpret_cast<unsigned long long*>(rowmax), n);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_stats_gamma(const uint64_t* colmax, const uint64_t* rowmax, int k, int inside, int32_t* gam,
                               int32_t* flag, ozk_stream_t stream_) {
    if (!colmax || !rowmax || !gam || !flag || k <= 0) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    if (cudaMemsetAsync(flag, 0, 4, st) != cudaSuccess) return OZK_ERR_CUDA_BASE + (int)cudaGetLastError();
    gamma_kernel<<<(k + 255) / 256, 256, 0, st>>>(reinterpret_cast<const unsigned long long*>(colmax),
                                                  reinterpret_cast<const unsigned long long*>(rowmax), gam, flag, k,
                                                  inside ? 1 : 0);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_stats_rows(const double* A, int m, int k, const int32_t* gam, int32_t* r, double* sA, double* nA,
                              ozk_stream_t stream_) {
    if (!A || !gam || !r || !sA || !nA) return OZK_ERR_ARG;
    if (m <= 0 || k <= 0 || (k & 1)) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(gam)) & 15) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    rowstats_a_kernel<<<m, kThreads, 0, st>>>(A, gam, k, r, sA, nA);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" size_t ozk_stats_cols_workspace_bytes(int k, int n) {
    if (n <= 0 || k <= 0) return 0;
    const size_t nchunks = ((size_t)k + col_chunk_rows(n, k) - 1) / col_chunk_rows(n, k);
    return align256(nchunks * (size_t)n * 8) * 2 + align256(nchunks * (size_t)n * 4);
}

extern "C" int ozk_stats_cols(const double* B, int k, int n, const int32_t* gam, int32_t* c, double* sB, double* nB,
                              void* workspace, size_t workspace_bytes, ozk_stream_t stream_) {
    if (!B || !gam || !c || !sB || !nB || !workspace) return OZK_ERR_ARG;
    if (n <= 0 || k <= 0 || (n & 1)) return OZK_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(B) & 15) return OZK_ERR_ARG;
    if (workspace_bytes < ozk_stats_cols_workspace_bytes(k, n)) return OZK_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    const int chunk = col_chunk_rows(n, k);
    const int nchunks = (k + chunk - 1) / chunk;
    char* ws = static_cast<char*>(workspace);
    double* ps = reinterpret_cast<double*>(ws);
    double* pq = reinterpret_cast<double*>(ws + align256((size_t)nchunks * n * 8));
    int32_t* pc = reinterpret_cast<int32_t*>(ws + 2 * align256((size_t)nchunks * n * 8));
    const dim3 g2((n / 2 + kThreads - 1) / kThreads, nchunks);
    colstats_b_kernel<<<g2, kThreads, 0, st>>>(B, gam, k, n, chunk, pc, ps, pq);
    OZK_CHECK_LAUNCH();
    colstats_final_kernel<<<(n + 31) / 32, kFinWarps * 32, 0, st>>>(pc, ps, pq, nchunks, n, c, sB, nB);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_stats(const double* A, const double* B, int m, int n, int k, int inside, int32_t* gam, int32_t* r,
                         int32_t* c, double* sA, double* nA, double* sB, double* nB, int32_t* flag, void* workspace,
                         size_t workspace_bytes, ozk_stream_t stream) {
    if (!workspace || workspace_bytes < ozk_stats_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    uint64_t* colmax = static_cast<uint64_t*>(workspace);   // the first region of the workspace
    int rc = ozk_stats_colmax(A, m, k, colmax, stream);
    if (rc != OZK_OK) return rc;
    return ozk_stats_finish(A, B, m, n, k, inside, colmax, gam, r, c, sA, nA, sB, nB, flag, workspace, workspace_bytes,
                            stream);
}

// ---- statistics without a caller-supplied workspace -------------------------------------------------------------
// For callers that cannot allocate device memory: code that only receives raw device pointers from another runtime
// (a solver or database plugin whose host owns every allocation), or code that must not call cudaMalloc in the middle
// of its work (inside a real-time loop, or while it is recording a CUDA graph).  The scratch of the statistics lives
// in the static array below instead of a workspace argument.  It exists once per device that loads this library and
// stays allocated until the process exits; every call uses the same bytes, so calls whose work overlaps on the GPU
// (different streams, or different host threads) race and must be serialised by the caller.
namespace {

__device__ __align__(256) unsigned char g_stats_scratch[OZK_STATS_NOALLOC_MAX_BYTES];

// device address of g_stats_scratch, per device ordinal (set up on first use); atomic because several host threads
// may make their first call at once (they all store the same address)
std::atomic<void*> g_stats_scratch_ptr[64];

}  // namespace

extern "C" int ozk_stats_noalloc(const double* A, const double* B, int m, int n, int k, int inside, int32_t* gam,
                                 int32_t* r, int32_t* c, double* sA, double* nA, double* sB, double* nB, int32_t* flag,
                                 ozk_stream_t stream) {
    const size_t need = ozk_stats_workspace_bytes(m, n, k);
    if (need == 0) return OZK_ERR_ARG;
    if (need > (size_t)OZK_STATS_NOALLOC_MAX_BYTES) return OZK_ERR_TOO_LARGE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return OZK_ERR_DEVICE;
    void* scratch = g_stats_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (!scratch) {
        // one-time set-up on this device (the current one): the host-side name of the array is not a device address
        const cudaError_t e = cudaGetSymbolAddress(&scratch, g_stats_scratch);
        if (e != cudaSuccess || !scratch) return OZK_ERR_CUDA_BASE + (int)e;
        g_stats_scratch_ptr[dev].store(scratch, std::memory_order_relaxed);
    }
    // the statistics clear what must start at zero (the column maxima, the flag); everything else is overwritten
    return ozk_stats(A, B, m, n, k, inside, gam, r, c, sA, nA, sB, nB, flag, scratch,
                     (size_t)OZK_STATS_NOALLOC_MAX_BYTES, stream);
}
