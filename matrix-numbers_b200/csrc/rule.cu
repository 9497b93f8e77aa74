// Stage 2: the a-priori plane-count rule (Lemma L1 on a probe set), entirely on the device.
//
// Mathematics of the reference's host rule OzakiCRT.choose (code/ozaki_engine.py:1250-1307):
//   nu_A = sqrt(max nA), nu_B = sqrt(max nB); pv[N] = pmax_bits(N, nu_A, nu_B, k) for N = 6..32 (:1119-1139);
//   probe rows I = random rows (RandomState(seed), given by the caller) + the 32 largest 2^r_i k / sA_i, columns J
//   likewise (:1265-1271); D = |A_I| |B_J| (:1277); F1 = (2^r_i sB_j + 2^c_j sA_i) / 2, F2 = k 2^(r_i + c_j) / 4;
//   p_req = smallest p >= 1 with (F1 2^-p + F2 2^-2p) * safety <= tau * D on every probe entry with D > 0, searched
//   by the two while-loops of :1290-1296 (capped at 249); N = smallest N in [6, 32] with pv[N] >= p_req, else
//   fallback (:1300-1307).  The forced-configuration branch follows _rule_device (:1387-1396).
//
// The loop conditions are evaluated with explicitly rounded double operations (__dmul_rn, __dadd_rn), one rounding
// per operation as numpy does, so the decisions equal the host rule's for equal statistics and equal D.  Because
// ok(p) is monotone in p, the smallest p is found per probe entry and p_req is their maximum.
//
// Kernels: rule_prep (1 block: nu, pv, forced / non-finite decisions, the top-32 selections), probe_partial
// (split-K FP64 probe product), probe_reduce (partials added in block order), rule_preq (one probe entry per
// thread: p_req as the maximum of the per-entry p) and rule_final (one entry per thread: worst E/D; the last block
// to finish decides N and p).
#include <math.h>

#include "ozk_common.cuh"

namespace {

constexpr int kProbeMax = 96;          // at most 64 random + 32 hard indices per side
constexpr int kPrepThreads = 1024;
constexpr int kFinalThreads = 256;
constexpr int kFinalBlocks = (kProbeMax * kProbeMax + kFinalThreads - 1) / kFinalThreads;   // one probe entry per thread
constexpr int kProbeThreads = 256;
constexpr int kProbeK = 16;            // contraction rows per smem tile of the probe product
constexpr double kOnePlus = 1.0 + 1e-9;

struct MTable { double M[OZK_NMAX + 1]; };   // M[N] = float(prod of the first N moduli)

struct RuleCtl {            // lives at the start of the workspace
    int done;               // 1: the decision is already made (forced N, non-finite input)
    int nI, nJ;
    int pad;
    int pv[OZK_NMAX + 1];
    double nuA, nuB;
    int I[kProbeMax];
    int J[kProbeMax];
    int preq_max;                    // the rule's final kernels: largest per-entry p so far
    unsigned int fin_count;          // blocks of the last kernel that are done
    unsigned long long worst_bits;   // largest E / D at p_req (bit pattern of a non-negative double)
};

__device__ __forceinline__ bool fits(int p, double nuA, double nuB, double sk, double M) {
    const double tp = ldexp(1.0, p);
    const double x = __dadd_rn(__dmul_rn(tp, nuA), sk);
    const double y = __dadd_rn(__dmul_rn(tp, nuB), sk);
    double v = __dmul_rn(2.0, x);
    v = __dmul_rn(v, y);
    v = __dmul_rn(v, kOnePlus);
    v = __dadd_rn(v, 2.0);
    return v <= M;
}

// largest p in [0, 249] with fits(p): closed-form start, then the reference's fix-up loops (:1119-1139)
__device__ int pmax_bits_dev(double M, double nuA, double nuB, int k) {
    const double sk = __dmul_rn(__dsqrt_rn((double)k), 0.5);
    if (!fits(0, nuA, nuB, sk, M)) return 0;
    const double a = nuA * nuB, bq = sk * (nuA + nuB), cq = sk * sk - (M - 2.0) / (2.0 * kOnePlus);
    double y;
    if (a == 0.0) y = bq > 0.0 ? -cq / bq : ldexp(1.0, 249);
    else y = (-bq + sqrt(fmax(bq * bq - 4.0 * a * cq, 0.0))) / (2.0 * a);
    int p = 0;
    if (y > 0.0) { const double f = floor(log2(y)); p = f < 0.0 ? 0 : (f > 249.0 ? 249 : (int)f); }
    while (p > 0 && !fits(p, nuA, nuB, sk, M)) p--;
    while (p < 249 && fits(p + 1, nuA, nuB, sk, M)) p++;
    return p;
}

__device__ __forceinline__ double hard_value(int e, double s, int k) {
    // 2^e k / s where s > 0, else 0 (:1269-1270)
    return s > 0.0 ? __ddiv_rn(__dmul_rn(ldexp(1.0, e), (double)k), s) : 0.0;
}

// Stable top-32 selection ("larger value first, then lower index"): the values are hard values (>= 0, +inf possible,
// never NaN), so their bit patterns order like the values.  A warp keeps the sorted top-32 of its segment, one entry
// per lane (a 32-element bitonic sort per chunk of 32, then a bitonic merge with the running list); the warps' lists
// are merged pairwise through shared memory.  Ties between values are broken by index, so the result is the same set
// and order as a stable sort.
struct KeyIdx { unsigned long long key; int idx; };

__device__ __forceinline__ bool kbefore(unsigned long long k, int i, unsigned long long bk, int bi) {
    return k > bk || (k == bk && i < bi);
}

__device__ __forceinline__ void cswap_lane(unsigned long long& key, int& idx, int j, bool keep_better) {
    const unsigned long long pk = __shfl_xor_sync(0xffffffffu, key, j);
    const int pi = __shfl_xor_sync(0xffffffffu, idx, j);
    const bool take = keep_better ? kbefore(pk, pi, key, idx) : kbefore(key, idx, pk, pi);
    if (take) { key = pk; idx = pi; }
}

// lanes hold a bitonic sequence; leaves it sorted best-first
__device__ __forceinline__ void bitonic_merge_desc(unsigned long long& key, int& idx) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) cswap_lane(key, idx, j, (lane & j) == 0);
}

__device__ __forceinline__ void bitonic_sort_desc(unsigned long long& key, int& idx) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) cswap_lane(key, idx, j, (((lane & k) == 0) == ((lane & j) == 0)));
}

// merge the other sorted list (ok, oi: entry `lane` of it) into this one; keeps the best 32, sorted
__device__ __forceinline__ void merge_lists(unsigned long long& key, int& idx, unsigned long long ok, int oi) {
    const int lane = threadIdx.x & 31;
    const unsigned long long rk = __shfl_sync(0xffffffffu, ok, 31 - lane);
    const int ri = __shfl_sync(0xffffffffu, oi, 31 - lane);
    if (kbefore(rk, ri, key, idx)) { key = rk; idx = ri; }
    bitonic_merge_desc(key, idx);
}

constexpr int kNoIdx = 0x7fffffff;

// The stable top-32 of `len` (key, index) pairs given by ld(x) = (key, idx) for x in [0, len): each warp keeps the
// sorted top-32 of its contiguous segment, the warps' lists are merged pairwise in shared memory.  On return warp 0
// holds the result, entry `lane` in (key, idx) (idx kNoIdx where fewer than 32 pairs exist).
template <typename Loader>
__device__ void top32(Loader ld, int len, KeyIdx* lists, unsigned long long& key, int& idx) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int seg = (len + nw - 1) / nw;
    const int b0 = w * seg, b1 = min(len, b0 + seg);
    key = 0ULL;
    idx = kNoIdx;
    for (int c0 = b0; c0 < b1; c0 += 32) {
        const int x = c0 + lane;
        unsigned long long ck = 0ULL;
        int ci = kNoIdx;
        if (x < b1) ld(x, ck, ci);
        bitonic_sort_desc(ck, ci);
        merge_lists(key, idx, ck, ci);
    }
    lists[w * 32 + lane] = KeyIdx{key, idx};
    __syncthreads();
    for (int half = nw >> 1; half > 0; half >>= 1) {
        if (w < half) {
            const KeyIdx o = lists[(w + half) * 32 + lane];
            merge_lists(key, idx, o.key, o.idx);
        }
        __syncthreads();
        if (w < half) lists[w * 32 + lane] = KeyIdx{key, idx};
        __syncthreads();
    }
}

// Hard-index candidates: block b < nbr takes rows [b kHardSeg, (b + 1) kHardSeg) of the hard values 2^r_i k / sA_i,
// the other blocks the columns; each writes the stable top-32 of its segment as (key, global index) pairs.  The
// global top-32 of a side is the top-32 of its blocks' candidates (every member is in its own segment's top-32, and
// the pairs keep the original index for the ties), merged by rule_prep_kernel.
constexpr int kHardSeg = 256;
constexpr int kHardThreads = 256;
__host__ __device__ inline int hard_blocks(int len) { return (len + kHardSeg - 1) / kHardSeg; }

__global__ void __launch_bounds__(kHardThreads) hard_cand_kernel(const int32_t* __restrict__ r,
                                                                 const int32_t* __restrict__ c,
                                                                 const double* __restrict__ sA,
                                                                 const double* __restrict__ sB, int m, int n, int k,
                                                                 unsigned long long* __restrict__ ckey,
                                                                 int* __restrict__ cidx) {
    __shared__ KeyIdx lists[kHardThreads];
    const int nbr = hard_blocks(m);
    const bool rows = (int)blockIdx.x < nbr;
    const int b = rows ? (int)blockIdx.x : (int)blockIdx.x - nbr;
    const int base = b * kHardSeg;
    const int len = min(kHardSeg, (rows ? m : n) - base);
    const int32_t* e = rows ? r : c;
    const double* sv = rows ? sA : sB;
    unsigned long long key;
    int idx;
    top32([&](int x, unsigned long long& ck, int& ci) {
        ck = (unsigned long long)__double_as_longlong(hard_value(e[base + x], sv[base + x], k));
        ci = base + x;
    }, len, lists, key, idx);
    if (threadIdx.x < 32) {
        ckey[(size_t)blockIdx.x * 32 + threadIdx.x] = key;
        cidx[(size_t)blockIdx.x * 32 + threadIdx.x] = idx;
    }
}

__device__ double block_max(double v, double* sm) {
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_down_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double a = sm[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) a = fmax(a, sm[w]);
        sm[0] = a;
    }
    __syncthreads();
    const double r = sm[0];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(kPrepThreads) rule_prep_kernel(
    const int32_t* __restrict__ r, const int32_t* __restrict__ c, const double* __restrict__ sA,
    const double* __restrict__ nA, const double* __restrict__ sB, const double* __restrict__ nB,
    const int32_t* __restrict__ flag, const int64_t* __restrict__ Ir, int nIr, const int64_t* __restrict__ Jr, int nJr,
    int m, int n, int k, int force_N, int force_p, MTable mt, RuleCtl* __restrict__ ctl, int32_t* __restrict__ dec,
    int32_t* __restrict__ p_dev, double* __restrict__ aux, const unsigned long long* __restrict__ ckey,
    const int* __restrict__ cidx) {
    __shared__ double smv[32];
    // max nA, max nB (order-independent)
    double mA = 0.0, mB = 0.0;
    for (int i = threadIdx.x; i < m; i += blockDim.x) mA = fmax(mA, nA[i]);
    for (int j = threadIdx.x; j < n; j += blockDim.x) mB = fmax(mB, nB[j]);
    mA = block_max(mA, smv);
    mB = block_max(mB, smv);
    if (threadIdx.x == 0) { ctl->nuA = __dsqrt_rn(mA); ctl->nuB = __dsqrt_rn(mB); }
    __syncthreads();
    const double nuA = ctl->nuA, nuB = ctl->nuB;
    if (threadIdx.x >= 1 && threadIdx.x <= OZK_NMAX) ctl->pv[threadIdx.x] = pmax_bits_dev(mt.M[threadIdx.x], nuA, nuB, k);
    __syncthreads();
    const int nonfinite = flag[0] != 0;
    if (nonfinite || force_N > 0) {
        if (threadIdx.x == 0) {
            int N = 0, p = 0, fb = 1;
            if (!nonfinite) {
                p = ctl->pv[force_N];
                fb = 0;
                if (force_p >= 0) { fb = p < force_p; p = min(p, force_p); }
                N = fb ? 0 : force_N;
            }
            dec[0] = N; dec[1] = p; dec[2] = fb; dec[3] = 0;
            *p_dev = p;
            aux[0] = nuA; aux[1] = nuB; aux[2] = 0.0; aux[3] = 0.0; aux[4] = 0.0;
            aux[5] = 0.0; aux[6] = 0.0; aux[7] = 0.0;
            ctl->done = 1;
        }
        return;
    }
    const int hr = min(32, m), hc = min(32, n);
    if (threadIdx.x == 0) {
        ctl->done = 0;
        ctl->nI = nIr + hr;
        ctl->nJ = nJr + hc;
        ctl->preq_max = 1;
        ctl->fin_count = 0u;
        ctl->worst_bits = 0ull;
    }
    // caller-supplied probe indices are clamped into range (an out-of-range index must not be dereferenced)
    for (int x = threadIdx.x; x < nIr; x += blockDim.x) ctl->I[x] = (Ir[x] >= 0 && Ir[x] < m) ? (int)Ir[x] : 0;
    for (int x = threadIdx.x; x < nJr; x += blockDim.x) ctl->J[x] = (Jr[x] >= 0 && Jr[x] < n) ? (int)Jr[x] : 0;
    // the stable top-32 of rows and of columns from the blocks' candidates (hard_cand_kernel)
    __shared__ KeyIdx lists[kPrepThreads];
    const int nbr = hard_blocks(m), nbc = hard_blocks(n);
    unsigned long long key;
    int idx;
    top32([&](int x, unsigned long long& ck, int& ci) { ck = ckey[x]; ci = cidx[x]; }, nbr * 32, lists, key, idx);
    if (threadIdx.x < hr) ctl->I[nIr + threadIdx.x] = idx == kNoIdx ? 0 : idx;
    __syncthreads();
    top32([&](int x, unsigned long long& ck, int& ci) { ck = ckey[(size_t)nbr * 32 + x]; ci = cidx[(size_t)nbr * 32 + x]; },
          nbc * 32, lists, key, idx);
    if (threadIdx.x < hc) ctl->J[nJr + threadIdx.x] = idx == kNoIdx ? 0 : idx;
}

// split-K probe product: partial[b][a][j] = sum over this block's contraction tiles of |A_I[a] l| |B_l J[j]|
// A holds rows [row_begin, row_begin + rows) of the full matrix; probe rows outside it contribute zeros (another
// GPU's block supplies them; the callers sum the D matrices of all blocks)
__global__ void __launch_bounds__(kProbeThreads) probe_partial_kernel(const double* __restrict__ A, const double* __restrict__ B,
                                                                      int row_begin, int rows, int col_begin, int cols,
                                                                      int k,
                                                                      const RuleCtl* __restrict__ ctl,
                                                                      double* __restrict__ partial) {
    if (ctl->done) return;
    __shared__ double sa[kProbeMax][kProbeK + 1];
    __shared__ double sb[kProbeK][kProbeMax];
    __shared__ int sI[kProbeMax], sJ[kProbeMax];
    const int nI = ctl->nI, nJ = ctl->nJ;
    for (int x = threadIdx.x; x < kProbeMax; x += blockDim.x) {
        const int gi = x < nI ? ctl->I[x] - row_begin : -1;
        sI[x] = (gi >= 0 && gi < rows) ? gi : -1;
        const int gj = x < nJ ? ctl->J[x] - col_begin : -1;
        sJ[x] = (gj >= 0 && gj < cols) ? gj : -1;
    }
    const int a0 = (threadIdx.x >> 4) * 6, b0 = (threadIdx.x & 15) * 6;
    double acc[6][6];
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int v = 0; v < 6; v++) acc[u][v] = 0.0;
    const int ntiles = (k + kProbeK - 1) / kProbeK;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int l0 = tile * kProbeK;
        __syncthreads();
        for (int x = threadIdx.x; x < kProbeMax * kProbeK; x += blockDim.x) {
            const int a = x / kProbeK, l = x % kProbeK;
            const int row = sI[a];
            sa[a][l] = (row >= 0 && l0 + l < k) ? fabs(__ldg(A + (size_t)row * k + l0 + l)) : 0.0;
        }
        for (int x = threadIdx.x; x < kProbeMax * kProbeK; x += blockDim.x) {
            const int l = x / kProbeMax, b = x % kProbeMax;
            const int col = sJ[b];
            sb[l][b] = (col >= 0 && l0 + l < k) ? fabs(__ldg(B + (size_t)(l0 + l) * cols + col)) : 0.0;
        }
        __syncthreads();
#pragma unroll 4
        for (int l = 0; l < kProbeK; l++) {
            double av[6], bv[6];
#pragma unroll
            for (int u = 0; u < 6; u++) av[u] = sa[a0 + u][l];
#pragma unroll
            for (int v = 0; v < 6; v++) bv[v] = sb[l][b0 + v];
#pragma unroll
            for (int u = 0; u < 6; u++)
#pragma unroll
                for (int v = 0; v < 6; v++) acc[u][v] = fma(av[u], bv[v], acc[u][v]);
        }
    }
    double* out = partial + (size_t)blockIdx.x * kProbeMax * kProbeMax;
#pragma unroll
    for (int u = 0; u < 6; u++)
#pragma unroll
        for (int v = 0; v < 6; v++) out[(a0 + u) * kProbeMax + b0 + v] = acc[u][v];
}

// D[a][b] = sum of the per-block partials: one block per 32 entries (lane = entry, coalesced), 8 warps over the
// partials (warp w: partials w, w + 8, ...), the warps' sums added in warp order (fixed order: bitwise reproducible)
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(kReduceWarps * 32) probe_reduce_kernel(const double* __restrict__ partial,
                                                                         int nblocks, const RuleCtl* __restrict__ ctl,
                                                                         double* __restrict__ D) {
    if (ctl->done) return;
    __shared__ double sm[kReduceWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int e = blockIdx.x * 32 + lane;              // kProbeMax^2 is a multiple of 32
    double s = 0.0;
    for (int h = w; h < nblocks; h += kReduceWarps) s += partial[(size_t)h * kProbeMax * kProbeMax + e];
    sm[w][lane] = s;
    __syncthreads();
    if (w == 0) {
        double t = 0.0;
#pragma unroll
        for (int u = 0; u < kReduceWarps; u++) t += sm[u][lane];
        D[e] = t;
    }
}

struct EntryTerms { double F1, F2, rhs; };   // rhs = tau * D

__device__ __forceinline__ bool ok_entry(const EntryTerms& t, int p, double safety) {
    const double E = __dadd_rn(__dmul_rn(t.F1, ldexp(1.0, -p)), __dmul_rn(t.F2, ldexp(1.0, -2 * p)));
    return __dmul_rn(E, safety) <= t.rhs;
}

// The rule's last step over the probe entries, one entry per thread on kFinalBlocks blocks.
// rule_preq_kernel: the smallest p of every entry with D > 0 (closed-form start, then the exact comparisons of the
// host rule), the maximum over the entries into ctl->preq_max.
__global__ void __launch_bounds__(kFinalThreads) rule_preq_kernel(
    const int32_t* __restrict__ r, const int32_t* __restrict__ c, const double* __restrict__ sA,
    const double* __restrict__ sB, int k, double tau, double safety, const double* __restrict__ Dg,
    RuleCtl* __restrict__ ctl) {
    if (ctl->done) return;
    __shared__ int s_red[kFinalThreads / 32];
    const int nI = ctl->nI, nJ = ctl->nJ;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    int mx = 1;
    if (e < nI * nJ) {
        const int a = e / nJ, b = e % nJ;
        const double D = Dg[a * kProbeMax + b];
        if (D > 0.0) {
            const int i = ctl->I[a], j = ctl->J[b];
            const int ri = r[i], cj = c[j];
            EntryTerms t;
            t.F1 = __dmul_rn(0.5, __dadd_rn(__dmul_rn(ldexp(1.0, ri), sB[j]), __dmul_rn(ldexp(1.0, cj), sA[i])));
            t.F2 = __dmul_rn(0.25 * (double)k, ldexp(1.0, ri + cj));
            t.rhs = __dmul_rn(tau, D);
            // closed-form start (largest 2^-p meeting E <= tau D / safety), then exact fix-up
            const double cq = tau * D / safety;
            const double xm = 2.0 * cq / (t.F1 + sqrt(t.F1 * t.F1 + 4.0 * t.F2 * cq));
            const double est = ceil(-log2(xm));
            int p = est != est ? 250 : (est < 1.0 ? 1 : (est > 250.0 ? 250 : (int)est));
            while (p > 1 && ok_entry(t, p - 1, safety)) p--;
            while (p < 250 && !ok_entry(t, p, safety)) p++;
            mx = p;
        }
    }
    for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_down_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        int v = 1;
        for (int w = 0; w < kFinalThreads / 32; w++) v = max(v, s_red[w]);
        atomicMax(&ctl->preq_max, v);
    }
}

// rule_final_kernel: the worst E / D at p_req (the host rule's info, :1297-1298), maximum over the entries into
// ctl->worst_bits; the last block to finish (a counter, no waiting) makes the decision: N = the smallest plane count
// in [6, 32] whose pmax_bits reaches p_req, fallback when none does or p_req > 249; it also counts the distinct probe
// rows and columns (the reference reports len(set(I)), len(set(J))) and resets the control fields for another call.
__global__ void __launch_bounds__(kFinalThreads) rule_final_kernel(
    const int32_t* __restrict__ r, const int32_t* __restrict__ c, const double* __restrict__ sA,
    const double* __restrict__ sB, int k, double tau, double safety, const double* __restrict__ Dg,
    RuleCtl* __restrict__ ctl, int32_t* __restrict__ dec, int32_t* __restrict__ p_dev, double* __restrict__ aux) {
    if (ctl->done) return;
    __shared__ double s_redd[kFinalThreads / 32];
    __shared__ int s_last, s_du, s_dv;
    const int nI = ctl->nI, nJ = ctl->nJ;
    const int preq_all = ctl->preq_max;          // written by rule_preq_kernel, earlier on the stream
    const int preq = min(preq_all, 249);
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    double worst = 0.0;
    if (e < nI * nJ) {
        const int a = e / nJ, b = e % nJ;
        const double D = Dg[a * kProbeMax + b];
        if (D > 0.0) {
            const int i = ctl->I[a], j = ctl->J[b];
            const int ri = r[i], cj = c[j];
            const double F1 = __dmul_rn(0.5, __dadd_rn(__dmul_rn(ldexp(1.0, ri), sB[j]), __dmul_rn(ldexp(1.0, cj), sA[i])));
            const double F2 = __dmul_rn(0.25 * (double)k, ldexp(1.0, ri + cj));
            const double E = __dadd_rn(__dmul_rn(F1, ldexp(1.0, -preq)), __dmul_rn(F2, ldexp(1.0, -2 * preq)));
            worst = fmax(worst, __ddiv_rn(E, D));
        }
    }
    for (int o = 16; o > 0; o >>= 1) worst = fmax(worst, __shfl_down_sync(0xffffffffu, worst, o));
    if ((threadIdx.x & 31) == 0) s_redd[threadIdx.x >> 5] = worst;
    __syncthreads();
    if (threadIdx.x == 0) {
        double w = 0.0;
        for (int q = 0; q < kFinalThreads / 32; q++) w = fmax(w, s_redd[q]);
        atomicMax(&ctl->worst_bits, (unsigned long long)__double_as_longlong(w));   // w >= 0: bits order as values
        __threadfence();
        s_last = atomicAdd(&ctl->fin_count, 1u) == gridDim.x - 1 ? 1 : 0;
        s_du = 0;
        s_dv = 0;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (threadIdx.x < nI) {
        const int a = threadIdx.x, v = ctl->I[a];
        bool seen = false;
        for (int b = 0; b < a; b++) seen |= ctl->I[b] == v;
        if (!seen) atomicAdd(&s_du, 1);
    } else if (threadIdx.x >= 128 && threadIdx.x - 128 < nJ) {
        const int a = threadIdx.x - 128, v = ctl->J[a];
        bool seen = false;
        for (int b = 0; b < a; b++) seen |= ctl->J[b] == v;
        if (!seen) atomicAdd(&s_dv, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const double w = __longlong_as_double((long long)atomicAdd(&ctl->worst_bits, 0ull));
        int N = 0, p = 0;
        if (preq_all <= 249) {
            for (int q = 6; q <= OZK_NMAX; q++)
                if (ctl->pv[q] >= preq) { N = q; p = ctl->pv[q]; break; }
        }
        dec[0] = N; dec[1] = p; dec[2] = N == 0; dec[3] = preq;
        *p_dev = p;
        aux[0] = ctl->nuA; aux[1] = ctl->nuB; aux[2] = w;
        aux[3] = (double)s_du; aux[4] = (double)s_dv;
        aux[5] = 0.0; aux[6] = 0.0; aux[7] = 0.0;
        ctl->preq_max = 1;
        ctl->worst_bits = 0ull;
        ctl->fin_count = 0u;
    }
}

int probe_blocks(int k) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // about four contraction tiles per block (each block writes a 96 x 96 partial) once there are enough tiles for
    // 64 blocks, one tile per block below that (short k: latency-bound gathers), at most two blocks per SM
    const int tiles = (k + kProbeK - 1) / kProbeK;
    return max(1, min(min(tiles, 2 * sms), max((tiles + 3) / 4, 64)));
}

size_t ctl_bytes() { return (sizeof(RuleCtl) + 255) & ~(size_t)255; }
size_t cand_count(int m, int n) { return (size_t)(hard_blocks(m) + hard_blocks(n)) * 32; }
// hard-index candidates: keys (8 bytes) then indices (4 bytes)
size_t hard_bytes(int m, int n) { return ((cand_count(m, n) * 12) + 255) & ~(size_t)255; }

// The rule driven by the full-matrix certificate (min xmax over all entries, csrc/certificate.cu) instead of the
// probe: p_req = ceil(-log2(xmin) + 1e-9) clamped to [1, 1000] as the sampled rule clamps it, N = the smallest plane
// count in [6, 32] whose pmax_bits reaches p_req; fallback on non-finite input, no such N, or p_req > 249.
__global__ void __launch_bounds__(kPrepThreads) rule_certified_kernel(
    const double* __restrict__ nA, const double* __restrict__ nB, const int32_t* __restrict__ flag, int m, int n, int k,
    const unsigned long long* __restrict__ xmin, MTable mt, int32_t* __restrict__ dec, int32_t* __restrict__ p_dev,
    double* __restrict__ aux) {
    __shared__ double smv[32];
    __shared__ int pv[OZK_NMAX + 1];
    double mA = 0.0, mB = 0.0;
    for (int i = threadIdx.x; i < m; i += blockDim.x) mA = fmax(mA, nA[i]);
    for (int j = threadIdx.x; j < n; j += blockDim.x) mB = fmax(mB, nB[j]);
    mA = block_max(mA, smv);
    mB = block_max(mB, smv);
    const double nuA = __dsqrt_rn(mA), nuB = __dsqrt_rn(mB);
    if (threadIdx.x >= 1 && threadIdx.x <= OZK_NMAX) pv[threadIdx.x] = pmax_bits_dev(mt.M[threadIdx.x], nuA, nuB, k);
    __syncthreads();
    if (threadIdx.x != 0) return;
    const unsigned long long xb = *xmin;
    const double need = xb == ~0ULL ? -1e30 : -log2(__longlong_as_double((long long)xb));
    double pr = ceil(__dadd_rn(need, 1e-9));
    pr = pr < 1.0 ? 1.0 : (pr > 1000.0 ? 1000.0 : pr);
    const int preq = (int)pr;
    int N = 0;
    for (int t = 6; t <= OZK_NMAX && !N; t++)
        if (pv[t] >= preq) N = t;
    const int fb = (flag[0] != 0 || N == 0 || preq > 249) ? 1 : 0;
    const int p = N ? pv[N] : 0;
    dec[0] = fb ? 0 : N; dec[1] = p; dec[2] = fb; dec[3] = preq;
    *p_dev = p;
    aux[0] = nuA; aux[1] = nuB; aux[2] = need; aux[3] = 0.0; aux[4] = 0.0; aux[5] = 0.0; aux[6] = 0.0; aux[7] = 0.0;
}

}  // namespace

extern "C" size_t ozk_rule_workspace_bytes(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return ctl_bytes() + hard_bytes(m, n) + (size_t)(probe_blocks(k) + 1) * kProbeMax * kProbeMax * sizeof(double);
}

extern "C" size_t ozk_rule_probe_offset(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return ctl_bytes() + hard_bytes(m, n) + (size_t)probe_blocks(k) * kProbeMax * kProbeMax * sizeof(double);
}

extern "C" int ozk_rule_prepare(const int32_t* r, const int32_t* c, const double* sA, const double* nA, const double* sB,
                                const double* nB, const int32_t* flag, int m, int n, int k, const int64_t* probe_rows,
                                int n_probe_rows, const int64_t* probe_cols, int n_probe_cols, int force_N, int force_p,
                                int32_t* dec, int32_t* p_dev, double* aux, void* workspace, size_t workspace_bytes,
                                ozk_stream_t stream_) {
    if (!r || !c || !sA || !nA || !sB || !nB || !flag || !dec || !p_dev || !aux || !workspace) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0) return OZK_ERR_ARG;
    if (force_N != 0 && (force_N < 1 || force_N > OZK_NMAX)) return OZK_ERR_ARG;
    if (force_N == 0) {
        if (n_probe_rows < 0 || n_probe_rows > 64 || n_probe_cols < 0 || n_probe_cols > 64) return OZK_ERR_ARG;
        if ((n_probe_rows && !probe_rows) || (n_probe_cols && !probe_cols)) return OZK_ERR_ARG;
    }
    if (workspace_bytes < ozk_rule_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    MTable mt;
    for (int N = 0; N <= OZK_NMAX; N++) mt.M[N] = N ? ozk_modulus_product(N) : 1.0;
    RuleCtl* ctl = static_cast<RuleCtl*>(workspace);
    unsigned long long* ckey = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) + ctl_bytes());
    int* cidx = reinterpret_cast<int*>(ckey + cand_count(m, n));
    if (force_N == 0) {
        hard_cand_kernel<<<hard_blocks(m) + hard_blocks(n), kHardThreads, 0, st>>>(r, c, sA, sB, m, n, k, ckey, cidx);
        OZK_CHECK_LAUNCH();
    }
    rule_prep_kernel<<<1, kPrepThreads, 0, st>>>(r, c, sA, nA, sB, nB, flag, probe_rows, n_probe_rows, probe_cols,
                                                 n_probe_cols, m, n, k, force_N, force_N > 0 ? force_p : -1, mt, ctl, dec,
                                                 p_dev, aux, ckey, cidx);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_rule_probe_block(const double* A_rows, const double* B_cols, int row_begin, int rows, int col_begin,
                                    int cols, int m, int n, int k, void* workspace, size_t workspace_bytes,
                                    ozk_stream_t stream_) {
    if (!A_rows || !B_cols || !workspace) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0 || rows <= 0 || row_begin < 0 || row_begin + rows > m) return OZK_ERR_ARG;
    if (cols <= 0 || col_begin < 0 || col_begin + cols > n) return OZK_ERR_ARG;
    if (workspace_bytes < ozk_rule_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    RuleCtl* ctl = static_cast<RuleCtl*>(workspace);
    double* partial = reinterpret_cast<double*>(static_cast<char*>(workspace) + ctl_bytes() + hard_bytes(m, n));
    const int nb = probe_blocks(k);
    probe_partial_kernel<<<nb, kProbeThreads, 0, st>>>(A_rows, B_cols, row_begin, rows, col_begin, cols, k, ctl, partial);
    OZK_CHECK_LAUNCH();
    double* D = partial + (size_t)nb * kProbeMax * kProbeMax;
    probe_reduce_kernel<<<kProbeMax * kProbeMax / 32, kReduceWarps * 32, 0, st>>>(partial, nb, ctl, D);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_rule_probe(const double* A_rows, const double* B, int row_begin, int rows, int m, int n, int k,
                              void* workspace, size_t workspace_bytes, ozk_stream_t stream) {
    return ozk_rule_probe_block(A_rows, B, row_begin, rows, 0, n, m, n, k, workspace, workspace_bytes, stream);
}

extern "C" int ozk_rule_finish(const int32_t* r, const int32_t* c, const double* sA, const double* sB, int m, int n,
                               int k, double tau, double safety, int32_t* dec, int32_t* p_dev, double* aux,
                               void* workspace, size_t workspace_bytes, ozk_stream_t stream_) {
    if (!r || !c || !sA || !sB || !dec || !p_dev || !aux || !workspace) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0) return OZK_ERR_ARG;
    if (workspace_bytes < ozk_rule_workspace_bytes(m, n, k)) return OZK_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    RuleCtl* ctl = static_cast<RuleCtl*>(workspace);
    const double* D = reinterpret_cast<const double*>(static_cast<char*>(workspace) + ozk_rule_probe_offset(m, n, k));
    rule_preq_kernel<<<kFinalBlocks, kFinalThreads, 0, st>>>(r, c, sA, sB, k, tau, safety, D, ctl);
    OZK_CHECK_LAUNCH();
    rule_final_kernel<<<kFinalBlocks, kFinalThreads, 0, st>>>(r, c, sA, sB, k, tau, safety, D, ctl, dec, p_dev, aux);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_rule(const double* A, const double* B, int m, int n, int k, const int32_t* r, const int32_t* c,
                        const double* sA, const double* nA, const double* sB, const double* nB, const int32_t* flag,
                        const int64_t* probe_rows, int n_probe_rows, const int64_t* probe_cols, int n_probe_cols,
                        double tau, double safety, int force_N, int force_p, int32_t* dec, int32_t* p_dev, double* aux,
                        void* workspace, size_t workspace_bytes, ozk_stream_t stream) {
    if (!A || !B) return OZK_ERR_ARG;
    int rc = ozk_rule_prepare(r, c, sA, nA, sB, nB, flag, m, n, k, probe_rows, n_probe_rows, probe_cols, n_probe_cols,
                              force_N, force_p, dec, p_dev, aux, workspace, workspace_bytes, stream);
    if (rc != OZK_OK) return rc;
    if ((rc = ozk_rule_probe(A, B, 0, m, m, n, k, workspace, workspace_bytes, stream)) != OZK_OK) return rc;
    return ozk_rule_finish(r, c, sA, sB, m, n, k, tau, safety, dec, p_dev, aux, workspace, workspace_bytes, stream);
}

extern "C" int ozk_rule_certified(const double* nA, const double* nB, const int32_t* flag, int m, int n, int k,
                                  const double* xmin, int32_t* dec, int32_t* p_dev, double* aux, ozk_stream_t stream_) {
    if (!nA || !nB || !flag || !xmin || !dec || !p_dev || !aux) return OZK_ERR_ARG;
    if (m <= 0 || n <= 0 || k <= 0) return OZK_ERR_ARG;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    MTable mt;
    for (int N = 0; N <= OZK_NMAX; N++) mt.M[N] = N ? ozk_modulus_product(N) : 1.0;
    rule_certified_kernel<<<1, kPrepThreads, 0, st>>>(nA, nB, flag, m, n, k,
                                                      reinterpret_cast<const unsigned long long*>(xmin), mt, dec,
                                                      p_dev, aux);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
