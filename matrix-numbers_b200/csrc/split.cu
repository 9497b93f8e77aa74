// Stage 3a: residue split.  FP64 A and B are read once and all N symmetric INT8 residue planes are written in the
// same pass, both K-major (the operand layout of the tcgen05 GEMM).
//
// Semantics (the reference's decomp / resid / resA_k / resB_k, code/ozaki_engine.py:971-1038):
//   x = round(|v| 2^ag) (exact when the shift is to the left, round half away from zero otherwise),
//   X = sign(v) x, residue = X mod m_t mapped to the symmetric range [-floor(m_t/2), ceil(m_t/2) - 1] as int8,
//   with ag = p - r_i + gamma_l for A and ag = p - c_j - gamma_l for B.
//
// Method (this build's own).  Each element becomes a little-endian byte string of KB bytes (KB = 16 for p <= 119,
// 32 for p <= 159): bytes 0 .. KB-2 hold |X| (<= 2^p), one's-complemented when v < 0, and byte KB-1 is a sign flag.
// With weights w_q = 2^(8q) mod m_t for the value bytes and w_(KB-1) = (1 - 2^(8(KB-1))) mod m_t for the flag,
// s_t = sum_q b_q w_q is congruent to X modulo m_t (2^(8(KB-1)) - 1 - |X| + 1 - 2^(8(KB-1)) = -|X| for negative v)
// and lies in [0, 2^21]:
// for a warp chunk of 32 elements the sums of all moduli are one small integer matrix product,
// [16 moduli x KB bytes] x [KB bytes x 32 elements], run as mma.m16n8k16 / m16n8k32 (u8 x u8 -> s32, exact) on the
// byte strings staged in shared memory.  The MMA runs twice, accumulating onto h_t
// (m_t / 2 for m_t = 256, (m_t - 1) / 2 for odd m_t) and onto 0: q = floor((s + h) / m_t) is one multiply-high by
// ceil(2^32 / m_t) (exact for s + h < 2^24), and the low byte of s - m_t q is the symmetric residue -- two integer
// instructions per residue, no per-modulus digit sums and no sign handling.  The element -> MMA column assignment
// gives each thread 8 consecutive elements of a modulus: one 8-byte store.  Moduli beyond the first 16 take a second
// 16-modulus row tile, except for 16 < N <= 20 with 16-byte strings, where the rows of one tile are (chunk, modulus)
// pairs of several chunks (packed_tail) so that few rows stay idle.
#include "ozk_common.cuh"

namespace {

struct SplitTables {
    unsigned W16[OZK_NMAX][4];   // KB = 16: weight bytes packed 4 per word (little-endian)
    unsigned W32[OZK_NMAX][8];   // KB = 32
    unsigned M[OZK_NMAX];        // ceil(2^32 / m_t)
    int P[OZK_NMAX];
};

constexpr int pow2_mod(int e, int P) {
    int w = 1 % P;
    for (int i = 0; i < e; i++) w = (w * 2) % P;
    return w;
}

constexpr SplitTables make_split_tables() {
    SplitTables t{};
    for (int i = 0; i < OZK_NMAX; i++) {
        const int P = ozk_mod(i);
        t.P[i] = P;
        t.M[i] = (unsigned)((0x100000000ULL + (unsigned long long)P - 1ULL) / (unsigned long long)P);
        for (int kb = 16; kb <= 32; kb += 16) {
            for (int q = 0; q < kb; q++) {
                const int w = q < kb - 1 ? pow2_mod(8 * q, P) : (1 + P - pow2_mod(8 * (kb - 1), P)) % P;
                if (kb == 16) t.W16[i][q >> 2] |= (unsigned)w << (8 * (q & 3));
                else t.W32[i][q >> 2] |= (unsigned)w << (8 * (q & 3));
            }
        }
    }
    return t;
}

__constant__ SplitTables c_split = make_split_tables();

#ifndef OZK_SPLIT_MINB
#define OZK_SPLIT_MINB 2   // resident blocks per SM the register budget is sized for
#endif
#ifndef OZK_SPLIT_TC16
#define OZK_SPLIT_TC16 8   // chunks per warp task for 16-byte strings
#endif

constexpr int kWarps = 8;                            // warps per block
constexpr int kRowBytes = 16;                        // 16 bytes of an element's byte string
constexpr int kHalfBytes = 32 * kRowBytes;           // one 16-byte half of the strings of a 32-element chunk
constexpr int kWarpSmem = 8 * (kHalfBytes + 16);     // 8 chunks of KB = 16 (or 4 of KB = 32) per warp, padded

// 64-bit shifts with PTX semantics: amounts at or above 64 (including "negative" ones, as unsigned) give 0
__device__ __forceinline__ unsigned long long shl64(unsigned long long x, unsigned n) {
    unsigned long long r;
    asm("shl.b64 %0, %1, %2;" : "=l"(r) : "l"(x), "r"(n));
    return r;
}
__device__ __forceinline__ unsigned long long shr64(unsigned long long x, unsigned n) {
    unsigned long long r;
    asm("shr.b64 %0, %1, %2;" : "=l"(r) : "l"(x), "r"(n));
    return r;
}

// Byte string of one element as KW 32-bit words (KW = KB / 4).  |v| 2^ag = mant 2^s; X = mant << s for s >= 0,
// round half up of mant 2^s otherwise (x < 2^54 either way), placed as 64-bit limbs
// floor(X / 2^(64 j)) mod 2^64 = (x << (sh - 64 j)) | (x >> (64 j - sh)) with clamped shifts.  A negative v takes
// the one's complement of the value bytes and sets the flag byte; with the flag weight (1 - 2^(8(KB-1))) mod m the
// string is then congruent to -X (for X = 0 too).
template <int KW>
__device__ __forceinline__ void element_words(double v, int ag, unsigned (&w)[KW]) {
    const unsigned hi = (unsigned)__double2hiint(v), lo = (unsigned)__double2loint(v);
    const unsigned E = (hi >> 20) & 0x7FFu;
    const unsigned long long mant = ((unsigned long long)((hi & 0xFFFFFu) | (E ? 0x100000u : 0u)) << 32) | lo;
    const int s = (int)(E ? E : 1u) - 1075 + ag;
    const unsigned long long xr = (shr64(mant, (unsigned)(-s - 1)) + 1ULL) >> 1;   // s < 0: below 2^54, one limb
#pragma unroll
    for (int j = 0; j < KW / 2; j++) {
        unsigned long long limb = shl64(mant, (unsigned)(s - 64 * j)) | shr64(mant, (unsigned)(64 * j - s));
        if (j == 0) limb = s < 0 ? xr : limb;
        else limb = s < 0 ? 0ULL : limb;
        w[2 * j] = (unsigned)limb;
        w[2 * j + 1] = (unsigned)(limb >> 32);
    }
    const unsigned msk = (unsigned)((int)hi >> 31);
#pragma unroll
    for (int i = 0; i < KW; i++) w[i] ^= msk;
    w[KW - 1] = (w[KW - 1] & 0x00FFFFFFu) | ((hi >> 7) & 0x01000000u);
}

// Shared-memory row of element e (0..31) of a chunk: the fragments of n-tile j come from rows 8j .. 8j+7, and row
// 8j + (c ^ 2j) holds element 8(c >> 1) + 2j + (c & 1), so that the MMA column pairs (2 tig, 2 tig + 1) of the four
// n-tiles are elements 8 tig .. 8 tig + 7.  The XOR keeps both the row writes of 8 consecutive elements and the 8
// rows of an n-tile on distinct 16-byte bank groups.
__device__ __forceinline__ int row_of_element(int e) {
    const int j = (e >> 1) & 3;
    return 8 * j + (((e & 1) + 2 * (e >> 3)) ^ (2 * j));
}

__device__ __forceinline__ void mma_k16(int (&d)[4], const unsigned* a, unsigned b0, int cA, int cB) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %8, %9, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(b0), "r"(cA), "r"(cA), "r"(cB), "r"(cB));
}

__device__ __forceinline__ void mma_k32(int (&d)[4], const unsigned* a, unsigned b0, unsigned b1, int cA, int cB) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %11, %12, %13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(cA), "r"(cA), "r"(cB), "r"(cB));
}

// d += A B (m16n8k32, u8 x u8 -> s32), the accumulator carried in d
__device__ __forceinline__ void mma_k32_acc(int (&d)[4], const unsigned* a, unsigned b0, unsigned b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per-lane constants of one row tile: the moduli of rows g and g + 8 of lane (g, tig) -- t0 + g and t0 + g + 8 for a
// 16-modulus tile, or the pair chosen by the packed tail below.  The lane-dependent indices into constant memory are
// read once per thread.
template <int KB>
struct TileConsts {
    unsigned a[KB / 8];   // A fragment: {row g, row g+8} of bytes 4 tig .. 4 tig + 3 (k32: and 16 + 4 tig ..)
    unsigned MA, MB, nPA, nPB;
    __device__ __forceinline__ void init(int t0) {
        const int g = (threadIdx.x & 31) >> 2;
        init_rows(t0 + g, t0 + g + 8);
    }
    __device__ __forceinline__ void init_rows(int tA, int tB) {   // tA, tB < 32 = OZK_NMAX
        const int tig = threadIdx.x & 3;
        if (KB == 16) {
            a[0] = c_split.W16[tA][tig];
            a[1] = c_split.W16[tB][tig];
        } else {
            a[0] = c_split.W32[tA][tig];
            a[1] = c_split.W32[tB][tig];
            a[2] = c_split.W32[tA][4 + tig];
            a[3] = c_split.W32[tB][4 + tig];
        }
        MA = c_split.M[tA];
        MB = c_split.M[tB];
        nPA = 0u - (unsigned)c_split.P[tA];
        nPB = 0u - (unsigned)c_split.P[tB];
    }
};

// s - m floor((s + h) / m) in [-128, 127], from sh = s + h and s
__device__ __forceinline__ int residue(int sh, int s, unsigned M, unsigned nP) {
    return (int)(__umulhi((unsigned)sh, M) * nP + (unsigned)s);
}

// four residues in [-128, 127] as the bytes (r0, r1, r2, r3) of a word
__device__ __forceinline__ unsigned pack_s8(int r0, int r1, int r2, int r3) {
    unsigned hi, w;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(r3), "r"(r2));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(r1), "r"(r0), "r"(hi));
    return w;
}

// B fragments of a chunk (32 elements, byte strings at `chunk` in shared memory): for n-tile j, lane (g, tig) needs
// word tig of element 8(g >> 1) + 2j + (g & 1), stored in row 8j + (g ^ 2j) (k 0-15; k 16-31 in the second half).
// Plain 32-bit shared loads (a warp reads 8 whole rows, conflict-free), which the compiler can schedule freely.
template <int KB>
__device__ __forceinline__ void chunk_fragments(const unsigned char* chunk, unsigned (&b)[KB / 4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const unsigned* row = reinterpret_cast<const unsigned*>(chunk + (8 * j + (g ^ (2 * j))) * kRowBytes);
        b[j] = row[tig];
        if (KB == 32) b[4 + j] = row[kHalfBytes / 4 + tig];
    }
}

// Residues of one chunk for the 16 moduli of a row tile; row A of lane (g, tig) is modulus t0 + g, row B modulus
// t0 + g + 8.  `o` points at byte 8 tig of the chunk in plane 0.  Each pair of n-tiles gives one packed word per
// row, so few products are live at a time.
template <int KB>
__device__ __forceinline__ void chunk_residues(const unsigned (&b)[KB / 4], const TileConsts<KB>& tc, int t0, int N,
                                               int8_t* o, size_t plane_bytes) {
    const int g = (threadIdx.x & 31) >> 2;
    const bool needB = t0 + 8 < N;   // warp-uniform
    const int hA = (int)((0u - tc.nPA) >> 1), hB = (int)((0u - tc.nPB) >> 1);   // floor(m / 2)
    unsigned wA[2], wB[2];
#pragma unroll
    for (int half = 0; half < 2; half++) {
        int rA[4], rB[4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int nt = 2 * half + u;
            int d1[4], d0[4];
            if (KB == 16) {
                mma_k16(d1, tc.a, b[nt], hA, hB);
                mma_k16(d0, tc.a, b[nt], 0, 0);
            } else {
                mma_k32(d1, tc.a, b[nt], b[4 + nt], hA, hB);
                mma_k32(d0, tc.a, b[nt], b[4 + nt], 0, 0);
            }
            rA[2 * u] = residue(d1[0], d0[0], tc.MA, tc.nPA);
            rA[2 * u + 1] = residue(d1[1], d0[1], tc.MA, tc.nPA);
            rB[2 * u] = needB ? residue(d1[2], d0[2], tc.MB, tc.nPB) : 0;
            rB[2 * u + 1] = needB ? residue(d1[3], d0[3], tc.MB, tc.nPB) : 0;
        }
        wA[half] = pack_s8(rA[0], rA[1], rA[2], rA[3]);
        wB[half] = pack_s8(rB[0], rB[1], rB[2], rB[3]);
    }
    const int tA = t0 + g, tB = tA + 8;
    if (tA < N) *reinterpret_cast<uint2*>(o + (size_t)tA * plane_bytes) = make_uint2(wA[0], wA[1]);
    if (needB && tB < N) *reinterpret_cast<uint2*>(o + (size_t)tB * plane_bytes) = make_uint2(wB[0], wB[1]);
}

// Moduli 16 .. N-1 for 16 < N <= 20 (16-byte strings): a 16-row tile of one chunk would leave most rows idle, so
// the rows are (chunk, modulus) pairs instead -- G chunks x E = 16 / G moduli (G = 8 for N <= 18, 4 for N <= 20).
// Row g (and g + 8) of lane (g, tig) is chunk c = g % G of the group with modulus 16 + g / G (and 16 + g / G + 8 / G);
// its weights are non-zero only on the k-half of m16n8k32 product q that holds chunk c's string (chunks 2q and
// 2q + 1 fill k 0-15 and 16-31), so the G / 2 products of a chain sum exactly each row's own chunk.  One chain per
// n-tile, accumulated onto 0; h is added on the integer pipe.  `pc` holds the lane's two moduli (init_rows).
template <int G>
__device__ __forceinline__ void packed_tail(const unsigned char* wsm, int chunk_bytes, const TileConsts<16>& pc,
                                            int N, int cnt, int8_t* o0, size_t chunk_stride, size_t plane_bytes) {
    const int g = (threadIdx.x & 31) >> 2;
    const int c = g % G, tA = 16 + g / G, tB = tA + 8 / G;
    const int hA = (int)((0u - pc.nPA) >> 1), hB = (int)((0u - pc.nPB) >> 1);
    const int tig = threadIdx.x & 3;
#pragma unroll
    for (int grp = 0; grp < 8 / G; grp++) {
        unsigned wA[2], wB[2];
#pragma unroll
        for (int half = 0; half < 2; half++) {          // n-tiles 2 half and 2 half + 1: few live accumulators
            int d[2][4];
#pragma unroll
            for (int q = 0; q < G / 2; q++) {
                const bool mine = (c >> 1) == q, odd = (c & 1) != 0;
                const unsigned a[4] = {mine && !odd ? pc.a[0] : 0u, mine && !odd ? pc.a[1] : 0u,
                                       mine && odd ? pc.a[0] : 0u, mine && odd ? pc.a[1] : 0u};
                const unsigned char* c0 = wsm + (grp * G + 2 * q) * chunk_bytes;
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int j = 2 * half + u;          // the n-tile's word tig of element row 8j + (g ^ 2j)
                    const int roff = (8 * j + (g ^ (2 * j))) * kRowBytes + 4 * tig;
                    const unsigned b0 = *reinterpret_cast<const unsigned*>(c0 + roff);
                    const unsigned b1 = *reinterpret_cast<const unsigned*>(c0 + chunk_bytes + roff);
                    if (q == 0) mma_k32(d[u], a, b0, b1, 0, 0);
                    else mma_k32_acc(d[u], a, b0, b1);
                }
            }
            int rA[4], rB[4];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                rA[2 * u] = residue(d[u][0] + hA, d[u][0], pc.MA, pc.nPA);
                rA[2 * u + 1] = residue(d[u][1] + hA, d[u][1], pc.MA, pc.nPA);
                rB[2 * u] = residue(d[u][2] + hB, d[u][2], pc.MB, pc.nPB);
                rB[2 * u + 1] = residue(d[u][3] + hB, d[u][3], pc.MB, pc.nPB);
            }
            wA[half] = pack_s8(rA[0], rA[1], rA[2], rA[3]);
            wB[half] = pack_s8(rB[0], rB[1], rB[2], rB[3]);
        }
        const int ch = grp * G + c;
        if (ch < cnt) {
            int8_t* o = o0 + (size_t)ch * chunk_stride;
            if (tA < N) *reinterpret_cast<uint2*>(o + (size_t)tA * plane_bytes) = make_uint2(wA[0], wA[1]);
            if (tB < N) *reinterpret_cast<uint2*>(o + (size_t)tB * plane_bytes) = make_uint2(wB[0], wB[1]);
        }
    }
}

// One kernel for both operands.  A "vector" v is a row of A (v = i) or a column of B (v = j); its elements are
// indexed by the contraction index l and its planes are out[t][v][l] (K-major).  A chunk is 32 consecutive l of one
// vector (k % 32 == 0).  A warp task is TC chunks (TC = 8 for KB = 16, 4 for KB = 32), loaded with TC independent
// 8-byte loads per lane:
//   A: TC consecutive chunks of the row-major (v, l-block) order -- chunk ch covers A elements 32 ch .. 32 ch + 31
//      and plane bytes 32 ch .. 32 ch + 31; lane L loads element L of each chunk (coalesced);
//   B: TC adjacent columns of one l-block; lane (rg, c) = (lane / TC, lane % TC) loads rows TC rg + i (i < TC) of
//      column c, so that each load instruction reads whole sectors.  Tasks run along l first, so the warps of a
//      block write adjacent pieces of the same plane rows.
template <int KB, bool IS_B, bool PACKED>
__device__ __forceinline__ void split_tasks(const double* __restrict__ src, const int32_t* __restrict__ vexp,
                                            const int32_t* __restrict__ gam, int p, int V, int k, int N,
                                            int8_t* __restrict__ out, unsigned char* wsm) {
    constexpr int TC = KB == 16 ? OZK_SPLIT_TC16 : 4;     // chunks per task
    constexpr int KW = KB / 4;               // words per byte string
    constexpr int kChunkBytes = (KB / 16) * kHalfBytes + 16;
    const int lane = threadIdx.x & 31, tig = lane & 3;
    const int lblocks = k >> 5;
    const size_t plane_bytes = (size_t)V * (size_t)k;
    // chunk and task counts fit in 31 bits (checked on the host)
    const int nchunks = V * lblocks;
    const int ntasks = IS_B ? (V / TC) * lblocks : (nchunks + TC - 1) / TC;
    const int gwarp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * blockDim.x) >> 5);
    // moduli 16 .. N-1: a second 16-modulus tile per chunk, or for 16 < N <= 20 the packed tail (16-byte strings;
    // a separate instantiation, launched only for those N, so that the common path keeps its register budget)
    constexpr bool packed = PACKED && KB == 16;
    TileConsts<KB> tc0, tc1;
    tc0.init(0);
    if constexpr (packed) {
        const int g = lane >> 2, G = N <= 18 ? 8 : 4;
        tc1.init_rows(16 + g / G, 16 + g / G + 8 / G);
    } else {
        tc1.init(16);
    }
    // task coordinates, advanced by the grid stride without divisions in the loop:
    //   A: (v, lb) of the task's first chunk;  B: (vector group, l-block)
    //   B: consecutive warps take the two column groups of a pair (one 128-byte line of a row of B for TC = 8) at
    //   the same l-block, then the pair moves along l; the warp count is even, so a warp keeps its half
    const int step = IS_B ? (nwarps >> 1) : nwarps * TC;
    const int first = IS_B ? (gwarp >> 1) : gwarp * TC;
    const int bhalf = IS_B ? (gwarp & 1) : 0;
    int tv = first / lblocks;
    int clb = first - tv * lblocks;
    const int sv = step / lblocks;
    const int slb = step - sv * lblocks;
    for (int task = gwarp; task < ntasks; task += nwarps) {
        const int cv = IS_B ? 2 * tv + bhalf : tv;
        double x[TC];
        int ag[TC];
        int cnt = TC;
        if (!IS_B) {
            const int ch0 = task * TC;
            cnt = nchunks - ch0 < TC ? nchunks - ch0 : TC;
            int v = cv;
            int lb = clb;
#pragma unroll
            for (int i = 0; i < TC; i++) {
                if (i < cnt) {
                    const int l = 32 * lb + lane;
                    x[i] = __ldg(src + (size_t)(ch0 + i) * 32 + lane);
                    ag[i] = p - __ldg(vexp + v) + __ldg(gam + l);
                } else {
                    x[i] = 0.0;
                    ag[i] = 0;
                }
                if (++lb == lblocks) { lb = 0; v++; }
            }
        } else {
            const int c = lane % TC, rg = lane / TC;
            const int v = cv * TC + c;
            const int cexp = p - __ldg(vexp + v);
#pragma unroll
            for (int i = 0; i < TC; i++) {
                const int l = 32 * clb + TC * rg + i;
                x[i] = __ldg(src + (size_t)l * V + v);
                ag[i] = cexp - __ldg(gam + l);
            }
        }
        __syncwarp();   // the previous task's fragment reads are done before the strings are overwritten
#pragma unroll
        for (int i = 0; i < TC; i++) {
            unsigned w[KW];
            element_words<KW>(x[i], ag[i], w);
            const int chunk = IS_B ? lane % TC : i;
            const int e = IS_B ? TC * (lane / TC) + i : lane;
            unsigned char* row = wsm + chunk * kChunkBytes + row_of_element(e) * kRowBytes;
            *reinterpret_cast<uint4*>(row) = make_uint4(w[0], w[1], w[2], w[3]);
            if (KB == 32) *reinterpret_cast<uint4*>(row + kHalfBytes) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < TC; i++) {
            if (i < cnt) {
                int8_t* o = IS_B ? out + (size_t)(cv * TC + i) * k + 32 * clb + 8 * tig
                                 : out + (size_t)(task * TC + i) * 32 + 8 * tig;
                unsigned b[KB / 4];
                chunk_fragments<KB>(wsm + i * kChunkBytes, b);
                chunk_residues<KB>(b, tc0, 0, N, o, plane_bytes);
                if (N > 16 && !packed) chunk_residues<KB>(b, tc1, 16, N, o, plane_bytes);
            }
        }
        if constexpr (packed) {
            int8_t* o0 = IS_B ? out + (size_t)(cv * TC) * k + 32 * clb + 8 * tig : out + (size_t)task * TC * 32 + 8 * tig;
            const size_t stride = IS_B ? (size_t)k : (size_t)32;
            if (N <= 18) packed_tail<8>(wsm, kChunkBytes, tc1, N, cnt, o0, stride, plane_bytes);
            else packed_tail<4>(wsm, kChunkBytes, tc1, N, cnt, o0, stride, plane_bytes);
        }
        tv += sv;
        clb += slb;
        if (clb >= lblocks) { clb -= lblocks; tv++; }
    }
}

template <bool IS_B, bool PACKED>
__global__ void __launch_bounds__(kWarps * 32, OZK_SPLIT_MINB) split_kernel(const double* __restrict__ src,
                                                               const int32_t* __restrict__ vexp,
                                                               const int32_t* __restrict__ gam,
                                                               const int32_t* __restrict__ p_dev, int V, int k, int N,
                                                               int8_t* __restrict__ out, int p_lo) {
    __shared__ __align__(16) unsigned char strings[kWarps][kWarpSmem];
    const int p = *p_dev;
    if (p < p_lo) return;   // split_tc.cu's kernel has produced the planes
    unsigned char* wsm = strings[threadIdx.x >> 5];
    if (p <= 119) split_tasks<16, IS_B, PACKED>(src, vexp, gam, p, V, k, N, out, wsm);
    else split_tasks<32, IS_B, false>(src, vexp, gam, p, V, k, N, out, wsm);
}

int split_blocks(long long tasks) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = (tasks + kWarps - 1) / kWarps;
    const long long cap = 8LL * sms;
    return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

// split_tc.cu: the tensor-core split for p <= 119 on the shapes it takes; *p_lo = 120 when it was launched
int ozk_split_tc_launch(int is_b, const double* src, const int32_t* vexp, const int32_t* gam, const int32_t* p_dev,
                        int V, int k, int N, int8_t* out, int32_t* err, cudaStream_t st, int* p_lo);

// Both kernels are launched: the tensor-core one returns at once for p > 119 and this one for p < p_lo, so that the
// choice follows the device-side p (graph capture included).
extern "C" int ozk_split_a(const double* A, const int32_t* r, const int32_t* gam, const int32_t* p_dev, int m, int k,
                           int N, int8_t* Ares, int32_t* err, ozk_stream_t stream_) {
    if (!A || !r || !gam || !p_dev || !Ares || !err) return OZK_ERR_ARG;
    if (m <= 0 || k <= 0 || (k & 31) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(Ares)) & 15) return OZK_ERR_ARG;
    if ((long long)m * (k >> 5) >= 0x7fffffffLL - (1LL << 24)) return OZK_ERR_ARG;   // chunk indices in 31 bits
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    int p_lo = 0;
    const int rc = ozk_split_tc_launch(0, A, r, gam, p_dev, m, k, N, Ares, err, st, &p_lo);
    if (rc != OZK_OK) return rc;
    const long long tasks = ((long long)m * (k >> 5) + 7) / 8;
    if (N > 16 && N <= 20)
        split_kernel<false, true><<<split_blocks(tasks), kWarps * 32, 0, st>>>(A, r, gam, p_dev, m, k, N, Ares, p_lo);
    else
        split_kernel<false, false><<<split_blocks(tasks), kWarps * 32, 0, st>>>(A, r, gam, p_dev, m, k, N, Ares, p_lo);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}

extern "C" int ozk_split_b(const double* B, const int32_t* c, const int32_t* gam, const int32_t* p_dev, int k, int n,
                           int N, int8_t* Bres, int32_t* err, ozk_stream_t stream_) {
    if (!B || !c || !gam || !p_dev || !Bres || !err) return OZK_ERR_ARG;
    if (n <= 0 || k <= 0 || (k & 31) || (n & 31) || N < 1 || N > OZK_NMAX) return OZK_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(Bres) & 15) return OZK_ERR_ARG;
    if ((long long)n * (k >> 5) >= 0x7fffffffLL - (1LL << 24)) return OZK_ERR_ARG;   // chunk indices in 31 bits
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream_);
    int p_lo = 0;
    const int rc = ozk_split_tc_launch(1, B, c, gam, p_dev, n, k, N, Bres, err, st, &p_lo);
    if (rc != OZK_OK) return rc;
    const long long tasks = (long long)(n / 8) * (k >> 5);
    if (N > 16 && N <= 20)
        split_kernel<true, true><<<split_blocks(tasks), kWarps * 32, 0, st>>>(B, c, gam, p_dev, n, k, N, Bres, p_lo);
    else
        split_kernel<true, false><<<split_blocks(tasks), kWarps * 32, 0, st>>>(B, c, gam, p_dev, n, k, N, Bres, p_lo);
    OZK_CHECK_LAUNCH();
    return OZK_OK;
}
