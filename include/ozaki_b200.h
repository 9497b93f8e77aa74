/*
 * ozaki_b200.h -- C ABI of the B200 (sm_100a) FP64-on-INT8 (Ozaki-II / CRT) GEMM engine, libozaki_b200.so.
 *
 * The engine computes C = A B for float64 A (m x k, row-major) and B (k x n, row-major) from N exact INT8
 * residue-plane products and a Chinese-Remainder reconstruction, with the moduli set, scaling, plane-count
 * rule and rounding of the reference engine dl1683/matrix-numbers, code/ozaki_engine.py (citations below are
 * file:line in that file).  The reference binds its GPU path through ctypes (ozaki_engine.py:20-229); these
 * entry points replace the calls it makes there, one C function per reference stage.
 *
 * Conventions (all entry points):
 *   - pointers are CUDA device pointers of the current device unless stated otherwise; the caller owns every
 *     buffer, and no entry point allocates device memory;
 *   - `stream` is a cudaStream_t (a CUstream handle; NULL = the legacy default stream); work is enqueued, never
 *     synchronised, so every entry point may be captured in a CUDA graph;
 *   - the return value is OZK_OK (0) or an error code (ozk_error_string); an error is returned before any
 *     launch when an argument is invalid;
 *   - device-side failures (a bounded wait that ran out) are reported through the `err` word of the GEMM
 *     entry points (bit flags OZK_DEVERR_*), which the caller reads after its next synchronisation.
 *
 * Shape rules (the reference's, ozaki_engine.py:1315-1316, except the k bound): m % 4 == 0, n % 32 == 0,
 * k % 32 == 0, m, n, k > 0.  k has no upper bound here: the products accumulate exactly in segments of 65536
 * (INT32 cannot overflow inside a segment) and the segments are combined modulo each modulus.
 */
#ifndef OZAKI_B200_H
#define OZAKI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* ozk_stream_t;

#define OZK_OK 0
#define OZK_ERR_ARG (-1)          /* invalid shape, alignment, null pointer or out-of-range count           */
#define OZK_ERR_P_RANGE (-2)      /* scaling bits p outside [0, 159]                                        */
#define OZK_ERR_DEVICE (-3)       /* no CUDA device, or the device is not sm_100                            */
#define OZK_ERR_DRIVER (-4)       /* driver entry point or TMA tensor-map encoding failed                   */
#define OZK_ERR_WORKSPACE (-5)    /* workspace smaller than the *_workspace_bytes query                     */
#define OZK_ERR_TOO_LARGE (-6)    /* problem needs more scratch than ozk_stats_noalloc's static array holds  */
#define OZK_ERR_CUDA_BASE 1000    /* OZK_ERR_CUDA_BASE + cudaError_t of a failed launch or attribute call  */

#define OZK_DEVERR_TIMEOUT_PRODUCER 1   /* GEMM: the TMA producer's bounded wait ran out   */
#define OZK_DEVERR_TIMEOUT_MMA 2        /* GEMM: the MMA issuer's bounded wait ran out     */
#define OZK_DEVERR_TIMEOUT_EPILOGUE 4   /* GEMM: an epilogue warp's bounded wait ran out   */
#define OZK_DEVERR_TIMEOUT_RECON 8      /* reconstruction: a bounded wait (TMA or MMA) ran out */
#define OZK_DEVERR_TIMEOUT_SPLIT 16     /* residue split: a bounded wait (TMA or MMA) ran out  */

/* ---- library information -------------------------------------------------------------------------------- */
int ozk_version(void);
const char* ozk_error_string(int code);
/* number of SMs of the current device (the persistent GEMM's grid); OZK_ERR_DEVICE without a device */
int ozk_device_sm_count(int* out);

/* ---- host helpers (no device work) ----------------------------------------------------------------------- */
/* modulus t of the fixed list 256, 255, 253, ... 107 (ozaki_engine.py:824-825); 0 outside [0, 32) */
int ozk_modulus(int t);
/* float(prod of the first N moduli), correctly rounded (the Mvec of ozaki_engine.py:1160) */
double ozk_modulus_product(int N);
/* limb count ceil(bits(prod m)/32), at least 2 (ozaki_engine.py:1104-1106) */
int ozk_limbs_for(int N);
/* largest p in [0, 249] with 2 Xmax(p) + 1 <= M_N (ozaki_engine.py:1119-1139) */
int ozk_pmax_bits(int N, double nuA, double nuB, int k);

/* ---- stage 1: statistics (replaces OzakiCRT.stats, ozaki_engine.py:1229-1247 with kernels :846-951) ------ *
 * gam[k]: inside scaling gamma_l (0 when inside == 0); r[m], sA[m], nA[m]: row exponent and sums of A;
 * c[n], sB[n], nB[n]: column exponent (0 for an all-zero column) and sums of B; flag[1]: 1 if a non-finite
 * value was seen.  Sums are reduced in a fixed order (bitwise reproducible run to run).                    */
size_t ozk_stats_workspace_bytes(int m, int n, int k);
int ozk_stats(const double* A, const double* B, int m, int n, int k, int inside, int32_t* gam, int32_t* r,
              int32_t* c, double* sA, double* nA, double* sB, double* nB, int32_t* flag, void* workspace,
              size_t workspace_bytes, ozk_stream_t stream);

/* Stage 1 in two phases, for C row blocks spread over several GPUs (the column max of |A| is all-reduced with MAX
 * between them): colmax[k] = max_i |A_il| as IEEE bit patterns (the reference's colmax_k, :847-854), then the rest
 * of stage 1 given the (global) colmax.  ozk_stats == ozk_stats_colmax + ozk_stats_finish.                  */
int ozk_stats_colmax(const double* A, int m, int k, uint64_t* colmax, ozk_stream_t stream);
int ozk_stats_finish(const double* A, const double* B, int m, int n, int k, int inside, const uint64_t* colmax,
                     int32_t* gam, int32_t* r, int32_t* c, double* sA, double* nA, double* sB, double* nB,
                     int32_t* flag, void* workspace, size_t workspace_bytes, ozk_stream_t stream);

/* Stage 1 in pieces, for a 2-D grid of C blocks over several GPUs (row blocks of A x column blocks of B; the
 * maxima are all-reduced with MAX between the ranks before gamma):
 *   ozk_stats_rowmax: rowmax[k] = max_j |B_lj| over this rank's columns (B_cols: k x n, row-major), as IEEE bit
 *                     patterns (the reference's rowmax_k, :856-868);
 *   ozk_stats_gamma:  gamma[k] and the non-finite flag from the (global) colmax and rowmax (gamma_k, :870-879);
 * then ozk_stats_rows / ozk_stats_cols below for this rank's rows of A and columns of B.                    */
int ozk_stats_rowmax(const double* B_cols, int k, int n, uint64_t* rowmax, ozk_stream_t stream);
int ozk_stats_gamma(const uint64_t* colmax, const uint64_t* rowmax, int k, int inside, int32_t* gam, int32_t* flag,
                    ozk_stream_t stream);

/* One operand's statistics for a given gamma[k] (inside scaling already decided), for the persistent fixed
 * operand mode (the reference's PersistA, ozaki_engine.py:2417-2466, which launches rowstatsA_k alone in encode,
 * :2433-2442, and colexpB_k + colsumsB_k alone in _stats_B, :2444-2454, with gamma = 0):
 *   ozk_stats_rows: r[m], sA[m], nA[m] of A (rowstatsA_k, :904-925);
 *   ozk_stats_cols: c[n], sB[n], nB[n] of B (colexpB_k + colsumsB_k, :926-951), scratch of
 *                   ozk_stats_cols_workspace_bytes(k, n) bytes (ozk_stats_workspace_bytes(m, n, k) is enough).
 * Outputs equal those of ozk_stats for the same gamma.                                                       */
int ozk_stats_rows(const double* A, int m, int k, const int32_t* gam, int32_t* r, double* sA, double* nA,
                   ozk_stream_t stream);
size_t ozk_stats_cols_workspace_bytes(int k, int n);
int ozk_stats_cols(const double* B, int k, int n, const int32_t* gam, int32_t* c, double* sB, double* nB,
                   void* workspace, size_t workspace_bytes, ozk_stream_t stream);

/* Stage 1 without a workspace argument, for callers that cannot allocate device memory (they only hold device
 * pointers handed to them by another runtime, or must not call cudaMalloc while they run or record a CUDA graph).
 * This entry point has no counterpart in the reference.  Its scratch is a static device array of
 * OZK_STATS_NOALLOC_MAX_BYTES (16 MiB) inside the library, held on every device that loads the library until the
 * process exits; a problem with ozk_stats_workspace_bytes(m, n, k) above that size is rejected with
 * OZK_ERR_TOO_LARGE before any launch (16 MiB covers m, n, k <= 16384 and m = n = 32768 with k = 8192).  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress) and must therefore come before any
 * stream capture on that device.  All calls share the array: calls whose work overlaps on the GPU race, so the
 * caller serialises them (one stream, or an event between streams).  Outputs equal ozk_stats's.             */
#define OZK_STATS_NOALLOC_MAX_BYTES (16u << 20)
int ozk_stats_noalloc(const double* A, const double* B, int m, int n, int k, int inside, int32_t* gam, int32_t* r,
                      int32_t* c, double* sA, double* nA, double* sB, double* nB, int32_t* flag, ozk_stream_t stream);

/* ---- stage 2: the a-priori plane-count rule on the device (replaces OzakiCRT.choose, ozaki_engine.py:
 * 1250-1307, and OzakiCRT._rule_device, :1372-1426).  probe_rows / probe_cols: the random part of the probe
 * set (RandomState(seed).choice, :1265-1267), device int64; the 32 "hard" rows and columns are added on the
 * device.  dec[4] = {N (0 on fallback), p, fallback, p_req}; p_dev[1] = p (read by the later stages, so that a
 * captured graph does not depend on p); aux[8] = {nuA, nuB, worst E/D at p_req, distinct probe rows, distinct
 * probe columns, 0, 0, 0}.  force_N > 0 skips the probe (N = force_N, p = pmax_bits); force_p >= 0 with
 * force_N caps p and flags fallback when the data allow less (ozaki_engine.py:1389-1396, :1492-1498).      */
size_t ozk_rule_workspace_bytes(int m, int n, int k);
int ozk_rule(const double* A, const double* B, int m, int n, int k, const int32_t* r, const int32_t* c,
             const double* sA, const double* nA, const double* sB, const double* nB, const int32_t* flag,
             const int64_t* probe_rows, int n_probe_rows, const int64_t* probe_cols, int n_probe_cols, double tau,
             double safety, int force_N, int force_p, int32_t* dec, int32_t* p_dev, double* aux, void* workspace,
             size_t workspace_bytes, ozk_stream_t stream);

/* Stage 2 in three phases, for C row blocks spread over several GPUs: ozk_rule == prepare + probe + finish.
 * prepare: nu, pv, forced / non-finite decisions and the probe sets (r, sA, nA over ALL m rows);
 * probe:   the probe product D = |A_I| |B_J| restricted to the probe rows inside [row_begin, row_begin + rows),
 *          A_rows pointing at that row block (other rows give 0); D (96 x 96 doubles, row-major, padded) sits at
 *          byte offset ozk_rule_probe_offset() of the workspace, where the callers sum the blocks' D matrices;
 * finish:  p_req, N, p and the outputs of ozk_rule from D.                                                    */
size_t ozk_rule_probe_offset(int m, int n, int k);
int ozk_rule_prepare(const int32_t* r, const int32_t* c, const double* sA, const double* nA, const double* sB,
                     const double* nB, const int32_t* flag, int m, int n, int k, const int64_t* probe_rows,
                     int n_probe_rows, const int64_t* probe_cols, int n_probe_cols, int force_N, int force_p,
                     int32_t* dec, int32_t* p_dev, double* aux, void* workspace, size_t workspace_bytes,
                     ozk_stream_t stream);
int ozk_rule_probe(const double* A_rows, const double* B, int row_begin, int rows, int m, int n, int k,
                   void* workspace, size_t workspace_bytes, ozk_stream_t stream);
/* The probe product for the rows [row_begin, row_begin + rows) of A and the columns [col_begin, col_begin +
 * cols) of B held by one rank (B_cols: k x cols, row-major); entries outside the block are zero, the callers sum
 * the D matrices of all blocks.  ozk_rule_probe == ozk_rule_probe_block with the full column range.          */
int ozk_rule_probe_block(const double* A_rows, const double* B_cols, int row_begin, int rows, int col_begin, int cols,
                         int m, int n, int k, void* workspace, size_t workspace_bytes, ozk_stream_t stream);
int ozk_rule_finish(const int32_t* r, const int32_t* c, const double* sA, const double* sB, int m, int n, int k,
                    double tau, double safety, int32_t* dec, int32_t* p_dev, double* aux, void* workspace,
                    size_t workspace_bytes, ozk_stream_t stream);

/* ---- stage 3a: residue split (replaces resA_k / resB_k, ozaki_engine.py:996-1038 and :1328-1331) --------- *
 * Ares[t][i][l] = symmetric residue of round(A_il 2^(p - r_i + gam_l)) modulo m_t, t < N, as int8;
 * Bres[t][j][l] = the same for B_lj 2^(p - c_j - gam_l), contraction index contiguous (K-major planes).     */
int ozk_split_a(const double* A, const int32_t* r, const int32_t* gam, const int32_t* p_dev, int m, int k, int N,
                int8_t* Ares, int32_t* err, ozk_stream_t stream);
int ozk_split_b(const double* B, const int32_t* c, const int32_t* gam, const int32_t* p_dev, int k, int n, int N,
                int8_t* Bres, int32_t* err, ozk_stream_t stream);

/* ---- stage 3b: the N INT8 products with the modular reduction fused into the epilogue (replaces the
 * cuBLASLt INT8 GEMM loop and reduce_k, ozaki_engine.py:1333-1341 and :952-967).  Persistent tcgen05.mma
 * kind::i8 kernel fed by TMA; the INT32 accumulators live in TMEM and never reach HBM.
 * X[t][i][j] = (sum_l Ares[t][i][l] Bres[t][j][l]) mod m_t in [0, m_t).  err: device int32, OR'ed flags.   */
int ozk_gemm_residues(const int8_t* Ares, const int8_t* Bres, int m, int n, int k, int N, uint8_t* X, int32_t* err,
                      ozk_stream_t stream);
/* The same kernel with an INT32 epilogue, for one plane pair: C32 = A_plane B_plane^T (the per-modulus
 * product of ozaki_engine.py:1336, exact while k <= 131071).                                                 */
int ozk_gemm_i32(const int8_t* A_plane, const int8_t* B_plane, int m, int n, int k, int32_t* C32, int32_t* err,
                 ozk_stream_t stream);
/* Self-test of the GEMM's failure path (the reference has none: its waits are cuBLASLt's and the host's).
 * One CTA runs the GEMM's roles over mbarriers that nothing arrives on: role 0 (the TMA producer) or role 1
 * (an epilogue warp) waits limit_ns (1 us .. 4 s) of wall time, gives up, ORs its OZK_DEVERR_TIMEOUT_* flag
 * into *err and raises the CTA's abort flag; the other role leaves through that flag; the TMEM the CTA holds is
 * freed and the kernel returns.  waited_ns: device int64[2], the wall time each role waited (producer first).    */
int ozk_wait_selftest(int role, int64_t limit_ns, int32_t* err, int64_t* waited_ns, ozk_stream_t stream);

/* ---- stage 3c: CRT reconstruction and unscale (replaces recon_k, ozaki_engine.py:1040-1101) ------------- *
 * C[i][j] = the correctly rounded double of the symmetric CRT lift of X[.][i][j], times 2^(r_i + c_j - 2p)
 * (the ldexp rounding of the reference in the subnormal range).  The CRT sums run on the tensor cores
 * (tcgen05.mma kind::i8 over TMA tiles of X); err: device int32, OZK_DEVERR_TIMEOUT_RECON is OR'ed in if one of
 * the kernel's bounded waits runs out (C is then invalid).                                                    */
int ozk_reconstruct(const uint8_t* X, const int32_t* r, const int32_t* c, const int32_t* p_dev, int m, int n, int N,
                    double* C, int32_t* err, ozk_stream_t stream);

/* ---- residue chains (the chain cost law of code/digit_gemm.py:1252-1291, executed): the product planes of
 * ozk_gemm_residues, X[t] in [0, m_t), mapped to the symmetric int8 residues of the split,
 * out[t][e] = X[t][e] - m_t when X[t][e] >= ceil(m_t / 2), else X[t][e]; so that a product stays in residue form
 * and is the left operand of the next product.  plane_elems = elements per plane (a multiple of 16); X and out
 * 16-byte aligned; out may be X itself.                                                                      */
int ozk_residue_symmetric(const uint8_t* X, int N, size_t plane_elems, int8_t* out, ozk_stream_t stream);

/* ---- stage 3 in one call (replaces OzakiCRT.core, ozaki_engine.py:1310-1350): split A (unless skip_a),
 * split B, products, reconstruction.                                                                        */
int ozk_core(const double* A, const double* B, const int32_t* gam, const int32_t* r, const int32_t* c,
             const int32_t* p_dev, int m, int n, int k, int N, int skip_a, int8_t* Ares, int8_t* Bres, uint8_t* X,
             double* C, int32_t* err, ozk_stream_t stream);

/* ---- full-matrix certificate of the plane count (replaces full_certificate, ozaki_engine.py:1542-1583) --- *
 * For the statistics gam, r, c, sA, sB of the problem (inside scaling on): a lower bound of
 * D_ij = sum_l |A_il||B_lj| on every entry from one FP16 tensor-core product (tcgen05.mma kind::f16, FP32
 * accumulation) of the magnitudes scaled by 2^(gamma_l - r_i) and 2^(-c_j - gamma_l) and rounded down by
 * (1 - 2^-10), derated by (1 - 8 k 2^-24); for every entry with D > 0 the largest x with
 * F1 x + F2 x^2 <= tau D / safety (F1 = (2^r_i sB_j + 2^c_j sA_i) / 2, F2 = k 2^(r_i + c_j) / 4).
 * Outputs (device): xmin[0] = min of that x over the entries with D > 0 (all bits set when there is none; the
 * required p is ceil(-log2(xmin) + 1e-9)), uncertified[0] = number of entries with D not > 0.  D_out (optional,
 * m x n, may be NULL) receives D.  Scratch: ozk_certificate_workspace_bytes(m, n, k), 256-byte aligned.
 * err: device int32, OR'ed OZK_DEVERR_* flags of the bounded waits.                                          */
size_t ozk_certificate_workspace_bytes(int m, int n, int k);
int ozk_certificate(const double* A, const double* B, int m, int n, int k, const int32_t* gam, const int32_t* r,
                    const int32_t* c, const double* sA, const double* sB, double tau, double safety, double* xmin,
                    uint64_t* uncertified, double* D_out, int32_t* err, void* workspace, size_t workspace_bytes,
                    ozk_stream_t stream);

/* The plane-count rule driven by the certificate instead of the probe (the certified variant of the rule in the
 * timed path, from the reference's full_certificate, :1570-1575): p_req = ceil(-log2(xmin) + 1e-9) clamped to
 * [1, 1000] (xmin from ozk_certificate), N = the smallest N in [6, 32] with pmax_bits(N, nu_A, nu_B, k) >= p_req;
 * dec[4] = {N (0 on fallback), p = pmax_bits(N, ..), fallback, p_req}, p_dev[1] = p, aux[8] = {nuA, nuB,
 * -log2(xmin), 0...}.  Fallback on a non-finite flag, no such N, or p_req > 249.                             */
int ozk_rule_certified(const double* nA, const double* nB, const int32_t* flag, int m, int n, int k,
                       const double* xmin, int32_t* dec, int32_t* p_dev, double* aux, ozk_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* OZAKI_B200_H */
