"""CPU oracle for the FP64-on-INT8 (Ozaki-II / CRT) GEMM path -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline / reference arm of ``bench.py`` import this module,
and only as the checker (or, in bench.py, as the timed CPU baseline).  The product package never imports it.

It wraps ``libozaki_oracle.so`` (``ozaki_oracle.c``: a C/OpenMP restatement of the reference engine
dl1683/matrix-numbers ``code/ozaki_engine.py``, file:line citations in that file) with numpy-level functions, and
adds the pieces of the reference's host logic that are plain Python there:

* ``probe_sets``          -- the probe rows/columns of ``choose`` (ozaki_engine.py:1265-1273)
* ``rule``                -- the host form of the a-priori rule (ozaki_engine.py:1250-1307), computed in C
* ``run``                 -- stats -> rule -> core, the eager ``OzakiCRT.run`` (ozaki_engine.py:1460-1505)

The oracle is pinned against the reference itself by ``tests/test_oracle_golden.py`` (golden vectors generated
by ``tests/golden/make_golden.py`` from the reference's own ``np_stats``, ``expected_core``, ``pmax_bits``,
``choose`` and ``_rule_device``).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libozaki_oracle.so")

MODS = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181, 179, 173, 167, 163,
        157, 151, 149, 139, 137, 131, 127, 113, 109, 107]
NMAX = 32
NEG = -1000000

_lib = None


def build(force: bool = False) -> str:
    """Compile libozaki_oracle.so with the committed Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
            os.path.join(HERE, "ozaki_oracle.c")):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        i32, f64 = ctypes.c_int, ctypes.c_double
        L.ozo_stats.argtypes = [P, P, i32, i32, i32, i32, P, P, P, P, P, P, P, P]
        L.ozo_stats_ext.argtypes = [P, P, i32, i32, i32, i32, P, P, P, P, P, P, P, P, P, P]
        L.ozo_colmax.argtypes = [P, i32, i32, P]
        L.ozo_pmax_bits.argtypes = [i32, f64, f64, i32]
        L.ozo_pmax_bits.restype = i32
        L.ozo_modulus_product.argtypes = [i32]
        L.ozo_modulus_product.restype = f64
        L.ozo_limbs_for.argtypes = [i32]
        L.ozo_limbs_for.restype = i32
        L.ozo_probe_D.argtypes = [P, P, i32, i32, i32, P, i32, P, i32, P]
        L.ozo_rule.argtypes = [P, P, P, P, P, P, i32, i32, i32, i32, P, i32, P, i32, P, f64, f64, i32, P, P, P]
        L.ozo_split_A.argtypes = [P, P, P, i32, i32, i32, i32, P]
        L.ozo_split_B.argtypes = [P, P, P, i32, i32, i32, i32, P]
        L.ozo_gemm_mod.argtypes = [P, P, i32, i32, i32, i32, P]
        L.ozo_gemm_i32.argtypes = [P, P, i32, i32, i32, P]
        L.ozo_recon.argtypes = [P, P, P, i32, i32, i32, i32, P]
        L.ozo_core.argtypes = [P, P, P, P, P, i32, i32, i32, i32, i32, P]
        L.ozo_core.restype = i32
        L.ozo_num_threads.restype = i32
        L.ozo_set_threads.argtypes = [i32]
        L.ozo_set_threads.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


def _c64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


def num_threads() -> int:
    return int(lib().ozo_num_threads())


def set_threads(n: int) -> int:
    """Run the parallel loops on n threads (overrides OMP_NUM_THREADS); returns the count now in effect."""
    lib().ozo_set_threads(int(n))
    return num_threads()


def stats(A, B, inside=True):
    """Reference statistics (ozaki_engine.py:846-951): dict gam, r, c, sA, nA, sB, nB, flag."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    out = {"gam": np.zeros(k, np.int32), "r": np.zeros(m, np.int32), "c": np.zeros(n, np.int32),
           "sA": np.zeros(m), "nA": np.zeros(m), "sB": np.zeros(n), "nB": np.zeros(n)}
    flag = np.zeros(1, np.int32)
    lib().ozo_stats(_p(A), _p(B), m, n, k, 1 if inside else 0, _p(out["gam"]), _p(out["r"]), _p(out["c"]),
                    _p(out["sA"]), _p(out["nA"]), _p(out["sB"]), _p(out["nB"]), _p(flag))
    out["flag"] = int(flag[0])
    return out


def colmax(A):
    """max over rows of the |A_il| bit patterns (uint64 as int64)."""
    A = _c64(A)
    m, k = A.shape
    out = np.zeros(k, np.uint64)
    lib().ozo_colmax(_p(A), m, k, _p(out))
    return out.view(np.int64)


def rowmax(B):
    """max over columns of the |B_lj| bit patterns (uint64 as int64)."""
    B = _c64(B)
    return (B.view(np.uint64) & np.uint64(0x7FFFFFFFFFFFFFFF)).max(axis=1).view(np.int64)


def stats_given_maxima(A, B, colmax_global, rowmax_global=None, inside=True):
    """Statistics of a row block of A and a column block of B given the column max of |A| over all rows and (if
    given) the row max of |B| over all columns (blocked products)."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    cm = np.ascontiguousarray(np.asarray(colmax_global).view(np.uint64))
    rm = None if rowmax_global is None else np.ascontiguousarray(np.asarray(rowmax_global).view(np.uint64))
    out = {"gam": np.zeros(k, np.int32), "r": np.zeros(m, np.int32), "c": np.zeros(n, np.int32),
           "sA": np.zeros(m), "nA": np.zeros(m), "sB": np.zeros(n), "nB": np.zeros(n)}
    flag = np.zeros(1, np.int32)
    lib().ozo_stats_ext(_p(A), _p(B), m, n, k, 1 if inside else 0, _p(cm), None if rm is None else _p(rm),
                        _p(out["gam"]), _p(out["r"]), _p(out["c"]), _p(out["sA"]), _p(out["nA"]), _p(out["sB"]),
                        _p(out["nB"]), _p(flag))
    out["flag"] = int(flag[0])
    return out


def stats_given_colmax(A, B, colmax_global, inside=True):
    """Statistics of a row block of A given the column max of |A| over all rows (row-sharded products)."""
    return stats_given_maxima(A, B, colmax_global, None, inside)


def pmax_bits(N, nuA, nuB, k) -> int:
    return int(lib().ozo_pmax_bits(int(N), float(nuA), float(nuB), int(k)))


def modulus_product(N) -> float:
    return float(lib().ozo_modulus_product(int(N)))


def limbs_for(N) -> int:
    return int(lib().ozo_limbs_for(int(N)))


def probe_random(m, n, seed=0):
    """Random part of the probe set: RandomState(seed).choice without replacement, rows then columns
    (ozaki_engine.py:1265-1267 and :1399-1401)."""
    rs = np.random.RandomState(seed)
    Ir = rs.choice(m, min(64, m), replace=False)
    Jr = rs.choice(n, min(64, n), replace=False)
    return Ir.astype(np.int64), Jr.astype(np.int64)


def hard_top(r, s, k, count=32):
    """Indices of the `count` largest 2^r k / s (0 where s == 0); ties broken by the lower index
    (ozaki_engine.py:1268-1271)."""
    r = np.asarray(r, dtype=np.float64)
    s = np.asarray(s, dtype=np.float64)
    with np.errstate(all="ignore"):
        h = np.where(s > 0, np.exp2(r) * k / s, 0.0)
    order = np.argsort(-h, kind="stable")
    return order[:min(count, len(h))].astype(np.int64)


def probe_sets(st, m, n, k, seed=0):
    Ir, Jr = probe_random(m, n, seed)
    I = np.unique(np.concatenate([Ir, hard_top(st["r"], st["sA"], k)]))
    J = np.unique(np.concatenate([Jr, hard_top(st["c"], st["sB"], k)]))
    return I.astype(np.int64), J.astype(np.int64)


def probe_D(A, B, I, J):
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    I = np.ascontiguousarray(I, dtype=np.int64)
    J = np.ascontiguousarray(J, dtype=np.int64)
    D = np.zeros((len(I), len(J)))
    lib().ozo_probe_D(_p(A), _p(B), m, n, k, _p(I), len(I), _p(J), len(J), _p(D))
    return D


def rule(st, m, n, k, I, J, D, tau=2.0 ** -52, safety=2.0, force_N=None):
    """Host form of the a-priori rule given stats, probe sets and D (ozaki_engine.py:1250-1307).
    Returns dict N (None on fallback), p, fallback, p_req, worst_ratio_E_over_D, nuA, nuB."""
    I = np.ascontiguousarray(I, dtype=np.int64)
    J = np.ascontiguousarray(J, dtype=np.int64)
    D = _c64(D)
    out = np.zeros(4, np.int32)
    worst = np.zeros(1)
    nus = np.zeros(2)
    r = np.ascontiguousarray(st["r"], np.int32)
    c = np.ascontiguousarray(st["c"], np.int32)
    sA, sB, nA, nB = (_c64(st[x]) for x in ("sA", "sB", "nA", "nB"))
    lib().ozo_rule(_p(r), _p(c), _p(sA), _p(sB), _p(nA), _p(nB), m, n, k, int(st.get("flag", 0)), _p(I), len(I), _p(J),
                   len(J), _p(D), float(tau), float(safety), int(force_N or 0), _p(out), _p(worst), _p(nus))
    return {"N": int(out[0]) if out[0] else None, "p": int(out[1]), "fallback": bool(out[2]), "p_req": int(out[3]),
            "worst_ratio_E_over_D": float(worst[0]), "nuA": float(nus[0]), "nuB": float(nus[1])}


def split_A(A, r, gam, p, N):
    A = _c64(A)
    m, k = A.shape
    out = np.zeros((N, m, k), np.int8)
    lib().ozo_split_A(_p(A), _p(np.ascontiguousarray(r, np.int32)), _p(np.ascontiguousarray(gam, np.int32)), m, k,
                      int(p), int(N), _p(out))
    return out


def split_B(B, c, gam, p, N):
    B = _c64(B)
    k, n = B.shape
    out = np.zeros((N, n, k), np.int8)
    lib().ozo_split_B(_p(B), _p(np.ascontiguousarray(c, np.int32)), _p(np.ascontiguousarray(gam, np.int32)), k, n,
                      int(p), int(N), _p(out))
    return out


def gemm_mod(Ares, Bres):
    N, m, k = Ares.shape
    n = Bres.shape[1]
    X = np.zeros((N, m, n), np.uint8)
    lib().ozo_gemm_mod(_p(np.ascontiguousarray(Ares)), _p(np.ascontiguousarray(Bres)), m, n, k, N, _p(X))
    return X


def gemm_i32(At, Bt):
    m, k = At.shape
    n = Bt.shape[0]
    C = np.zeros((m, n), np.int32)
    lib().ozo_gemm_i32(_p(np.ascontiguousarray(At)), _p(np.ascontiguousarray(Bt)), m, n, k, _p(C))
    return C


def recon(X, r, c, p):
    N, m, n = X.shape
    C = np.zeros((m, n))
    lib().ozo_recon(_p(np.ascontiguousarray(X)), _p(np.ascontiguousarray(r, np.int32)),
                    _p(np.ascontiguousarray(c, np.int32)), m, n, N, int(p), _p(C))
    return C


def core(A, B, st, N, p):
    """split + exact products + reconstruction for given (N, p): the CPU port of core() (ozaki_engine.py:1310)."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    C = np.zeros((m, n))
    rc = lib().ozo_core(_p(A), _p(B), _p(np.ascontiguousarray(st["gam"], np.int32)),
                        _p(np.ascontiguousarray(st["r"], np.int32)), _p(np.ascontiguousarray(st["c"], np.int32)),
                        m, n, k, int(N), int(p), _p(C))
    if rc != 0:
        raise MemoryError("oracle core: allocation failed")
    return C


def run(A, B, tau=2.0 ** -52, force_N=None, inside=True, seed=0, force_p=None, safety=2.0):
    """Eager OzakiCRT.run on the CPU (ozaki_engine.py:1460-1505): returns (C, info).  Fallback cases return
    C = None (the reference would call native DGEMM there)."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    st = stats(A, B, inside)
    info = {"nonfinite": bool(st["flag"])}
    if st["flag"]:
        info["fallback"] = True
        return None, info
    I, J = probe_sets(st, m, n, k, seed)
    D = probe_D(A, B, I, J) if not force_N else np.zeros((len(I), len(J)))
    ru = rule(st, m, n, k, I, J, D, tau, safety, force_N)
    info.update(ru)
    info["probe"] = [len(I), len(J)]
    if ru["fallback"] or ru["N"] is None:
        info["fallback"] = True
        return None, info
    N, p = ru["N"], ru["p"]
    if force_p is not None:
        if force_p > p:
            info["fallback"] = True
            info["config_rejected"] = True
            return None, info
        p = int(force_p)
    info["N"], info["p"], info["L"] = N, p, limbs_for(N)
    info["stats"] = st
    return core(A, B, st, N, p), info


# ------------------------------------------------------------------ the exact sampled reference (measurement)
def persist_product(A, B, N, p):
    """One product of the persistent fixed operand mode (PersistA, ozaki_engine.py:2417-2466) on the CPU: A encoded
    at (N, p) with gamma = 0 (encode, :2433-2442), B's column statistics with gamma = 0, the forced rule for (N, p)
    (_stats_B -> _rule_device, :2444-2454, :1387-1396: p_B = min(pmax_bits(N, nu_A, nu_B, k), p), fallback flag when
    that is below p), then core with skipA: B residues and reconstruction at p_B, the A planes kept at p.
    Returns (C, {"p_B", "fallback"})."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    n = B.shape[1]
    st = stats(A, B, inside=False)                         # gamma = 0: the row and column statistics of encode/_stats_B
    nuA, nuB = math.sqrt(float(np.max(st["nA"]))), math.sqrt(float(np.max(st["nB"])))
    pv = pmax_bits(N, nuA, nuB, k)
    pB = min(pv, int(p))
    Ares = split_A(A, st["r"], st["gam"], p, N)
    Bres = split_B(B, st["c"], st["gam"], pB, N)
    C = recon(gemm_mod(Ares, Bres), st["r"], st["c"], pB)
    return C, {"p_B": pB, "fallback": pv < int(p)}


def full_certificate(A, B, st, tau=2.0 ** -52, safety=2.0):
    """The reference's full_certificate arithmetic (ozaki_engine.py:1542-1583) in numpy: FP16 magnitudes scaled by
    2^(gamma - r) and 2^(-c - gamma), rounded down by (1 - 2^-10) and converted through float32 as torch's
    .to(float16) does; their product summed in float64 (the reference sums in FP32 on the tensor cores: both sums
    differ from the exact one by far less than the 8 k 2^-24 derating); the bound of every entry; the maximum need.
    Returns need, preq, uncertified and the matrices D (derated lower bound) and xmax."""
    A, B = _c64(A), _c64(B)
    m, k = A.shape
    r = np.asarray(st["r"], np.int64)
    c = np.asarray(st["c"], np.int64)
    gam = np.asarray(st["gam"], np.int64)
    g = np.ldexp(1.0, gam)
    As = (np.abs(A) * (g[None, :] * np.ldexp(1.0, -r)[:, None]) * (1 - 2.0 ** -10)).astype(np.float32).astype(np.float16)
    Bs = (np.abs(B) * (np.ldexp(1.0, -c)[None, :] / g[:, None]) * (1 - 2.0 ** -10)).astype(np.float32).astype(np.float16)
    Dl = As.astype(np.float64) @ Bs.astype(np.float64)
    rI, cJ = np.ldexp(1.0, r)[:, None], np.ldexp(1.0, c)[None, :]
    D = Dl * (1 - 8 * k * 2.0 ** -24) * rI * cJ
    F1 = 0.5 * (rI * np.asarray(st["sB"])[None, :] + cJ * np.asarray(st["sA"])[:, None])
    F2 = 0.25 * k * rI * cJ
    thr = tau * D / safety
    mask = D > 0
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        xmax = 2 * thr / (F1 + np.sqrt(F1 * F1 + 4 * F2 * thr))
        need = float(np.where(mask, -np.log2(xmax), -1e30).max())
    return {"need": need, "preq": int(math.ceil(need + 1e-9)), "uncertified": int((~mask).sum()), "D": D,
            "xmax": xmax}


def certificate_xmin(A, B, st, tau=2.0 ** -52, safety=2.0):
    """min xmax over the entries with D > 0 of ``full_certificate``'s bound (ozaki_engine.py:1542-1583) as the float64
    bit pattern (int; -1 when no entry has D > 0), and the number of entries with D not > 0."""
    cert = full_certificate(A, B, st, tau, safety)
    mask = cert["D"] > 0
    if not mask.any():
        return -1, cert["uncertified"]
    x = float(np.min(cert["xmax"][mask]))
    return int(np.array([x], dtype=np.float64).view(np.int64)[0]), cert["uncertified"]


def rule_certified(nA, nB, flag, k, xmin_bits):
    """The plane-count decision from the certificate's minimum (the device rule of the certified mode):
    p_req = ceil(-log2(xmin) + 1e-9) clamped to [1, 1000] (the reference's preq_full, :1570-1573), N = the smallest
    plane count in [6, 32] whose pmax_bits reaches it (:1119-1139), fallback on a non-finite flag, no such N or
    p_req > 249.  Returns (N, p, fallback, p_req)."""
    nuA, nuB = math.sqrt(float(np.max(nA))), math.sqrt(float(np.max(nB)))
    if xmin_bits == -1:
        need = -1e30
    else:
        need = -math.log2(float(np.array([xmin_bits], dtype=np.int64).view(np.float64)[0]))
    preq = int(min(max(math.ceil(need + 1e-9), 1), 1000))
    N = next((t for t in range(6, NMAX + 1) if pmax_bits(t, nuA, nuB, k) >= preq), 0)
    fb = bool(flag) or N == 0 or preq > 249
    p = pmax_bits(N, nuA, nuB, k) if N else 0
    return (0 if fb else N), p, fb, preq


def run_certified(A, B, tau=2.0 ** -52, safety=2.0):
    """The certified-mode product on the CPU: statistics, the full-matrix certificate's minimum, the certified rule,
    then core at (N, p); (C, info) with C None on fallback."""
    A, B = _c64(A), _c64(B)
    st = stats(A, B, True)
    xb, unc = certificate_xmin(A, B, st, tau, safety)
    N, p, fb, preq = rule_certified(st["nA"], st["nB"], st["flag"], A.shape[1], xb)
    if fb:
        return None, {"fallback": True, "p_req": preq}
    return core(A, B, st, N, p), {"N": N, "p": p, "p_req": preq, "uncertified": unc}


def chain_exact(mats):
    """Exact product A_1 A_2 ... A_q of integer matrices as Python integers (numpy object arrays), the value an exact
    residue chain must reproduce (code/digit_gemm.py:1252-1291 models its cost: one INT8 GEMM per modulus per
    product, residues reduced after every product).  Returns the object array."""
    out = np.asarray(mats[0]).astype(np.int64).astype(object)
    for A in mats[1:]:
        out = out.dot(np.asarray(A).astype(np.int64).astype(object))
    return out


def chain_residues(mats, N):
    """The chain computed the way the residue form computes it: per modulus m_t (the first N of MODS) the running
    product is reduced modulo m_t after every product and mapped to the split's symmetric range
    [-floor(m/2), ceil(m/2) - 1] (ozaki_engine.py:989-995) before the next one; the last product is left in
    [0, m_t) (the GEMM epilogue's range, ozaki_engine.py:952-967).  int64 arithmetic (|products| < 2^63 for the
    dimensions tests use).  Returns uint8 planes (N, m, n)."""
    planes = []
    for t in range(N):
        P = MODS[t]

        def sym(x):
            x = np.mod(x, P)
            return np.where(x >= (P + 1) // 2, x - P, x)
        cur = sym(np.asarray(mats[0]).astype(np.int64))
        for s, A in enumerate(mats[1:]):
            cur = np.mod(cur @ sym(np.asarray(A).astype(np.int64)), P)
            if s + 2 < len(mats):
                cur = sym(cur)
        planes.append(cur.astype(np.uint8))
    return np.stack(planes)


def _split(a):
    t = 134217729.0 * a
    hi = t - (t - a)
    return hi, a - hi


def exact_sample(Ar, Bc):
    """Correctly rounded Ar @ Bc by Dekker TwoProduct + math.fsum (the reference's exact_sample,
    ozaki_engine.py:477-496)."""
    r, n = Ar.shape
    c = Bc.shape[1]
    out = np.empty((r, c))
    bh, bl = _split(Bc)
    for i in range(r):
        a = Ar[i][:, None]
        ah, al = _split(a)
        p = a * Bc
        e = ((ah * bh - p) + ah * bl + al * bh) + al * bl
        for j in range(c):
            out[i, j] = math.fsum(p[:, j].tolist() + e[:, j].tolist())
    return out
