"""Host-side planning helpers of the reference's digit-GEMM theory (dl1683/matrix-numbers code/digit_gemm.py):
the choice of pairwise-coprime INT8 moduli for exact integer products and the cost law of residue chains.

These decide configurations; they run on the host (scipy's HiGHS MILP) and are not on the GPU path.  The engine
itself uses the fixed moduli list MODS (constants.py), as the reference's engine does; ``int8_crt`` answers the
different question of the fewest moduli <= 256 that make an integer product of b-bit entries exact.
"""
from __future__ import annotations

import math

import numpy as np


def _primes_upto(n: int):
    sieve = np.ones(n + 1, dtype=bool)
    sieve[:2] = False
    for p in range(2, int(n ** 0.5) + 1):
        if sieve[p]:
            sieve[p * p::p] = False
    return [int(p) for p in np.nonzero(sieve)[0]]


def coprime_ip(cands, target_log2, bound_int=None):
    """Cheapest set of pairwise-coprime moduli whose log2-product reaches ``target_log2`` (digit_gemm.py:1224-1241).

    cands: list of (modulus, cost).  0/1 integer program: minimise sum cost_m x_m - 1e-6 log2(m) x_m (the small term
    prefers the larger product among equal costs) subject to sum log2(m) x_m >= target_log2 + 1e-9 and, for every prime
    q, sum over moduli divisible by q of x_m <= 1 (pairwise coprime).  If ``bound_int`` is given, the chosen product
    must exceed it exactly (the log2 constraint is only a float test).  Returns (moduli descending, total cost) or
    (None, None) when no set reaches the target."""
    from scipy.optimize import Bounds, LinearConstraint, milp
    ms = [int(m) for m, _ in cands]
    cost = np.array([float(c) for _, c in cands])
    lg = np.array([math.log2(m) for m in ms])
    top = max(ms) if ms else 1
    rows = [[1.0 if m % q == 0 else 0.0 for m in ms] for q in _primes_upto(top) if any(m % q == 0 for m in ms)]
    cons = [LinearConstraint(np.array(rows), -np.inf, 1.0), LinearConstraint(lg[None, :], target_log2 + 1e-9, np.inf)]
    res = milp(cost - 1e-6 * lg, constraints=cons, integrality=np.ones(len(ms)), bounds=Bounds(0, 1))
    if res.x is None:
        return None, None
    chosen = [m for m, x in zip(ms, res.x) if x > 0.5]
    if bound_int is not None and math.prod(chosen) <= bound_int:
        raise AssertionError("coprime_ip: the float log2 constraint admitted a product that does not exceed the bound")
    total = int(round(sum(c for (m, c), x in zip(cands, res.x) if x > 0.5)))
    return sorted(chosen, reverse=True), total


def int8_crt(b, k):
    """Fewest pairwise-coprime moduli <= 256 (one INT8 GEMM each, symmetric residues) that make the product of
    b-bit-magnitude integer matrices (|x| <= 2^b - 1) with inner dimension k exact: prod m > 2 k (2^b - 1)^2
    (digit_gemm.py:1244-1249).  Returns (moduli, count)."""
    bound = 2 * k * (2 ** b - 1) ** 2
    return coprime_ip([(m, 1) for m in range(2, 257)], math.log2(bound), bound)


def chain_cost_model(configs=((7, 4096), (8, 4096), (16, 4096), (24, 4096), (53, 4096)), qmax=40):
    """INT8 GEMM counts of exact product CHAINS A_1 A_2 ... A_q kept in residue form (digit_gemm.py:1252-1291).

    Entries bounded by H = 2^b - 1 and inner dimension k give |(A_1..A_s)_ij| <= R_s = H^s k^(s-1); N(R) = fewest
    pairwise-coprime moduli <= 256 with product > 2R.  A fixed base (the final one) costs (q - 1) N(R_q) GEMMs, a base
    grown before every product sum_{s=2..q} N(R_s); rounding after every product costs (q - 1) N(R_2) (CRT) or
    (q - 1)(2 ceil((b + 1) / 8) - 1) (the one-modulus floor).  Exactness is capped by lcm(1..256): the chain stops at
    the first q whose 2 R_q exceeds it.  Returns {"cap_log2_lcm_1_256", "rows"} like the reference's table."""
    cap = math.log2(math.lcm(*range(1, 257)))
    rows = []
    for b, k in configs:
        H = 2 ** b - 1
        memo = {}

        def count(s):
            if s not in memo:
                R = H ** s * k ** (s - 1)
                memo[s] = None if math.log2(2 * R) > cap else coprime_ip([(m, 1) for m in range(2, 257)],
                                                                         math.log2(2 * R), 2 * R)[1]
            return memo[s]

        for q in range(2, qmax + 1):
            if count(q) is None:
                rows.append({"b": b, "k": k, "q": q, "exact_cap_exceeded": True})
                break
            rows.append({"b": b, "k": k, "q": q, "log2_R_q": round(math.log2(H ** q * k ** (q - 1)), 1),
                         "N_final": count(q), "gemms_fixed_base": (q - 1) * count(q),
                         "gemms_growing_base": sum(count(s) for s in range(2, q + 1)),
                         "rounded_chain_crt": (q - 1) * count(2),
                         "rounded_chain_M1_floor": (q - 1) * (2 * ((b + 1 + 7) // 8) - 1)})
    return {"cap_log2_lcm_1_256": round(cap, 2), "rows": rows}


__all__ = ["coprime_ip", "int8_crt", "chain_cost_model"]
