"""Moduli, range bounds and the data-independent configuration table of the FP64-on-INT8 engine.

Host helpers with the names and meaning of the reference engine's (dl1683/matrix-numbers code/ozaki_engine.py):
``MODS``/``NMAX``/``NEG`` (:824-829), ``_limbs_for`` (:1104-1106), ``_pow2tab`` (:1109-1116), ``pmax_bits``
(:1119-1139), ``bound_matrix`` (:1142-1147, Lemma L1), ``worst_case_p``/``sigma_of`` (:1511-1520),
``make_config_table``/``pick_config`` (:1523-1539, schema ``ozaki_crt_int8_config_v1``).  ``pmax_bits`` is evaluated by
the compiled library (``ozk_pmax_bits``), the same code the device rule runs.
"""
from __future__ import annotations

import json
import math

import numpy as np

from . import _lib

MODS = [256, 255, 253, 251, 247, 241, 239, 233, 229, 227, 223, 217, 211, 199, 197, 193, 191, 181, 179, 173, 167, 163,
        157, 151, 149, 139, 137, 131, 127, 113, 109, 107]
NMAX = len(MODS)
NEG = -1000000
assert all(math.gcd(a, b) == 1 for i, a in enumerate(MODS) for b in MODS[i + 1:]), "moduli not pairwise coprime"


def limbs_for(N: int) -> int:
    """32-bit limbs of prod(MODS[:N]), at least 2."""
    return int(_lib.lib().ozk_limbs_for(int(N)))


_limbs_for = limbs_for


def _pow2tab() -> np.ndarray:
    """2^s mod m_t for t < 32, s < 256 (uint8)."""
    t = np.zeros((NMAX, 256), dtype=np.uint8)
    for ti, p in enumerate(MODS):
        v = 1 % p
        for s in range(256):
            t[ti, s] = v
            v = (v * 2) % p
    return t


def modulus_product(N: int) -> float:
    """float(prod(MODS[:N])), correctly rounded."""
    return float(_lib.lib().ozk_modulus_product(int(N)))


def pmax_bits(N: int, nuA: float, nuB: float, k: int) -> int:
    """Largest p in [0, 249] with 2 Xmax(p) + 1 <= M_N, Xmax(p) = (2^p nuA + sqrt(k)/2)(2^p nuB + sqrt(k)/2)."""
    return int(_lib.lib().ozk_pmax_bits(int(N), float(nuA), float(nuB), int(k)))


def bound_matrix(r, c, sA, sB, k, p, I, J) -> np.ndarray:
    """Lemma L1 bound E_ij(p) = 2^(r_i-p) sB_j / 2 + 2^(c_j-p) sA_i / 2 + k 2^(r_i+c_j-2p) / 4 on the pairs I x J."""
    rI = np.asarray(r, dtype=np.float64)[I][:, None]
    cJ = np.asarray(c, dtype=np.float64)[J][None, :]
    return (0.5 * np.exp2(rI - p) * np.asarray(sB)[J][None, :] + 0.5 * np.exp2(cJ - p) * np.asarray(sA)[I][:, None]
            + 0.25 * k * np.exp2(rI + cJ - 2 * p))


def worst_case_p(N: int, k: int) -> int:
    """Data-independent p for N moduli and inner dimension k (nu_A = nu_B = sqrt(k), the range bound's worst case)."""
    return pmax_bits(N, math.sqrt(k), math.sqrt(k), k)


def sigma_of(p: int) -> float:
    """Scaled contract of Lemma L1: |C_hat - C|_ij <= sigma k 2^(r_i + c_j) + 2^-53 |C_hat_ij| (normal range)."""
    return 2.0 ** -p * (1 + 2.0 ** (-p - 2))


def make_config_table(path=None, ks=(1024, 2048, 4096, 8192, 16384)) -> dict:
    tab = {"schema": "ozaki_crt_int8_config_v1",
           "value_set": "int8 signed residues, INT32 accumulation, pairwise-coprime moduli <= 256",
           "moduli": MODS,
           "contract": "for finite inputs with normal-range results: |C_hat_ij - C_ij| <= sigma * k * 2^(r_i + c_j) + "
                       "2^-53 |C_hat_ij| + 2^-1075; 2^r_i > max_l |A_il| 2^gamma_l, 2^c_j > max_l |B_lj| 2^-gamma_l "
                       "(row/column scales after inside scaling); exact CRT stage needs 2 Xmax(p) + 1 <= prod(moduli[:N])",
           "rigor": "Lemma L1; sigma is a worst-case guarantee, not a sample",
           "entries": [{"k": k, "N": N, "p": worst_case_p(N, k), "sigma": sigma_of(worst_case_p(N, k))}
                       for k in ks for N in range(6, NMAX + 1)]}
    if path is not None:
        with open(path, "w") as f:
            json.dump(tab, f, indent=1)
    return tab


def pick_config(table, k, sigma_target):
    """Smallest-N entry of the table whose k >= k and whose guaranteed sigma <= sigma_target, else None."""
    ks = sorted({e["k"] for e in table["entries"] if e["k"] >= k})
    if not ks:
        return None
    for e in sorted((e for e in table["entries"] if e["k"] == ks[0]), key=lambda e: e["N"]):
        if e["sigma"] <= sigma_target:
            return {"N": e["N"], "p": e["p"], "sigma": e["sigma"], "table_k": e["k"]}
    return None
