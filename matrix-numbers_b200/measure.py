"""Measurement helpers: the seeded synthetic inputs of the benchmark configurations, and the sampled accuracy of a
product against its correctly rounded value.

* ``CONFIGS`` / ``make_inputs`` -- A, B with entries (U(0,1) - 0.5) exp(phi N(0,1)) drawn by numpy
  ``default_rng(seed)`` on the host: all of A's uniforms, then A's normals, then the same for B.  (The reference's
  family "X", code/ozaki_engine.py:457-459, is phi = 2 with torch's CUDA generator, which a CPU cannot reproduce;
  this generator is the host-side stand-in of the same distribution.)  ``alt_sign`` gives the cancellation stress of
  the long-K configuration: A_il = |A_il| (-1)^l and B = |B|, so every dot product alternates in sign.
* ``AccuracySample`` -- the accuracy figures the reference reports (its ``Sample`` / ``exact_sample``,
  :477-521): on a fixed set of rows and columns (default_rng(7) picks, plus the row and the column of the largest
  |C| of a native product), E1 = max |C_hat - C| / max |C| and E2 = max |C_hat - C| / (|A||B|)_ij, with C the
  correctly rounded product.  The correctly rounded value is computed here with Dekker's error-free product and
  Veltkamp's splitting (T. J. Dekker, "A floating-point technique for extending the available precision", 1971),
  then ``math.fsum`` (Shewchuk's exact summation) of the 2k parts.
* ``audit_bound`` -- the reference's Lemma L1 audit (:1755-1766): the sampled error against the a-priori bound.
"""
from __future__ import annotations

import math

import numpy as np
import torch

CONFIGS = {
    # name: (m, k, n, phi, alt_sign, force_N, description)
    "c1": (1024, 1024, 1024, 0.5, False, None, "square M=N=K=1024, phi=0.5, dynamic plane rule"),
    "c2": (4096, 4096, 4096, 0.5, False, None, "square M=N=K=4096, phi=0.5, dynamic plane rule"),
    "c3": (16384, 16384, 16384, 2.0, False, None, "square M=N=K=16384, phi=2.0 (18-20 planes), dynamic plane rule"),
    "c4": (32768, 8192, 32768, 0.5, False, None, "rectangular M=N=32768, K=8192, phi=0.5, C row-blocks over GPUs"),
    "c5": (2048, 262144, 2048, 1.0, True, 16, "long K=262144, M=N=2048, phi=1.0, alternating-sign rows, forced N=16"),
}


def _fill_chunked(g, shape, phi, out):
    """out = (U - 0.5) exp(phi Z): all of U first, then all of Z, each drawn in row chunks (the same stream order
    as one draw of the whole matrix)."""
    m, k = shape
    step = max(1, (1 << 24) // k)
    for i in range(0, m, step):
        out[i:i + step] = g.random((min(step, m - i), k))
    out -= 0.5
    for i in range(0, m, step):
        z = g.standard_normal((min(step, m - i), k))
        z *= phi
        np.exp(z, out=z)
        out[i:i + step] *= z


def make_inputs(m, k, n, phi, seed=0, alt_sign=False):
    """Host float64 (numpy) A (m x k) and B (k x n) of the benchmark generator."""
    g = np.random.default_rng(seed)
    A = np.empty((m, k))
    B = np.empty((k, n))
    _fill_chunked(g, (m, k), phi, A)
    _fill_chunked(g, (k, n), phi, B)
    if alt_sign:
        np.abs(A, out=A)
        A[:, 1::2] *= -1.0
        np.abs(B, out=B)
    return A, B


def config_inputs(name, seed=0, device="cuda"):
    m, k, n, phi, alt, _, _ = CONFIGS[name]
    A, B = make_inputs(m, k, n, phi, seed, alt)
    return torch.from_numpy(A).to(device), torch.from_numpy(B).to(device)


def make_inputs_w(n, seed=0):
    """The reference's rotated ill-scaled family W (make_inputs_ext, :1618-1631), from numpy's generator:
    A = rotate_rows(At diag(d)), B = rotate_cols(diag(d)^-1 Bt) with d_l = 2^(20 l / (n - 1)) and At, Bt standard
    normal, so A B keeps 20 binades of column / row scaling that inside scaling has to undo."""
    g = np.random.default_rng(1000 * seed + n + 7)
    At = g.standard_normal((n, n))
    Bt = g.standard_normal((n, n))
    d = np.exp2(20.0 * np.arange(n) / (n - 1))
    idx = (np.arange(n)[None, :] + np.arange(n)[:, None]) % n
    A = np.take_along_axis(At * d[None, :], idx, axis=1)
    B = np.take_along_axis(Bt / d[:, None], idx, axis=0)
    return np.ascontiguousarray(A), np.ascontiguousarray(B)


# ------------------------------------------------------------------------------------------------ exact products
_VELTKAMP = float(2 ** 27 + 1)


def _veltkamp(x):
    """x = hi + lo exactly, hi and lo with at most 26 significant bits each (no overflow below 2^996)."""
    c = _VELTKAMP * x
    hi = c - (c - x)
    return hi, x - hi


def two_products(a, b):
    """Dekker's error-free product, elementwise: a b = p + e exactly, p = fl(a b) (finite inputs, no underflow)."""
    p = a * b
    ah, al = _veltkamp(a)
    bh, bl = _veltkamp(b)
    e = al * bl - (((p - ah * bh) - al * bh) - ah * bl)
    return p, e


def correctly_rounded_products(rows, cols):
    """fl(rows @ cols) with every entry correctly rounded: each of the k products is split exactly into p + e, and
    ``math.fsum`` rounds the exact sum of the 2k parts once.  rows (r, k), cols (k, c) float64 numpy."""
    r = rows.shape[0]
    c = cols.shape[1]
    out = np.empty((r, c))
    for j in range(c):
        p, e = two_products(rows, cols[:, j][None, :])
        parts = np.concatenate((p, e), axis=1)
        for i in range(r):
            out[i, j] = math.fsum(parts[i].tolist())
    return out


class AccuracySample:
    """Sampled accuracy of products of one (A, B) against the correctly rounded product (module docstring)."""

    def __init__(self, A, B, C_native=None, nr=48, nc=48, seed=7):
        m, n = A.shape[0], B.shape[1]
        pick = np.random.default_rng(seed)
        rows = set(pick.choice(m, min(nr, m), replace=False).tolist())
        cols = set(pick.choice(n, min(nc, n), replace=False).tolist())
        if C_native is not None:
            mag = torch.abs(C_native)
            rows.add(int(mag.amax(dim=1).argmax().item()))
            cols.add(int(mag.amax(dim=0).argmax().item()))
        self.ri = np.array(sorted(rows))
        self.ci = np.array(sorted(cols))
        self.tri = torch.as_tensor(self.ri, device=A.device)
        self.tci = torch.as_tensor(self.ci, device=A.device)
        A_rows = A.index_select(0, self.tri).cpu().numpy()
        B_cols = B.index_select(1, self.tci).cpu().numpy()
        self.ref = correctly_rounded_products(A_rows, B_cols)
        self.absab = np.abs(A_rows) @ np.abs(B_cols)
        self.den1 = float(np.abs(self.ref).max())

    def take(self, C):
        """The sampled entries of a product C (device or host tensor) as numpy."""
        return C.index_select(0, self.tri.to(C.device)).index_select(1, self.tci.to(C.device)).cpu().numpy()

    def errors(self, C):
        diff = np.abs(self.take(C) - self.ref)
        with np.errstate(all="ignore"):
            rel = np.where(self.absab > 0, diff / self.absab, 0.0)
        worst = float(diff.max())
        return {"E1": worst / self.den1 if self.den1 > 0 else worst, "E2": float(rel.max())}


def audit_bound(S, info, k, C, scale=1.0):
    """Lemma L1 audit on a sample (the reference's audit_bound, :1755-1766): the error of every sampled entry against
    scale E_ij(p) plus the two roundings 2^-53 (|C_hat| + |C_ref|), with a relative slack of 1e-9.  Returns the
    violation count, the worst error / limit, the median bound / error and the worst error / D."""
    from .constants import bound_matrix
    st = info["stats"]
    bound = scale * bound_matrix(st["r"], st["c"], st["sA"], st["sB"], k, info["p"], S.ri, S.ci)
    got = S.take(C)
    err = np.abs(got - S.ref)
    limit = (bound + 2.0 ** -53 * (np.abs(got) + np.abs(S.ref))) * (1.0 + 1e-9)
    hit = err > 0
    return {"max_err_over_bound": float((err / limit).max()), "violations": int(np.count_nonzero(err > limit)),
            "median_bound_over_err": float(np.median(bound[hit] / err[hit])) if hit.any() else None,
            "max_err_over_D": float((err / S.absab).max())}


# the reference's names for the accuracy sample and the exact products
Sample = AccuracySample
exact_sample = correctly_rounded_products

__all__ = ["CONFIGS", "make_inputs", "config_inputs", "make_inputs_w", "two_products", "correctly_rounded_products",
           "AccuracySample", "Sample", "exact_sample", "audit_bound"]
