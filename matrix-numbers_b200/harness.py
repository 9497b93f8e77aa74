"""Measurement helpers: the seeded synthetic inputs of the benchmark configurations and the sampled accuracy
metrics E1 / E2 against a correctly rounded reference.

* ``make_inputs`` -- A, B with entries (U(0,1) - 0.5) exp(phi N(0,1)): numpy ``default_rng(seed)`` on the host,
  A before B, U before N (the generator of the benchmark configurations; the reference's family "X" is phi = 2,
  code/ozaki_engine.py:457-459).  ``alt_sign`` gives the cancellation stress of the long-K configuration:
  A_il = |A_il| (-1)^l, B = |B|, so every dot product is a fully alternating sum.
* ``Sample`` -- 48 + 1 rows and columns (the row / column of the largest native |C| included), correctly rounded
  reference by TwoProduct + ``math.fsum``, E1 = max|C_hat - C| / max|C|, E2 = max |C_hat - C| / (|A||B|) (the
  reference's ``Sample`` and ``exact_sample``, ozaki_engine.py:477-521).
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
    """out = (U - 0.5) exp(phi Z): all of U first, then all of Z, each drawn in row chunks (same stream order as
    single draws)."""
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


def _split(a):
    t = 134217729.0 * a
    hi = t - (t - a)
    return hi, a - hi


def exact_sample(Ar, Bc):
    """Correctly rounded Ar @ Bc (float64): Dekker TwoProduct of every term, then math.fsum of all parts."""
    r = Ar.shape[0]
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


class Sample:
    """Sampled accuracy of a product against the correctly rounded reference on a fixed set of rows / columns."""

    def __init__(self, A, B, Cnat=None, nr=48, nc=48, seed=7):
        m, n = A.shape[0], B.shape[1]
        rng = np.random.default_rng(seed)
        ri = set(rng.choice(m, min(nr, m), replace=False).tolist())
        ci = set(rng.choice(n, min(nc, n), replace=False).tolist())
        if Cnat is not None:
            ri.add(int(torch.abs(Cnat).max(dim=1).values.argmax().item()))
            ci.add(int(torch.abs(Cnat).max(dim=0).values.argmax().item()))
        self.ri = np.array(sorted(ri))
        self.ci = np.array(sorted(ci))
        dev = A.device
        Ar = A[torch.as_tensor(self.ri, device=dev)].cpu().numpy()
        Bc = B[:, torch.as_tensor(self.ci, device=dev)].cpu().numpy()
        self.ref = exact_sample(Ar, Bc)
        self.absab = np.abs(Ar) @ np.abs(Bc)
        self.den1 = np.abs(self.ref).max()
        self.tri = torch.as_tensor(self.ri, device=dev)
        self.tci = torch.as_tensor(self.ci, device=dev)

    def errors(self, C):
        Cs = C[self.tri][:, self.tci].cpu().numpy()
        d = np.abs(Cs - self.ref)
        with np.errstate(all="ignore"):
            e2 = np.where(self.absab > 0, d / self.absab, 0.0)
        return {"E1": float(d.max() / self.den1) if self.den1 > 0 else float(d.max()), "E2": float(e2.max())}


def make_inputs_w(n, seed=0):
    """The reference's rotated ill-scaled family W (make_inputs_ext, ozaki_engine.py:1618-1631), from numpy's generator:
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


def audit_bound(S, info, k, C, scale=1.0):
    """Lemma L1 audit on a Sample (the reference's audit_bound, ozaki_engine.py:1755-1766): |C_hat - C_ref| against
    scale E_ij(p) + 2^-53 (|C_hat| + |C_ref|); returns violations and the worst ratio."""
    from .constants import bound_matrix
    h, p = info["stats"], info["p"]
    Eb = scale * bound_matrix(h["r"], h["c"], h["sA"], h["sB"], k, p, S.ri, S.ci)
    Cs = C[S.tri][:, S.tci].cpu().numpy()
    err = np.abs(Cs - S.ref)
    lim = Eb * (1 + 1e-9) + 2.0 ** -53 * (np.abs(Cs) + np.abs(S.ref)) * (1 + 1e-9)
    nz = err > 0
    return {"max_err_over_bound": float((err / lim).max()), "violations": int((err > lim).sum()),
            "median_bound_over_err": float(np.median(Eb[nz] / err[nz])) if nz.any() else None,
            "max_err_over_D": float((err / S.absab).max())}
