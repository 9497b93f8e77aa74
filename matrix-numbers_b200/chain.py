"""Exact integer product chains A_1 A_2 ... A_q kept in INT8 residue form on the GPU.

The reference models the cost of such chains (dl1683/matrix-numbers code/digit_gemm.py:1252-1291, ``cmd_chain``):
with one INT8 GEMM per modulus per product and the residues reduced after every product, a chain of q matrices costs
(q - 1) N GEMMs on a fixed base of N moduli, where the product of the moduli must exceed 2 R_q and R_q bounds the
chain's entries.  This module executes that model with the engine's kernels and moduli (the first N of MODS):

  1. the first matrix is split into N symmetric INT8 residue planes (the split kernel at scale 2^0: every entry is an
     integer, so round(v 2^0) = v and the planes are v mod m_t);
  2. each further matrix is split the same way as a right operand, and ``ozk_gemm_residues`` forms
     X[t] = (left_t right_t^T) mod m_t in [0, m_t) -- the INT32 products never leave TMEM;
  3. between products ``ozk_residue_symmetric`` maps X[t] back to the symmetric int8 range, so the running product
     never leaves the device or the residue form;
  4. the last product's planes are reconstructed by CRT into the correctly rounded double of the exact integer
     result (the reconstruction kernel at scale 2^0); the planes themselves, the exact result in residue form, can
     be returned too.

The number of moduli N is the fewest of MODS whose product exceeds 2 R, with R = prod_s max|A_s| x prod of the inner
dimensions (or the reference model's H^q k^(q-1) with H = 2^b - 1 when ``b`` is given); the 32 moduli of the engine
cap R at about 2^245.
"""
from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import check, ptr
from .constants import MODS, NMAX

_P_UNIT = 64          # split / reconstruction scaling exponent: r_i = c_j = p gives the scale 2^0


def planes_for(bound: int):
    """Fewest N <= 32 with prod(MODS[:N]) > 2 bound (the chain's fixed base), or None if even 32 moduli are too few."""
    prod = 1
    for N in range(1, NMAX + 1):
        prod *= MODS[N - 1]
        if prod > 2 * int(bound):
            return N
    return None


def chain_bound(maxabs, inner_dims) -> int:
    """R = prod_s max|A_s| x prod of the inner dimensions: |(A_1 ... A_q)_ij| <= R."""
    return math.prod(int(h) for h in maxabs) * math.prod(int(k) for k in inner_dims)


class ResidueChain:
    """``product(mats)``: the exact product of integer-valued float64 CUDA matrices, computed in residue form."""

    def __init__(self):
        self.lib = _lib.lib()
        self.launches = 0

    @staticmethod
    def _check(mats):
        if len(mats) < 2:
            raise ValueError("a chain needs at least two matrices")
        for s, A in enumerate(mats):
            if A.dtype != torch.float64 or not A.is_cuda or A.dim() != 2 or not A.is_contiguous():
                raise ValueError(f"matrix {s}: float64 CUDA contiguous 2-D tensor required")
            if s and A.shape[0] != mats[s - 1].shape[1]:
                raise ValueError(f"matrix {s}: inner dimensions do not match")
        m = mats[0].shape[0]
        dims = [A.shape[1] for A in mats]
        assert m % 4 == 0 and all(d % 32 == 0 for d in [mats[0].shape[1]] + dims), \
            "shape rule: rows % 4 == 0, every other dimension % 32 == 0"

    def product(self, mats, b=None, N=None, return_residues=False, stream=None):
        """Returns (C, info): C = the correctly rounded double of the exact integer product (float64, m x n); info
        has N, the bound's log2, the GEMM count (q - 1) N and, with ``return_residues``, ``residues`` = the final
        planes X[t] = C_exact mod m_t (uint8, N x m x n).  Entries must be integers of magnitude below 2^53."""
        self._check(mats)
        inner = [A.shape[1] for A in mats[:-1]]
        if b is not None:
            R = (2 ** int(b) - 1) ** len(mats) * math.prod(inner)
        else:
            maxabs = []
            for s, A in enumerate(mats):
                h = A.abs().max().item()
                if not math.isfinite(h) or h >= 2.0 ** 53 or not bool(torch.equal(A, torch.round(A))):
                    raise ValueError(f"matrix {s}: entries must be finite integers below 2^53 in magnitude")
                maxabs.append(int(h))
            R = chain_bound(maxabs, inner)
        need = planes_for(R)
        if N is None:
            N = need
        if N is None or N > NMAX:
            raise ValueError(f"chain bound 2^{math.log2(max(R, 1)):.1f} exceeds the product of the {NMAX} moduli")
        dev = mats[0].device
        st = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
        m = mats[0].shape[0]
        kmax = max(A.shape[0] for A in mats)
        nmax = max(A.shape[1] for A in mats)
        pdev = torch.full((1,), _P_UNIT, dtype=torch.int32, device=dev)
        gam = torch.zeros(kmax, dtype=torch.int32, device=dev)
        rows = torch.full((m,), _P_UNIT, dtype=torch.int32, device=dev)
        cols = torch.full((nmax,), _P_UNIT, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        k1 = mats[0].shape[1]
        left = torch.empty((N, m, k1), dtype=torch.int8, device=dev)
        check(self.lib.ozk_split_a(ptr(mats[0]), ptr(rows), ptr(gam), ptr(pdev), m, k1, N, ptr(left), ptr(err), st),
              "ozk_split_a")
        self.launches += _lib.split_kernels(mats[0], left, m, k1, False)
        X = None
        for s in range(1, len(mats)):
            k, n = mats[s].shape
            right = torch.empty((N, n, k), dtype=torch.int8, device=dev)
            check(self.lib.ozk_split_b(ptr(mats[s]), ptr(cols), ptr(gam), ptr(pdev), k, n, N, ptr(right), ptr(err),
                                       st),
                  "ozk_split_b")
            X = torch.empty((N, m, n), dtype=torch.uint8, device=dev)
            check(self.lib.ozk_gemm_residues(ptr(left), ptr(right), m, n, k, N, ptr(X), ptr(err), st),
                  "ozk_gemm_residues")
            self.launches += _lib.split_kernels(mats[s], right, n, k, True) + 1
            if s + 1 < len(mats):
                left = torch.empty((N, m, n), dtype=torch.int8, device=dev)
                check(self.lib.ozk_residue_symmetric(ptr(X), N, m * n, ptr(left), st), "ozk_residue_symmetric")
                self.launches += 1
            del right
        n = mats[-1].shape[1]
        C = torch.empty((m, n), dtype=torch.float64, device=dev)
        check(self.lib.ozk_reconstruct(ptr(X), ptr(rows), ptr(cols), ptr(pdev), m, n, N, ptr(C), ptr(err), st),
              "ozk_reconstruct")
        self.launches += 1
        if int(err.item()):
            raise RuntimeError(f"residue chain: device error flags {int(err.item())}")
        info = {"N": N, "N_needed": need, "bound_log2": math.log2(max(R, 1)), "products": len(mats) - 1,
                "gemms": (len(mats) - 1) * N}
        if return_residues:
            info["residues"] = X
        return C, info


__all__ = ["ResidueChain", "planes_for", "chain_bound"]
