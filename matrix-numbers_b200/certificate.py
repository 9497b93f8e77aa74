"""Full-matrix certificate of the plane count (the reference's ``full_certificate``, dl1683/matrix-numbers
code/ozaki_engine.py:1542-1583) on the library's tcgen05 FP16 kernel (``ozk_certificate``, csrc/certificate.cu).

The sampled a-priori rule checks the error bound E_ij(p) <= tau D_ij / safety on 96 x 96 probe entries; this checks
it on ALL m x n entries, with a lower bound of D_ij = sum_l |A_il||B_lj| from one FP16 tensor-core product of the
scaled magnitudes.  The m x n bound matrix is reduced inside the GEMM epilogue (min over entries), so the cost is one
FP16 GEMM and nothing of size m x n is written.

    C, info = E.run(A, B)                    # eager run: info holds the statistics and the sampled rule
    cert = full_certificate(E, A, B, info)   # same keys as the reference's dict
"""
from __future__ import annotations

import math

import torch

from ._lib import check, ptr
from .constants import NMAX, pmax_bits
from .engine import DEV, _stream_handle


def _workspace(E, m, n, k):
    cache = E.__dict__.setdefault("_cert_ws", {})
    ws = cache.get((m, n, k))
    if ws is None:
        cache.clear()
        ws = {"ws": torch.empty(max(1, E.lib.ozk_certificate_workspace_bytes(m, n, k)), dtype=torch.uint8, device=DEV),
              "xmin": torch.empty(1, dtype=torch.float64, device=DEV),
              "unc": torch.zeros(1, dtype=torch.int64, device=DEV),
              "err": torch.zeros(1, dtype=torch.int32, device=DEV)}
        cache[(m, n, k)] = ws
    return ws


def certificate_device(E, A, B, gam, r, c, sA, sB, tau=2.0 ** -52, safety=2.0, D_out=None, stream=None):
    """Launch ``ozk_certificate`` for device statistics; returns the workspace dict whose ``xmin`` (float64 bit
    pattern, all ones when no entry is certified) and ``unc`` (uncertified entries) hold the result on the device."""
    m, k = A.shape
    n = B.shape[1]
    w = _workspace(E, m, n, k)
    check(E.lib.ozk_certificate(ptr(A), ptr(B), m, n, k, ptr(gam), ptr(r), ptr(c), ptr(sA), ptr(sB), float(tau),
                                float(safety), ptr(w["xmin"]), ptr(w["unc"]), 0 if D_out is None else ptr(D_out),
                                ptr(w["err"]), ptr(w["ws"]), w["ws"].numel(), _stream_handle(stream)), "ozk_certificate")
    E.launches += 4                                   # 2^gamma tables, FP16 A and B, the product
    return w


def required_p(xmin_bits: int):
    """ceil(-log2(min xmax) + 1e-9), the reference's preq_full (:1570-1573); -1e30 stands for 'no certified entry'."""
    if xmin_bits == -1:                               # all bits set: no entry with D > 0
        need = -1e30
    else:
        x = torch.tensor([xmin_bits], dtype=torch.int64).view(torch.float64)
        need = float(-torch.log2(x.to(DEV)).item())   # CUDA log2, as the reference evaluates it
    return int(math.ceil(need + 1e-9)), need


def full_certificate(E, A, B, info, tau=2.0 ** -52, safety=2.0):
    """FULL-matrix certificate of E_ij(p) <= tau D_ij / safety for ALL (i, j), for an eager ``run`` whose ``info``
    holds the statistics.  Returns the reference's dict: N_full, preq_full, preq_sampled, uncertified_entries,
    cost_ms, N_sampled, sampled_config_fully_certified."""
    m, k = A.shape
    n = B.shape[1]
    h = info["stats"]
    b = E.buffers(m, n, k, 20)
    E.stats(A, B, b, True)                            # gamma of the configuration being certified (inside scaling on)
    torch.cuda.synchronize()
    r = torch.as_tensor(h["r"], device=DEV, dtype=torch.int32)
    c = torch.as_tensor(h["c"], device=DEV, dtype=torch.int32)
    sA = torch.as_tensor(h["sA"], device=DEV, dtype=torch.float64)
    sB = torch.as_tensor(h["sB"], device=DEV, dtype=torch.float64)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    w = certificate_device(E, A, B, b["gam"], r, c, sA, sB, tau, safety)
    e1.record()
    torch.cuda.synchronize()
    if int(w["err"].item()):
        raise RuntimeError(f"ozk_certificate: device error flag {int(w['err'].item()):#x} (a bounded wait ran out)")
    unc = int(w["unc"].item())
    preq, _ = required_p(int(w["xmin"].view(torch.int64).item()))
    nuA, nuB = info["nuA"], info["nuB"]
    N_full = next((N for N in range(6, NMAX + 1) if pmax_bits(N, nuA, nuB, k) >= preq), None)
    N_s = info.get("N")
    return {"N_full": N_full, "preq_full": preq, "preq_sampled": info.get("p_req"), "uncertified_entries": unc,
            "cost_ms": e0.elapsed_time(e1), "N_sampled": N_s,
            "sampled_config_fully_certified": bool(unc == 0 and N_full is not None and N_s is not None
                                                   and N_s >= N_full)}


__all__ = ["full_certificate", "certificate_device", "required_p"]
