"""``PersistA``: the persistent fixed operand mode of the reference (dl1683/matrix-numbers code/ozaki_engine.py:
2417-2466) on this library's kernels.

A is encoded ONCE at a fixed (N, p) with inside scaling off (gamma = 0): its row statistics and its N residue planes
stay in the engine's buffers.  Every product A B_j then pays only the B-side statistics, the forced rule (which
re-checks on the device that p is still within the exact range for B_j's norms), the B residues, the N INT8 products
and the reconstruction -- one CUDA graph per (B, C) pair, as the reference captures it.

    P = PersistA(E, A, B0, n)      # runs E.run(A, B0, inside=False): the a-priori rule on B0 fixes (N, p)
    P.encode()                      # A's statistics and residue planes
    P.product(B, C)                 # C = A B for any B of shape (k, n), finite

Same contract as the reference: B must be finite (no non-finite check in this mode), and the buffers are the engine's
own for the shape (m, n, k), so an ordinary ``E.run`` on the same shape between ``encode`` and ``product`` overwrites
the encoded operand.  When B_j's norms make p unsafe, the forced rule lowers the device p and sets the fallback flag,
exactly as the reference's ``_rule_device`` does (:1387-1396); the reference reads neither, and ``product`` does not
either (it returns without a host synchronisation).  ``last_decision()`` reads them for callers that want the check.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr
from .engine import DEV, _stream_handle


class PersistA:
    def __init__(self, E, A, B0, B_shape_n):
        self.E, self.A = E, A
        m, k = A.shape
        self.n = B_shape_n
        C0 = torch.empty(m, self.n, dtype=torch.float64, device=DEV)
        _, info = E.run(A, B0, C=C0, inside=False)          # the a-priori rule on the first product fixes (N, p)
        if info.get("fallback"):
            raise ValueError("PersistA: the first product falls back to native FP64 (non-finite input or no plane "
                             "count within range); there is no (N, p) to fix")
        self.N, self.p = info["N"], info["p"]
        self.b = E.buffers(m, self.n, k, max(self.N, 20))
        self.C = None
        self.graphs = {}

    def encode(self):
        """gamma = 0, A's row statistics (r, sA, nA) and its residue planes at the fixed p (:2433-2442)."""
        E, A, b = self.E, self.A, self.b
        m, k = A.shape
        st = _stream_handle()
        b["gam"].zero_()
        b["flag"].zero_()                                      # B is assumed finite in this mode
        check(E.lib.ozk_stats_rows(ptr(A), m, k, ptr(b["gam"]), ptr(b["r"]), ptr(b["sA"]), ptr(b["nA"]), st),
              "ozk_stats_rows")
        b["pdev"].fill_(self.p)
        check(E.lib.ozk_split_a(ptr(A), ptr(b["r"]), ptr(b["gam"]), ptr(b["pdev"]), m, k, self.N, ptr(b["Ares"]),
                                ptr(b["err"]), st),
              "ozk_split_a")
        E.launches += 1 + _lib.split_kernels(A, b["Ares"], m, k, False)

    def _stats_B(self, B):
        """B's column statistics for gamma = 0, then the forced rule (N, p): the device p drops (and the fallback
        flag is set) if p exceeds the exact range for this B (:2444-2454)."""
        E, b = self.E, self.b
        k, n = B.shape
        check(E.lib.ozk_stats_cols(ptr(B), k, n, ptr(b["gam"]), ptr(b["c"]), ptr(b["sB"]), ptr(b["nB"]),
                                   ptr(b["ws_stats"]), b["ws_stats"].numel(), _stream_handle()), "ozk_stats_cols")
        E.launches += 2
        E._rule_device(self.A, B, b, 2.0 ** -52, 2.0, self.N, self.p)

    def product(self, B, C):
        """C = A B with the encoded A (graph per (B, C) pair, captured on first use)."""
        E, b = self.E, self.b
        assert B.dtype == torch.float64 and B.is_contiguous() and tuple(B.shape) == (self.A.shape[1], self.n)
        assert C.dtype == torch.float64 and C.is_contiguous() and tuple(C.shape) == (self.A.shape[0], self.n)
        key = (B.data_ptr(), C.data_ptr())
        gr = self.graphs.get(key)
        if gr is None:
            gr = E._capture(lambda: (self._stats_B(B), E.core(self.A, B, b, self.N, C, skipA=True)))
            self.graphs[key] = gr
        gr.replay()
        E.launches += 9
        return C

    def last_decision(self):
        """(N, p, fallback) of the forced rule of the last product (synchronises)."""
        dec, words, _ = self.b.fetch()
        return dec.N, int(words[5]), dec.fallback


__all__ = ["PersistA"]
