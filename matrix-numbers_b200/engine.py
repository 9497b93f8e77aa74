"""``OzakiCRT``: drop-in replacement of the reference engine's Python entry point on B200.

Same constructor, methods, arguments, return values and error conventions as ``OzakiCRT`` in
dl1683/matrix-numbers code/ozaki_engine.py (:1150-1505); every stage runs in libozaki_b200.so (sm_100a kernels,
include/ozaki_b200.h), torch provides the device buffers, the stream and the CUDA graphs.

    E = OzakiCRT()
    C, info = E.run(A, B)                 # eager: stats -> device rule -> one host read -> core
    C, info = E.run(A, B, C, graph=True)  # timed path: [graph: stats + rule] -> host read of (N, p) -> [graph: core]

A, B: float64 CUDA tensors, row-major, A (m, k), B (k, n), with m % 4 == 0, n % 32 == 0, k % 32 == 0 (the
reference's shape rule, :1315; its k <= 131071 limit does not apply here: the products are accumulated exactly in
segments of 65536).  Non-finite input, N > 32 or an unsafe forced p fall back to native FP64 (torch.matmul, cuBLAS
DGEMM) with ``info["fallback"] = True``, as the reference does.

Differences from the reference: the rule of the eager path runs on the device too (the reference's ``choose`` runs it
on the host in numpy; both apply the same mathematics, see csrc/rule.cu); every kernel is compiled ahead of time
(``kernels(N)`` compiles nothing); statistics are reduced in a fixed order (the reference's column sums use double
atomics).
"""
from __future__ import annotations

import time

import numpy as np
import torch

from . import _lib
from .constants import MODS, NEG, NMAX, limbs_for, modulus_product, pmax_bits
from ._lib import check, ptr

DEV = "cuda"


def _stream_handle(stream=None) -> int:
    """cudaStream_t handle of a torch stream (default: the current stream), or an int handle passed through."""
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream if hasattr(s, "cuda_stream") else int(s)


class OzakiCRT:
    """FP64 GEMM from INT8 residue-plane products and CRT reconstruction (Ozaki scheme II) on B200."""

    def __init__(self, lt=None):
        # `lt` (the reference's cuBLASLt wrapper) is accepted for signature compatibility and unused: the INT8
        # products are this library's own tcgen05 kernel.
        self.lib = _lib.lib()
        if not torch.cuda.is_available():
            raise _lib.OzkError("OzakiCRT needs a CUDA device (B200, sm_100a); there is no CPU path")
        major, _ = torch.cuda.get_device_capability()
        if major != 10:
            raise _lib.OzkError(f"OzakiCRT is built for sm_100a (B200); the current device has compute capability {major}.x")
        self.per_n = {}
        self.bufs = {}
        self.graphs = {}
        self.probe = {}
        self.Mvec = torch.tensor([modulus_product(N) for N in range(6, NMAX + 1)], dtype=torch.float64, device=DEV)
        self.launches = 0   # kernels launched by this engine (for the benchmark's launch count)

    # ---- kernels: compiled ahead of time, the per-N tables live in the library ---------------------------------
    def kernels(self, N):
        d = self.per_n.get(N)
        if d is None:
            d = {"N": N, "L": limbs_for(N)}
            self.per_n[N] = d
        return d

    # ---- buffers (engine-owned scratch, grown on demand; growing clears the captured graphs) -------------------
    def buffers(self, m, n, k, N):
        key = (m, n, k)
        b = self.bufs.get(key)
        if b is None or b["N"] < N:
            self.bufs.pop(key, None)
            self.graphs.clear()
            b = None
            torch.cuda.empty_cache()
            cap = max(N, 20)
            bi = torch.empty(m + n + 1, dtype=torch.int32, device=DEV)          # r | c | flag
            bd = torch.empty(2 * m + 2 * n, dtype=torch.float64, device=DEV)    # sA | nA | sB | nB
            ctl = torch.zeros(8, dtype=torch.int32, device=DEV)                 # N, p, fallback, p_req | err | p
            b = {"N": cap,
                 "Ares": torch.empty(cap * m * k, dtype=torch.int8, device=DEV),
                 "Bres": torch.empty(cap * n * k, dtype=torch.int8, device=DEV),
                 "X": torch.empty(cap * m * n, dtype=torch.uint8, device=DEV),
                 "gam": torch.empty(k, dtype=torch.int32, device=DEV),
                 "bi": bi, "bd": bd, "r": bi[:m], "c": bi[m:m + n], "flag": bi[m + n:],
                 "sA": bd[:m], "nA": bd[m:2 * m], "sB": bd[2 * m:2 * m + n], "nB": bd[2 * m + n:],
                 "ctl": ctl, "dec": ctl[0:4], "err": ctl[4:5], "pdev": ctl[5:6],
                 "aux": torch.zeros(8, dtype=torch.float64, device=DEV),
                 "ws_stats": torch.empty(max(1, self.lib.ozk_stats_workspace_bytes(m, n, k)), dtype=torch.uint8, device=DEV),
                 "ws_rule": torch.empty(max(1, self.lib.ozk_rule_workspace_bytes(m, n, k)), dtype=torch.uint8, device=DEV),
                 "hi": torch.empty(m + n + 1, dtype=torch.int32).pin_memory(),
                 "hd": torch.empty(2 * m + 2 * n, dtype=torch.float64).pin_memory(),
                 "hctl": torch.zeros(8, dtype=torch.int32).pin_memory(),
                 "haux": torch.zeros(8, dtype=torch.float64).pin_memory()}
            self.bufs[key] = b
        return b

    @staticmethod
    def _shape_check(A, B, C=None):
        assert A.dtype == torch.float64 and B.dtype == torch.float64, "A and B must be float64"
        assert A.is_cuda and B.is_cuda and A.is_contiguous() and B.is_contiguous(), "A and B must be contiguous CUDA tensors"
        m, k = A.shape
        k2, n = B.shape
        assert k == k2, "inner dimensions differ"
        assert k % 32 == 0 and n % 32 == 0 and m % 4 == 0, "shape rule: k % 32 == 0, n % 32 == 0, m % 4 == 0"
        if C is not None:
            assert C.dtype == torch.float64 and C.is_contiguous() and tuple(C.shape) == (m, n), "C must be (m, n) float64"

    def _probe_sets(self, m, n, seed):
        """Random part of the probe set: RandomState(seed).choice without replacement, rows then columns
        (ozaki_engine.py:1265-1267, :1397-1403); cached per shape and seed."""
        key = ("probe", m, n, seed)
        if key not in self.probe:
            rs = np.random.RandomState(seed)
            Ir = rs.choice(m, min(64, m), replace=False)
            Jr = rs.choice(n, min(64, n), replace=False)
            self.probe[key] = (torch.as_tensor(Ir, dtype=torch.int64, device=DEV),
                               torch.as_tensor(Jr, dtype=torch.int64, device=DEV))
        return self.probe[key]

    # ---- stage 1: statistics ---------------------------------------------------------------------------------
    def stats(self, A, B, b, inside=True, stream=None):
        m, k = A.shape
        n = B.shape[1]
        st = _stream_handle(stream)
        rc = self.lib.ozk_stats(ptr(A), ptr(B), m, n, k, 1 if inside else 0, ptr(b["gam"]), ptr(b["r"]), ptr(b["c"]),
                                ptr(b["sA"]), ptr(b["nA"]), ptr(b["sB"]), ptr(b["nB"]), ptr(b["flag"]),
                                ptr(b["ws_stats"]), b["ws_stats"].numel(), st)
        check(rc, "ozk_stats")
        self.launches += 6

    # ---- stage 2: the a-priori rule on the device ---------------------------------------------------------------
    def _rule_device(self, A, B, b, tau, safety, force_N=None, force_p=None, seed=0, stream=None):
        m, k = A.shape
        n = B.shape[1]
        Ir, Jr = self._probe_sets(m, n, seed)
        rc = self.lib.ozk_rule(ptr(A), ptr(B), m, n, k, ptr(b["r"]), ptr(b["c"]), ptr(b["sA"]), ptr(b["nA"]),
                               ptr(b["sB"]), ptr(b["nB"]), ptr(b["flag"]), ptr(Ir), Ir.numel(), ptr(Jr), Jr.numel(),
                               float(tau), float(safety), int(force_N or 0),
                               -1 if force_p is None else int(force_p), ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]),
                               ptr(b["ws_rule"]), b["ws_rule"].numel(), _stream_handle(stream))
        check(rc, "ozk_rule")
        self.launches += 5 if force_N else 6

    def _stats_rule(self, A, B, b, tau, safety, inside, force_N=None, force_p=None):
        self.stats(A, B, b, inside)
        self._rule_device(A, B, b, tau, safety, force_N, force_p, seed=0)

    def _rule_certified(self, A, B, b, tau, safety):
        """The rule from the full-matrix certificate instead of the probe: one FP16 tensor-core product bounds D on
        every entry (csrc/certificate.cu), then N, p on the device (``ozk_rule_certified``)."""
        from .certificate import certificate_device
        m, k = A.shape
        n = B.shape[1]
        w = certificate_device(self, A, B, b["gam"], b["r"], b["c"], b["sA"], b["sB"], tau, safety)
        check(self.lib.ozk_rule_certified(ptr(b["nA"]), ptr(b["nB"]), ptr(b["flag"]), m, n, k, ptr(w["xmin"]),
                                          ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]), _stream_handle()),
              "ozk_rule_certified")
        self.launches += 1
        return w

    def _stats_rule_certified(self, A, B, b, tau, safety, inside):
        self.stats(A, B, b, inside)
        self._rule_certified(A, B, b, tau, safety)

    def _read_ctl(self, b):
        b["hctl"].copy_(b["ctl"], non_blocking=True)
        b["haux"].copy_(b["aux"], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        ctl = [int(x) for x in b["hctl"].tolist()]
        if ctl[4]:
            raise _lib.OzkError(f"device error flag {ctl[4]:#x} raised by an earlier INT8 GEMM launch "
                                "(a bounded wait ran out); results of that call are invalid")
        return ctl, b["haux"].tolist()

    def check_errors(self):
        """Raise if any GEMM launch of this engine reported a device-side error (reads the flags; synchronises)."""
        for b in self.bufs.values():
            self._read_ctl(b)

    def host_stats(self, b, m, n):
        b["hi"].copy_(b["bi"], non_blocking=True)
        b["hd"].copy_(b["bd"], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        hi, hd = b["hi"].numpy(), b["hd"].numpy()
        return {"r": hi[:m].copy(), "c": hi[m:m + n].copy(), "sA": hd[:m].copy(), "nA": hd[m:2 * m].copy(),
                "sB": hd[2 * m:2 * m + n].copy(), "nB": hd[2 * m + n:].copy()}, bool(hi[m + n] != 0)

    def choose(self, A, B, b, tau=2.0 ** -52, force_N=None, seed=0, safety=2.0, prof=None):
        """The a-priori rule (ozaki_engine.py:1250-1307), evaluated on the device; returns (N, p, info, host stats)
        like the reference.  The statistics must have been computed (``stats``)."""
        m, k = A.shape
        n = B.shape[1]
        t0 = time.perf_counter()
        self._rule_device(A, B, b, tau, safety, force_N, None, seed=seed)
        ctl, aux = self._read_ctl(b)
        h, nonfinite = self.host_stats(b, m, n)
        info = {"nonfinite": nonfinite}
        if nonfinite:
            info["fallback"] = True
            return None, None, info, h
        info["nuA"], info["nuB"] = aux[0], aux[1]
        N, p, fb, preq = ctl[0], ctl[1], ctl[2], ctl[3]
        if force_N is not None:
            return int(force_N), p, info, h
        info["probe"] = [int(aux[3]), int(aux[4])]
        info["worst_ratio_E_over_D"] = aux[2]
        info["p_req"] = preq
        if prof is not None:
            prof["rule_host"] = time.perf_counter() - t0
        if fb or N == 0:
            info["fallback"] = True
            return None, None, info, h
        return N, p, info, h

    # ---- stage 3: residues, INT8 products with the fused reduction, reconstruction ------------------------------
    def core(self, A, B, b, N, C, stream=None, prof=None, skipA=False):
        m, k = A.shape
        n = B.shape[1]
        assert k % 4 == 0 and n % 32 == 0 and m % 4 == 0 and (m * n) % 4 == 0 and k % 32 == 0
        assert 1 <= N <= NMAX and b["N"] >= N
        st = _stream_handle(stream)
        evs = []

        def mark(name):
            if prof is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                evs.append((name, e))
        mark("start")
        if not skipA:
            check(self.lib.ozk_split_a(ptr(A), ptr(b["r"]), ptr(b["gam"]), ptr(b["pdev"]), m, k, N, ptr(b["Ares"]), st),
                  "ozk_split_a")
        check(self.lib.ozk_split_b(ptr(B), ptr(b["c"]), ptr(b["gam"]), ptr(b["pdev"]), k, n, N, ptr(b["Bres"]), st),
              "ozk_split_b")
        mark("residues")
        check(self.lib.ozk_gemm_residues(ptr(b["Ares"]), ptr(b["Bres"]), m, n, k, N, ptr(b["X"]), ptr(b["err"]), st),
              "ozk_gemm_residues")
        mark("gemm+reduce")
        check(self.lib.ozk_reconstruct(ptr(b["X"]), ptr(b["r"]), ptr(b["c"]), ptr(b["pdev"]), m, n, N, ptr(C), st),
              "ozk_reconstruct")
        mark("recon")
        self.launches += 3 if skipA else 4
        if prof is not None:
            torch.cuda.synchronize()
            for (n0, e0), (n1, e1) in zip(evs[:-1], evs[1:]):
                prof[n1] = prof.get(n1, 0.0) + e0.elapsed_time(e1) / 1e3
        return C

    def _capture(self, fn):
        """Eager warm-up on a side stream, then capture on that stream; returns the CUDAGraph."""
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            fn()
        return g

    def core_graph(self, A, B, b, N, C):
        key = ("core", A.shape[0], B.shape[1], A.shape[1], N, A.data_ptr(), B.data_ptr(), C.data_ptr())
        g = self.graphs.get(key)
        if g is None:
            g = self._capture(lambda: self.core(A, B, b, N, C))
            self.graphs[key] = g
        g.replay()
        self.launches += 4

    def run_fast(self, A, B, C, tau=2.0 ** -52, safety=2.0, inside=True, force_N=None, force_p=None, events=None,
                 certify=False):
        """Timed path: [graph: statistics + rule] -> one host read of (N, p) -> [graph: residues, products, recon].
        ``events`` (a list) receives (name, CUDA event) marks after each part, for stage timing inside a run.
        ``certify``: the rule is the full-matrix certificate (every entry) instead of the 96 x 96 probe."""
        self._shape_check(A, B, C)
        m, k = A.shape
        n = B.shape[1]
        if force_N is not None and force_p is not None:
            return self._run_config(A, B, C, tau, safety, inside, int(force_N), int(force_p), events)
        if certify:
            force_N = force_p = None
        b = self.buffers(m, n, k, 20)
        key = ("sr", m, n, k, A.data_ptr(), B.data_ptr(), tau, safety, inside, force_N, force_p, bool(certify))

        def stats_rule(bb):
            if certify:
                return lambda: self._stats_rule_certified(A, B, bb, tau, safety, inside)
            return lambda: self._stats_rule(A, B, bb, tau, safety, inside, force_N, force_p)
        g = self.graphs.get(key)
        if g is None:
            g = self._capture(stats_rule(b))
            self.graphs[key] = g

        def mark(name):
            if events is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                events.append((name, e))
        mark("start")
        g.replay()
        mark("stats+rule")
        # statistics (6) + sampled rule (6, 5 when N is forced) or certificate (4) + certified rule (1)
        self.launches += 11 if (force_N or certify) else 12
        ctl, _ = self._read_ctl(b)
        mark("host read")
        N, p, fb, preq = ctl[0], ctl[1], ctl[2], ctl[3]
        if fb or N == 0:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": preq}
        if b["N"] < N:
            b = self.buffers(m, n, k, N)
            g = self._capture(stats_rule(b))
            self.graphs[key] = g
            g.replay()
            ctl, _ = self._read_ctl(b)
            N, p = ctl[0], ctl[1]
        self.core_graph(A, B, b, N, C)
        mark("core")
        out = {"N": N, "p": p, "preq": preq}
        if certify:
            out["certified"] = True
        return C, out

    def _run_config(self, A, B, C, tau, safety, inside, N, p, events=None):
        """Configuration-table fast path (N and p both given, e.g. by pick_config): ONE graph of statistics, the
        forced rule (no probe product), the core for N planes and the copy of the decision to pinned host memory,
        then one synchronisation.  The reference's graph path reads (N, p) on the host between two graphs
        (ozaki_engine.py:1432-1457); with N known beforehand nothing in the core depends on that read.  If the
        forced rule rejects the configuration (p above the data's exact range) or the input is not finite, the
        core's output is discarded and C is recomputed natively, as the reference does."""
        m, k = A.shape
        n = B.shape[1]
        if not 1 <= N <= NMAX:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": 0}
        b = self.buffers(m, n, k, N)
        key = ("cfg", m, n, k, A.data_ptr(), B.data_ptr(), C.data_ptr(), tau, safety, inside, N, p)
        g = self.graphs.get(key)
        if g is None:
            def body():
                self._stats_rule(A, B, b, tau, safety, inside, N, p)
                self.core(A, B, b, N, C)
                b["hctl"].copy_(b["ctl"], non_blocking=True)
            g = self._capture(body)
            self.graphs[key] = g
        if events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(("start", e))
        g.replay()
        self.launches += 15
        torch.cuda.current_stream().synchronize()
        if events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(("stats+rule+core", e))
        ctl = [int(x) for x in b["hctl"].tolist()]
        if ctl[4]:
            raise _lib.OzkError(f"device error flag {ctl[4]:#x} raised by an INT8 GEMM launch (a bounded wait ran "
                                "out); the result is invalid")
        Nd, pd, fb, preq = ctl[0], ctl[1], ctl[2], ctl[3]
        if fb or Nd == 0:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": preq}
        return C, {"N": Nd, "p": pd, "preq": preq}

    def _run_certified(self, A, B, C, tau, inside, safety=2.0):
        m, k = A.shape
        n = B.shape[1]
        b = self.buffers(m, n, k, 20)
        if C is None:
            C = torch.empty(m, n, dtype=torch.float64, device=DEV)
        self.stats(A, B, b, inside)
        w = self._rule_certified(A, B, b, tau, safety)
        ctl, aux = self._read_ctl(b)
        if int(w["err"].item()):
            raise _lib.OzkError(f"ozk_certificate: device error flag {int(w['err'].item()):#x} (a bounded wait ran out)")
        h, nonfinite = self.host_stats(b, m, n)
        info = {"nonfinite": nonfinite, "certified": True, "nuA": aux[0], "nuB": aux[1], "p_req": ctl[3],
                "uncertified_entries": int(w["unc"].item())}
        N, p, fb = ctl[0], ctl[1], ctl[2]
        if fb or N == 0:
            info["fallback"] = True
            torch.matmul(A, B, out=C)
            return C, info
        if b["N"] < N:
            b = self.buffers(m, n, k, N)
            self.stats(A, B, b, inside)
        b["pdev"].fill_(p)
        info.update({"N": N, "p": p, "L": limbs_for(N), "stats": h})
        self.core(A, B, b, N, C)
        return C, info

    def run_host(self, A_h, B_h, C_h=None, tau=2.0 ** -52, safety=2.0, inside=True, force_N=None, force_p=None,
                 blocks=4):
        """C_h = A_h B_h for host (CPU, ideally pinned) float64 tensors; returns (C_h, info) with C_h filled.

        The H2D copies of A and B come first (the statistics need all of both); after the rule, the core runs in
        `blocks` row blocks of C and each finished block is copied back on a second stream while the next block
        computes, so only the last block's D2H copy is not hidden.  Results equal ``run``'s bit for bit."""
        m, k = A_h.shape
        n = B_h.shape[1]
        assert A_h.dtype == torch.float64 and B_h.dtype == torch.float64 and B_h.shape[0] == k
        if C_h is None:
            C_h = torch.empty((m, n), dtype=torch.float64, pin_memory=True)
        io = self.__dict__.setdefault("_host_io", {})
        dv = io.get((m, n, k))
        if dv is None:
            io.clear()
            dv = {"A": torch.empty((m, k), dtype=torch.float64, device=DEV),
                  "B": torch.empty((k, n), dtype=torch.float64, device=DEV),
                  "C": torch.empty((m, n), dtype=torch.float64, device=DEV),
                  "copy": torch.cuda.Stream()}
            io[(m, n, k)] = dv
        A, B, C = dv["A"], dv["B"], dv["C"]
        self._shape_check(A, B, C)
        A.copy_(A_h, non_blocking=True)
        B.copy_(B_h, non_blocking=True)
        b = self.buffers(m, n, k, 20 if force_N is None else max(20, int(force_N)))
        self._stats_rule(A, B, b, tau, safety, inside, force_N, force_p)
        ctl, _ = self._read_ctl(b)
        N, p, fb, preq = ctl[0], ctl[1], ctl[2], ctl[3]
        if fb or N == 0:
            torch.matmul(A, B, out=C)
            C_h.copy_(C)
            return C_h, {"fallback": True, "preq": preq}
        if b["N"] < N:
            b = self.buffers(m, n, k, N)
            self._stats_rule(A, B, b, tau, safety, inside, force_N, force_p)
        st = _stream_handle()
        check(self.lib.ozk_split_b(ptr(B), ptr(b["c"]), ptr(b["gam"]), ptr(b["pdev"]), k, n, N, ptr(b["Bres"]), st),
              "ozk_split_b")
        rows = -(-m // blocks)
        rows = ((rows + 127) // 128) * 128                    # whole 128-row tiles per block
        cur = torch.cuda.current_stream()
        cs = dv["copy"]
        r0 = 0
        while r0 < m:
            r1 = min(m, r0 + rows)
            mb = r1 - r0
            check(self.lib.ozk_split_a(ptr(A[r0:r1]), ptr(b["r"][r0:r1]), ptr(b["gam"]), ptr(b["pdev"]), mb, k, N,
                                       ptr(b["Ares"]), st), "ozk_split_a")
            check(self.lib.ozk_gemm_residues(ptr(b["Ares"]), ptr(b["Bres"]), mb, n, k, N, ptr(b["X"]), ptr(b["err"]),
                                             st), "ozk_gemm_residues")
            check(self.lib.ozk_reconstruct(ptr(b["X"]), ptr(b["r"][r0:r1]), ptr(b["c"]), ptr(b["pdev"]), mb, n, N,
                                           ptr(C[r0:r1]), st), "ozk_reconstruct")
            done = torch.cuda.Event()
            done.record(cur)
            cs.wait_event(done)
            with torch.cuda.stream(cs):
                C_h[r0:r1].copy_(C[r0:r1], non_blocking=True)
            # the next block's residues overwrite Ares / X: the copy only reads C, so nothing else to wait for
            r0 = r1
        self.launches += (11 if force_N else 12) + 3 * (-(-m // rows)) + 1
        cur.wait_stream(cs)
        cur.synchronize()
        return C_h, {"N": N, "p": p, "preq": preq, "blocks": -(-m // rows)}

    def run_host_many(self, jobs, tau=2.0 ** -52, safety=2.0, inside=True, force_N=None, force_p=None, blocks=4):
        """A stream of host-buffer products: ``jobs`` is a list of (A_h, B_h, C_h) pinned float64 CPU tensors of one
        shape (C_h None to allocate); returns [(C_h, info), ...], each equal to ``run_host``'s bit for bit.

        A single call cannot overlap its input copies with its products (the statistics need all of A and B), but a
        stream can: the device holds two input slots, and the H2D copies of job i + 1 run on their own stream while
        job i computes and its row blocks of C go back on a third stream (PCIe carries both directions at once).
        Job i + 1's copies are issued before job i's one blocking read of (N, p)."""
        if not jobs:
            return []
        m, k = jobs[0][0].shape
        n = jobs[0][1].shape[1]
        for A_h, B_h, _ in jobs:
            assert A_h.dtype == torch.float64 and B_h.dtype == torch.float64
            assert tuple(A_h.shape) == (m, k) and tuple(B_h.shape) == (k, n), "all jobs must have one shape"
        io = self.__dict__.setdefault("_host_many", {})
        dv = io.get((m, n, k))
        if dv is None:
            io.clear()
            dv = {"slots": [{x: torch.empty(sh, dtype=torch.float64, device=DEV)
                             for x, sh in (("A", (m, k)), ("B", (k, n)), ("C", (m, n)))} for _ in range(2)],
                  "cin": torch.cuda.Stream(), "cout": torch.cuda.Stream()}
            io[(m, n, k)] = dv
        slots, cin, cout = dv["slots"], dv["cin"], dv["cout"]
        self._shape_check(slots[0]["A"], slots[0]["B"], slots[0]["C"])
        cur = torch.cuda.current_stream()
        cin.wait_stream(cur)
        cout.wait_stream(cur)
        in_done = [torch.cuda.Event(), torch.cuda.Event()]
        used = [None, None]                                   # (compute done, D2H done) events of the slot's last job
        outs = [C_h if C_h is not None else torch.empty((m, n), dtype=torch.float64, pin_memory=True)
                for _, _, C_h in jobs]

        def h2d(i):
            s = i % 2
            if used[s] is not None:
                cin.wait_event(used[s][0])                    # the slot's previous job has read its A and B
            with torch.cuda.stream(cin):
                slots[s]["A"].copy_(jobs[i][0], non_blocking=True)
                slots[s]["B"].copy_(jobs[i][1], non_blocking=True)
            in_done[s].record(cin)

        h2d(0)
        results = []
        rows = ((-(-m // blocks) + 127) // 128) * 128         # whole 128-row tiles per block
        for i in range(len(jobs)):
            s = i % 2
            A, B, C, C_h = slots[s]["A"], slots[s]["B"], slots[s]["C"], outs[i]
            if i + 1 < len(jobs):
                h2d(i + 1)
            cur.wait_event(in_done[s])
            if used[s] is not None:
                cur.wait_event(used[s][1])                    # C of the slot's previous job has been copied out
            b = self.buffers(m, n, k, 20 if force_N is None else max(20, int(force_N)))
            self._stats_rule(A, B, b, tau, safety, inside, force_N, force_p)
            ctl, _ = self._read_ctl(b)
            N, p, fb, preq = ctl[0], ctl[1], ctl[2], ctl[3]
            if not (fb or N == 0) and b["N"] < N:
                b = self.buffers(m, n, k, N)
                self._stats_rule(A, B, b, tau, safety, inside, force_N, force_p)
            if fb or N == 0:
                torch.matmul(A, B, out=C)
                cdone = torch.cuda.Event()
                cdone.record(cur)
                cout.wait_event(cdone)
                with torch.cuda.stream(cout):
                    C_h.copy_(C, non_blocking=True)
                info = {"fallback": True, "preq": preq}
            else:
                st = _stream_handle()
                check(self.lib.ozk_split_b(ptr(B), ptr(b["c"]), ptr(b["gam"]), ptr(b["pdev"]), k, n, N, ptr(b["Bres"]),
                                           st), "ozk_split_b")
                r0 = 0
                while r0 < m:
                    r1 = min(m, r0 + rows)
                    mb = r1 - r0
                    check(self.lib.ozk_split_a(ptr(A[r0:r1]), ptr(b["r"][r0:r1]), ptr(b["gam"]), ptr(b["pdev"]), mb, k,
                                               N, ptr(b["Ares"]), st), "ozk_split_a")
                    check(self.lib.ozk_gemm_residues(ptr(b["Ares"]), ptr(b["Bres"]), mb, n, k, N, ptr(b["X"]),
                                                     ptr(b["err"]), st), "ozk_gemm_residues")
                    check(self.lib.ozk_reconstruct(ptr(b["X"]), ptr(b["r"][r0:r1]), ptr(b["c"]), ptr(b["pdev"]), mb, n,
                                                   N, ptr(C[r0:r1]), st), "ozk_reconstruct")
                    done = torch.cuda.Event()
                    done.record(cur)
                    cout.wait_event(done)
                    with torch.cuda.stream(cout):
                        C_h[r0:r1].copy_(C[r0:r1], non_blocking=True)
                    r0 = r1
                self.launches += (11 if force_N else 12) + 3 * (-(-m // rows)) + 1
                info = {"N": N, "p": p, "preq": preq, "blocks": -(-m // rows)}
            cdone, odone = torch.cuda.Event(), torch.cuda.Event()
            cdone.record(cur)
            odone.record(cout)
            used[s] = (cdone, odone)
            results.append((C_h, info))
        cur.wait_stream(cout)
        cur.wait_stream(cin)
        cur.synchronize()
        return results

    def run(self, A, B, C=None, tau=2.0 ** -52, force_N=None, inside=True, graph=False, prof=None, seed=0, config=None,
            force_p=None, certify=False):
        """C = A B in emulated FP64; returns (C, info).  ``config`` ({'N':.., 'p':..}, e.g. from pick_config) overrides
        the a-priori rule (ozaki_engine.py:1460-1505).  ``certify=True`` (not in the reference's run) replaces the
        sampled probe by the full-matrix certificate of every entry (see certificate.py); info then carries
        ``certified``, ``p_req`` (the certificate's) and ``uncertified_entries``."""
        if config is not None:
            force_N, force_p = int(config["N"]), config.get("p")
        self._shape_check(A, B, C)
        m, k = A.shape
        n = B.shape[1]
        if graph:
            if C is None:
                C = torch.empty(m, n, dtype=torch.float64, device=DEV)
            return self.run_fast(A, B, C, tau=tau, inside=inside, force_N=force_N, force_p=force_p, certify=certify)
        if certify and force_N is None:
            return self._run_certified(A, B, C, tau, inside)
        b = self.buffers(m, n, k, force_N or 20)
        if C is None:
            C = torch.empty(m, n, dtype=torch.float64, device=DEV)
        t0 = time.perf_counter()
        if prof is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        self.stats(A, B, b, inside)
        if prof is not None:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
        N, p, info, h = self.choose(A, B, b, tau, force_N, seed, prof=prof)
        if prof is not None:
            prof["stats_gpu"] = e0.elapsed_time(e1) / 1e3
            prof["stats+rule_wall"] = time.perf_counter() - t0
        if N is None:
            info["fallback"] = True
            torch.matmul(A, B, out=C)
            return C, info
        if b["N"] < N:
            b = self.buffers(m, n, k, N)                   # grow (statistics are recomputed)
            self.stats(A, B, b, inside)
        if force_p is not None:
            if force_p > p:                                # unsafe table entry for this data: native fallback
                info["fallback"] = True
                info["config_rejected"] = True
                torch.matmul(A, B, out=C)
                return C, info
            p = int(force_p)
        b["pdev"].fill_(p)
        info.update({"N": N, "p": p, "L": limbs_for(N), "stats": h})
        if graph:
            self.core_graph(A, B, b, N, C)
        else:
            self.core(A, B, b, N, C, prof=prof)
        return C, info


__all__ = ["OzakiCRT", "DEV", "MODS", "NMAX", "NEG", "pmax_bits"]
