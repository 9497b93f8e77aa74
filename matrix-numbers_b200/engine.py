"""``OzakiCRT``: drop-in replacement of the reference engine's Python entry point on B200.

The public surface is that of ``OzakiCRT`` in dl1683/matrix-numbers code/ozaki_engine.py (:1150-1505): the
constructor, ``run``, ``run_fast``, ``stats``, ``choose``, ``core``, ``buffers``, ``kernels``, ``_rule_device``, their
arguments, return values, ``info`` keys and error conventions.  Every computation is a call into libozaki_b200.so
(sm_100a kernels behind the C ABI of include/ozaki_b200.h); torch provides device memory, streams and CUDA graphs.

    E = OzakiCRT()
    C, info = E.run(A, B)                 # eager: statistics -> device rule -> one host read -> core
    C, info = E.run(A, B, C, graph=True)  # timed path: [graph: statistics + rule] -> read (N, p) -> [graph: core]

A, B: float64 CUDA tensors, row-major, A (m, k), B (k, n), with m % 4 == 0, n % 32 == 0, k % 32 == 0 (the
reference's shape rule, :1315; its k <= 131071 limit does not apply: the products are accumulated exactly in
segments of 65536).  Non-finite input, N > 32 or an unsafe forced p give the native FP64 product (torch.matmul, cuBLAS
DGEMM) with ``info["fallback"] = True``, as in the reference.

How this engine is organised (its own design; only the interface follows the reference):

* ``Workspace`` -- the device scratch of one problem shape.  The statistics, the decision block and the rule / stats
  workspaces are sized by the shape alone; the residue planes (A, B and the products' residues) live in a separate
  ``PlaneStore`` whose capacity grows on demand.  Growing the planes keeps the statistics, so a plane count above
  the capacity costs one reallocation and no second statistics pass.  Item access gives the reference's buffer keys
  (``ws["r"]``, ``ws["pdev"]``, ``ws["N"]``, ...).
* ``Decision`` -- (N, p, fallback, p_req) as the device rule wrote them into the decision block; ``Workspace.fetch``
  copies the block to pinned memory, synchronises once and raises if any INT8 GEMM launch set the device error word.
* ``_Request`` -- the rule's arguments (tau, safety, inside scaling, forced N / p, seed, certify) as one hashable
  value: the graph caches are keyed by it.
* the core is one function, ``_launch_core``, over a row range of C; ``core`` runs it on all rows, the host-buffer
  paths on row blocks whose D2H copies overlap the next block's work.

Differences from the reference: the eager path's rule runs on the device as well (the reference's ``choose`` runs it
on the host in numpy; both apply the same comparisons, csrc/rule.cu); every kernel is compiled ahead of time
(``kernels(N)`` compiles nothing); statistics are reduced in a fixed order (the reference's column sums use double
atomics); the core reads the device p, so a forced p is written into the decision block.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr
from .constants import MODS, NEG, NMAX, limbs_for, modulus_product, pmax_bits

DEV = "cuda"
DEFAULT_PLANES = 20          # capacity of a new plane store: the largest plane count the rule picks on ordinary data
TAU = 2.0 ** -52

# slots of the int32 decision block written by the device rule (csrc/rule.cu) and read by the core kernels
_N, _P, _FALLBACK, _PREQ, _ERR, _PCORE = 0, 1, 2, 3, 4, 5
_CTL_WORDS = 8
# slots of the float64 auxiliary block: nu_A, nu_B, worst E/D on the probe, probe rows, probe columns
_AUX_WORDS = 8


def _stream_handle(stream=None) -> int:
    """cudaStream_t handle of a torch stream (default: the current stream), or an int handle passed through."""
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream if hasattr(s, "cuda_stream") else int(s)


@dataclass(frozen=True)
class Decision:
    N: int
    p: int
    fallback: bool
    p_req: int

    @property
    def native(self) -> bool:
        """True when the product must be the native FP64 one (the rule found no plane count, or non-finite input)."""
        return self.fallback or self.N == 0


@dataclass(frozen=True)
class _Request:
    tau: float = TAU
    safety: float = 2.0
    inside: bool = True
    force_N: Optional[int] = None
    force_p: Optional[int] = None
    seed: int = 0
    certify: bool = False

    @property
    def forced(self) -> bool:
        return self.force_N is not None


class PlaneStore:
    """Residue planes of one shape, ``capacity`` planes each: A (capacity, m, k) and B (capacity, n, k) as int8 with k
    contiguous (the K-major operands of the INT8 products), the products' residues X (capacity, m, n) as uint8."""

    def __init__(self, m, n, k, capacity):
        self.capacity = capacity
        self.A = torch.empty(capacity * m * k, dtype=torch.int8, device=DEV)
        self.B = torch.empty(capacity * n * k, dtype=torch.int8, device=DEV)
        self.X = torch.empty(capacity * m * n, dtype=torch.uint8, device=DEV)


class Workspace:
    """Engine-owned device scratch for one (m, n, k).  See the module docstring."""

    _ALIASES = {"Ares": "planes_A", "Bres": "planes_B", "X": "planes_X", "N": "capacity", "dec": "decision",
                "err": "error_word", "pdev": "p_core", "ctl": "control"}

    def __init__(self, lib, m, n, k, planes):
        self.shape = (m, n, k)
        # int32 arena: gamma[k] | r[m] | c[n] | non-finite flag | decision block
        i32 = torch.empty(k + m + n + 1 + _CTL_WORDS, dtype=torch.int32, device=DEV)
        self.gam, self.r, self.c = i32[:k], i32[k:k + m], i32[k + m:k + m + n]
        self.flag = i32[k + m + n:k + m + n + 1]
        self.control = i32[k + m + n + 1:]
        self.control.zero_()
        self.decision = self.control[_N:_PREQ + 1]
        self.error_word = self.control[_ERR:_ERR + 1]
        self.p_core = self.control[_PCORE:_PCORE + 1]
        # float64 arena: sA[m] | nA[m] | sB[n] | nB[n] | auxiliary outputs of the rule
        f64 = torch.zeros(2 * m + 2 * n + _AUX_WORDS, dtype=torch.float64, device=DEV)
        self.sA, self.nA = f64[:m], f64[m:2 * m]
        self.sB, self.nB = f64[2 * m:2 * m + n], f64[2 * m + n:2 * m + 2 * n]
        self.aux = f64[2 * m + 2 * n:]
        self.ws_stats = torch.empty(max(1, lib.ozk_stats_workspace_bytes(m, n, k)), dtype=torch.uint8, device=DEV)
        self.ws_rule = torch.empty(max(1, lib.ozk_rule_workspace_bytes(m, n, k)), dtype=torch.uint8, device=DEV)
        # pinned mirrors for the one host read per call
        self._h_control = torch.zeros(_CTL_WORDS, dtype=torch.int32).pin_memory()
        self._h_aux = torch.zeros(_AUX_WORDS, dtype=torch.float64).pin_memory()
        self._h_i32 = torch.empty(m + n + 1, dtype=torch.int32).pin_memory()
        self._h_f64 = torch.empty(2 * m + 2 * n, dtype=torch.float64).pin_memory()
        self._i32_stats = i32[k:k + m + n + 1]               # r | c | flag, contiguous
        self._f64_stats = f64[:2 * m + 2 * n]
        self.planes = PlaneStore(m, n, k, planes)

    # reference-compatible item access (b["r"], b["pdev"], b["N"], ...)
    def __getitem__(self, key):
        return getattr(self, self._ALIASES.get(key, key))

    @property
    def capacity(self) -> int:
        return self.planes.capacity

    @property
    def planes_A(self):
        return self.planes.A

    @property
    def planes_B(self):
        return self.planes.B

    @property
    def planes_X(self):
        return self.planes.X

    def grow(self, planes) -> bool:
        """Make room for ``planes`` planes; True if the plane buffers were replaced (graphs that use them are stale)."""
        if planes <= self.planes.capacity:
            return False
        m, n, k = self.shape
        self.planes = None
        torch.cuda.empty_cache()
        self.planes = PlaneStore(m, n, k, max(planes, DEFAULT_PLANES))
        return True

    def set_p(self, p: int):
        self.p_core.fill_(int(p))

    def fetch(self, stream=None):
        """Copy the decision block and the rule's auxiliary outputs to the host (one synchronisation) -> (Decision,
        control words, aux list).  Raises OzkError if a split, INT8 product or reconstruction launch has set the device
        error word."""
        s = torch.cuda.current_stream() if stream is None else stream
        with torch.cuda.stream(s):
            self._h_control.copy_(self.control, non_blocking=True)
            self._h_aux.copy_(self.aux, non_blocking=True)
        s.synchronize()
        words = self._h_control.tolist()
        self.raise_on_device_error(words[_ERR])
        return Decision(int(words[_N]), int(words[_P]), bool(words[_FALLBACK]), int(words[_PREQ])), words, \
            self._h_aux.tolist()

    @staticmethod
    def raise_on_device_error(word: int):
        if word:
            raise _lib.OzkError(f"device error flag {word:#x} raised by a split, product or reconstruction launch (a "
                                "bounded wait ran out); the results of that call are invalid")

    def host_stats(self):
        """(statistics dict of numpy arrays, non-finite flag) read from the device (synchronises)."""
        m, n, _ = self.shape
        self._h_i32.copy_(self._i32_stats, non_blocking=True)
        self._h_f64.copy_(self._f64_stats, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        hi, hd = self._h_i32.numpy(), self._h_f64.numpy()
        stats = {"r": hi[:m].copy(), "c": hi[m:m + n].copy(), "sA": hd[:m].copy(), "nA": hd[m:2 * m].copy(),
                 "sB": hd[2 * m:2 * m + n].copy(), "nB": hd[2 * m + n:].copy()}
        return stats, bool(hi[m + n])


class _StageClock:
    """CUDA events between the parts of a call, recorded only when a sink (dict or list) is given."""

    def __init__(self, sink):
        self.sink = sink
        self.marks = []

    def mark(self, name):
        if self.sink is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        if isinstance(self.sink, list):
            self.sink.append((name, e))
        else:
            self.marks.append((name, e))

    def flush(self):
        """Add the seconds between consecutive marks to the dict sink (synchronises)."""
        if not isinstance(self.sink, dict) or len(self.marks) < 2:
            return
        torch.cuda.synchronize()
        for (_, a), (name, b) in zip(self.marks[:-1], self.marks[1:]):
            self.sink[name] = self.sink.get(name, 0.0) + a.elapsed_time(b) / 1e3


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
        self.bufs = {}               # (m, n, k) -> Workspace
        self.graphs = {}             # captured CUDA graphs, keyed by what they were captured for
        self.probe = {}              # random probe rows / columns per (m, n, seed)
        self.launches = 0            # kernels launched by this engine (the benchmark's launch count)
        self._host = {}              # device slots and copy streams of the host-buffer paths

    # ---- per-N tables: compiled into the library ------------------------------------------------------------------
    def kernels(self, N):
        """The reference compiles kernels per plane count here (:1177-1201); this library is compiled ahead of time,
        so only the plane count's limb count and modulus product are recorded."""
        if N not in self.per_n:
            self.per_n[N] = {"N": N, "L": limbs_for(N), "M": modulus_product(N)}
        return self.per_n[N]

    # ---- scratch --------------------------------------------------------------------------------------------------
    def buffers(self, m, n, k, N) -> Workspace:
        """The workspace of shape (m, n, k) with room for at least N planes (created or grown on demand)."""
        shape = (m, n, k)
        ws = self.bufs.get(shape)
        if ws is None:
            ws = Workspace(self.lib, m, n, k, max(int(N), DEFAULT_PLANES))
            self.bufs[shape] = ws
        elif ws.grow(int(N)):
            self._forget_graphs(lambda key: key[1] == shape and key[0] in ("core", "config"))
        return ws

    def _forget_graphs(self, stale):
        for key in [k_ for k_ in self.graphs if stale(k_)]:
            del self.graphs[key]

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
        """Random part of the probe set, as the reference draws it (RandomState(seed).choice without replacement,
        rows then columns, :1265-1267, :1397-1403); device tensors cached per shape and seed."""
        key = (m, n, seed)
        cached = self.probe.get(key)
        if cached is None:
            draw = np.random.RandomState(seed)
            rows = draw.choice(m, min(64, m), replace=False)
            cols = draw.choice(n, min(64, n), replace=False)
            cached = tuple(torch.as_tensor(v, dtype=torch.int64, device=DEV) for v in (rows, cols))
            self.probe[key] = cached
        return cached

    # ---- stage 1: statistics ---------------------------------------------------------------------------------------
    def stats(self, A, B, b, inside=True, stream=None):
        m, k = A.shape
        n = B.shape[1]
        check(self.lib.ozk_stats(ptr(A), ptr(B), m, n, k, int(bool(inside)), ptr(b.gam), ptr(b.r), ptr(b.c),
                                 ptr(b.sA), ptr(b.nA), ptr(b.sB), ptr(b.nB), ptr(b.flag), ptr(b.ws_stats),
                                 b.ws_stats.numel(), _stream_handle(stream)), "ozk_stats")
        self.launches += 6

    # ---- stage 2: the a-priori rule on the device ------------------------------------------------------------------
    def _rule_device(self, A, B, b, tau, safety, force_N=None, force_p=None, seed=0, stream=None):
        m, k = A.shape
        n = B.shape[1]
        rows, cols = self._probe_sets(m, n, seed)
        check(self.lib.ozk_rule(ptr(A), ptr(B), m, n, k, ptr(b.r), ptr(b.c), ptr(b.sA), ptr(b.nA), ptr(b.sB),
                                ptr(b.nB), ptr(b.flag), ptr(rows), rows.numel(), ptr(cols), cols.numel(), float(tau),
                                float(safety), int(force_N or 0), -1 if force_p is None else int(force_p),
                                ptr(b.decision), ptr(b.p_core), ptr(b.aux), ptr(b.ws_rule), b.ws_rule.numel(),
                                _stream_handle(stream)), "ozk_rule")
        self.launches += 5 if force_N else 6

    def _rule_certified(self, A, B, b, tau, safety):
        """The rule from the full-matrix certificate instead of the probe: one FP16 tensor-core product bounds D on
        every entry (csrc/certificate.cu), then N and p on the device (``ozk_rule_certified``)."""
        from .certificate import certificate_device
        m, k = A.shape
        n = B.shape[1]
        w = certificate_device(self, A, B, b.gam, b.r, b.c, b.sA, b.sB, tau, safety)
        check(self.lib.ozk_rule_certified(ptr(b.nA), ptr(b.nB), ptr(b.flag), m, n, k, ptr(w["xmin"]),
                                          ptr(b.decision), ptr(b.p_core), ptr(b.aux), _stream_handle()),
              "ozk_rule_certified")
        self.launches += 1
        return w

    def _decide(self, A, B, b, req: _Request):
        """Statistics, then the rule the request asks for (device only; nothing is read back)."""
        self.stats(A, B, b, req.inside)
        if req.certify:
            self._rule_certified(A, B, b, req.tau, req.safety)
        else:
            self._rule_device(A, B, b, req.tau, req.safety, req.force_N, req.force_p, seed=req.seed)

    @staticmethod
    def _decide_launches(req: _Request) -> int:
        # statistics (6) + sampled rule (6, 5 when N is forced) or certificate (4) + certified rule (1)
        return 11 if (req.forced or req.certify) else 12

    def check_errors(self):
        """Raise if any split, INT8 product or reconstruction launch of this engine reported a device-side error
        (synchronises)."""
        for ws in self.bufs.values():
            ws.fetch()

    def choose(self, A, B, b, tau=TAU, force_N=None, seed=0, safety=2.0, prof=None):
        """The a-priori rule (:1250-1307), evaluated on the device from statistics already in ``b`` (``stats``);
        returns (N, p, info, host statistics) like the reference, N = p = None on fallback."""
        t_start = time.perf_counter()
        self._rule_device(A, B, b, tau, safety, force_N, None, seed=seed)
        dec, _, aux = b.fetch()
        host, nonfinite = b.host_stats()
        info = {"nonfinite": nonfinite}
        if nonfinite:
            info["fallback"] = True
            return None, None, info, host
        info["nuA"], info["nuB"] = aux[0], aux[1]
        if force_N is not None:
            return int(force_N), dec.p, info, host
        info.update({"probe": [int(aux[3]), int(aux[4])], "worst_ratio_E_over_D": aux[2], "p_req": dec.p_req})
        if prof is not None:
            prof["rule_host"] = time.perf_counter() - t_start
        if dec.native:
            info["fallback"] = True
            return None, None, info, host
        return dec.N, dec.p, info, host

    # ---- stage 3: residues, INT8 products with the fused reduction, reconstruction ---------------------------------
    def _launch_core(self, A, B, b, N, C, row_begin=0, row_end=None, with_B=True, with_A=True, stream=None,
                     clock=None):
        """The core on rows [row_begin, row_end) of C: split of those rows of A (unless with_A is False: planes
        already encoded), split of B (unless with_B is False: planes of an earlier block), the N INT8 products with
        their fused mod-m_t reduction, the reconstruction into C's rows."""
        m, k = A.shape
        n = B.shape[1]
        row_end = m if row_end is None else row_end
        rows = row_end - row_begin
        st = _stream_handle(stream)
        mark = clock.mark if clock is not None else (lambda _name: None)
        A_rows, r_rows, C_rows = A[row_begin:row_end], b.r[row_begin:row_end], C[row_begin:row_end]
        launched = 0
        if with_A:
            check(self.lib.ozk_split_a(ptr(A_rows), ptr(r_rows), ptr(b.gam), ptr(b.p_core), rows, k, N,
                                       ptr(b.planes_A), ptr(b.error_word), st), "ozk_split_a")
            launched += _lib.split_kernels(A_rows, b.planes_A, rows, k, False)
        if with_B:
            check(self.lib.ozk_split_b(ptr(B), ptr(b.c), ptr(b.gam), ptr(b.p_core), k, n, N, ptr(b.planes_B),
                                       ptr(b.error_word), st),
                  "ozk_split_b")
            launched += _lib.split_kernels(B, b.planes_B, n, k, True)
        mark("residues")
        check(self.lib.ozk_gemm_residues(ptr(b.planes_A), ptr(b.planes_B), rows, n, k, N, ptr(b.planes_X),
                                         ptr(b.error_word), st), "ozk_gemm_residues")
        mark("gemm+reduce")
        check(self.lib.ozk_reconstruct(ptr(b.planes_X), ptr(r_rows), ptr(b.c), ptr(b.p_core), rows, n, N, ptr(C_rows),
                                       ptr(b.error_word), st), "ozk_reconstruct")
        mark("recon")
        self.launches += launched + 2

    def core(self, A, B, b, N, C, stream=None, prof=None, skipA=False):
        """Residue split, INT8 products, reconstruction for N planes at the device p (:1310-1350)."""
        m, k = A.shape
        n = B.shape[1]
        assert k % 4 == 0 and n % 32 == 0 and m % 4 == 0 and (m * n) % 4 == 0 and k % 32 == 0
        assert 1 <= N <= NMAX and b.capacity >= N
        clock = _StageClock(prof)
        clock.mark("start")
        self._launch_core(A, B, b, N, C, with_A=not skipA, stream=stream, clock=clock)
        clock.flush()
        return C

    # ---- CUDA graphs -------------------------------------------------------------------------------------------------
    def _capture(self, body):
        """Run ``body`` once eagerly on a side stream (warm-up), then capture it on that stream."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            body()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            body()
        return graph

    def _graph(self, key, body):
        g = self.graphs.get(key)
        if g is None:
            g = self.graphs[key] = self._capture(body)
        return g

    def core_graph(self, A, B, b, N, C):
        m, k = A.shape
        n = B.shape[1]
        key = ("core", (m, n, k), N, A.data_ptr(), B.data_ptr(), C.data_ptr())
        self._graph(key, lambda: self._launch_core(A, B, b, N, C)).replay()
        self.launches += 4

    # ---- public entry points ---------------------------------------------------------------------------------------
    def run_fast(self, A, B, C, tau=TAU, safety=2.0, inside=True, force_N=None, force_p=None, events=None,
                 certify=False):
        """Timed path: [graph: statistics + rule] -> one host read of (N, p) -> [graph: residues, products, recon].
        ``events`` (a list) receives (name, CUDA event) marks after each part, for stage timing inside a run.
        ``certify``: the rule is the full-matrix certificate (every entry) instead of the 96 x 96 probe."""
        self._shape_check(A, B, C)
        if force_N is not None and force_p is not None:
            return self._run_config(A, B, C, tau, safety, inside, int(force_N), int(force_p), events)
        req = _Request(float(tau), float(safety), bool(inside), None if certify else force_N,
                       None if certify else force_p, 0, bool(certify))
        m, k = A.shape
        n = B.shape[1]
        ws = self.buffers(m, n, k, DEFAULT_PLANES)
        clock = _StageClock(events)
        clock.mark("start")
        self._graph(("decide", (m, n, k), A.data_ptr(), B.data_ptr(), req),
                    lambda: self._decide(A, B, ws, req)).replay()
        clock.mark("stats+rule")
        self.launches += self._decide_launches(req)
        dec, _, _ = ws.fetch()
        clock.mark("host read")
        if dec.native:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": dec.p_req}
        self.buffers(m, n, k, dec.N)           # more planes than the store holds: grow it (statistics stay valid)
        self.core_graph(A, B, ws, dec.N, C)
        clock.mark("core")
        out = {"N": dec.N, "p": dec.p, "preq": dec.p_req}
        if certify:
            out["certified"] = True
        return C, out

    def _run_config(self, A, B, C, tau, safety, inside, N, p, events=None):
        """Configuration-table fast path (N and p both given, e.g. by pick_config): ONE graph of statistics, the
        forced rule (no probe product), the core for N planes and the copy of the decision block to pinned memory,
        then one synchronisation.  The reference's graph path reads (N, p) on the host between two graphs
        (:1432-1457); with N known beforehand nothing in the core depends on that read.  If the forced rule rejects
        the configuration (p above the data's exact range) or the input is not finite, the core's output is
        discarded and C is recomputed natively, as the reference does."""
        if not 1 <= N <= NMAX:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": 0}
        m, k = A.shape
        n = B.shape[1]
        req = _Request(float(tau), float(safety), bool(inside), N, p)
        ws = self.buffers(m, n, k, N)

        def body():
            self._decide(A, B, ws, req)
            self._launch_core(A, B, ws, N, C)
            ws._h_control.copy_(ws.control, non_blocking=True)

        clock = _StageClock(events)
        clock.mark("start")
        self._graph(("config", (m, n, k), A.data_ptr(), B.data_ptr(), C.data_ptr(), req), body).replay()
        self.launches += 15
        torch.cuda.current_stream().synchronize()
        clock.mark("stats+rule+core")
        words = ws._h_control.tolist()
        ws.raise_on_device_error(words[_ERR])
        if words[_FALLBACK] or words[_N] == 0:
            torch.matmul(A, B, out=C)
            return C, {"fallback": True, "preq": int(words[_PREQ])}
        return C, {"N": int(words[_N]), "p": int(words[_P]), "preq": int(words[_PREQ])}

    def _run_certified(self, A, B, C, tau, inside, safety=2.0):
        m, k = A.shape
        n = B.shape[1]
        ws = self.buffers(m, n, k, DEFAULT_PLANES)
        req = _Request(float(tau), float(safety), bool(inside), certify=True)
        self.stats(A, B, ws, req.inside)
        cert = self._rule_certified(A, B, ws, req.tau, req.safety)
        dec, _, aux = ws.fetch()
        cert_err = int(cert["err"].item())
        if cert_err:
            raise _lib.OzkError(f"ozk_certificate: device error flag {cert_err:#x} (a bounded wait ran out)")
        host, nonfinite = ws.host_stats()
        info = {"nonfinite": nonfinite, "certified": True, "nuA": aux[0], "nuB": aux[1], "p_req": dec.p_req,
                "uncertified_entries": int(cert["unc"].item())}
        if dec.native:
            info["fallback"] = True
            torch.matmul(A, B, out=C)
            return C, info
        self.buffers(m, n, k, dec.N)
        info.update({"N": dec.N, "p": dec.p, "L": limbs_for(dec.N), "stats": host})
        self.core(A, B, ws, dec.N, C)
        return C, info

    def _run_eager(self, A, B, C, req: _Request, prof=None):
        """The eager call (:1460-1505 semantics): statistics, the device rule with a host read of its outcome and the
        host statistics, then the core; a forced p above the rule's exact range is a rejected configuration."""
        m, k = A.shape
        n = B.shape[1]
        ws = self.buffers(m, n, k, req.force_N or DEFAULT_PLANES)
        wall0 = time.perf_counter()
        clock = _StageClock({} if prof is not None else None)
        clock.mark("start")
        self.stats(A, B, ws, req.inside)
        clock.mark("stats_gpu")
        N, p, info, host = self.choose(A, B, ws, req.tau, req.force_N, req.seed, safety=req.safety, prof=prof)
        if prof is not None:
            clock.flush()
            prof.update(clock.sink)
            prof["stats+rule_wall"] = time.perf_counter() - wall0
        rejected = N is not None and req.force_p is not None and req.force_p > p
        if N is None or rejected:
            info["fallback"] = True
            if rejected:
                info["config_rejected"] = True
            torch.matmul(A, B, out=C)
            return C, info
        if req.force_p is not None:
            p = int(req.force_p)
        self.buffers(m, n, k, N)
        ws.set_p(p)
        info.update({"N": N, "p": p, "L": limbs_for(N), "stats": host})
        self.core(A, B, ws, N, C, prof=prof)
        return C, info

    def run(self, A, B, C=None, tau=TAU, force_N=None, inside=True, graph=False, prof=None, seed=0, config=None,
            force_p=None, certify=False):
        """C = A B in emulated FP64; returns (C, info).  ``config`` ({'N':.., 'p':..}, e.g. from pick_config) overrides
        the a-priori rule.  ``certify=True`` (not in the reference's run) replaces the sampled probe by the
        full-matrix certificate of every entry (certificate.py); info then carries ``certified``, ``p_req`` (the
        certificate's) and ``uncertified_entries``."""
        if config is not None:
            force_N, force_p = int(config["N"]), config.get("p")
        self._shape_check(A, B, C)
        if C is None:
            C = torch.empty(A.shape[0], B.shape[1], dtype=torch.float64, device=DEV)
        if graph:
            return self.run_fast(A, B, C, tau=tau, inside=inside, force_N=force_N, force_p=force_p, certify=certify)
        if certify and force_N is None:
            return self._run_certified(A, B, C, tau, inside)
        req = _Request(float(tau), 2.0, bool(inside), None if force_N is None else int(force_N),
                       None if force_p is None else int(force_p), int(seed))
        return self._run_eager(A, B, C, req, prof)

    # ---- host buffers ----------------------------------------------------------------------------------------------
    def _host_slots(self, m, n, k, count):
        """``count`` device slots (A, B, C) for the host-buffer paths and their input / output copy streams; one set
        per shape, replaced when the shape changes, a second slot added when a stream of products first needs it."""
        state = self._host.get((m, n, k))
        if state is None:
            self._host.clear()
            state = self._host[(m, n, k)] = {"slots": [], "h2d": torch.cuda.Stream(), "d2h": torch.cuda.Stream()}
        while len(state["slots"]) < count:
            state["slots"].append({"A": torch.empty((m, k), dtype=torch.float64, device=DEV),
                                   "B": torch.empty((k, n), dtype=torch.float64, device=DEV),
                                   "C": torch.empty((m, n), dtype=torch.float64, device=DEV)})
        return state

    def run_host(self, A_h, B_h, C_h=None, tau=TAU, safety=2.0, inside=True, force_N=None, force_p=None, blocks=4):
        """C_h = A_h B_h for host (CPU, ideally pinned) float64 tensors; returns (C_h, info) with C_h filled.

        The H2D copies of A and B come first (the statistics need all of both); after the rule the core runs in
        ``blocks`` row blocks of C, and each finished block is copied back on a second stream while the next block
        computes.  Results equal ``run``'s bit for bit."""
        return self.run_host_many([(A_h, B_h, C_h)], tau=tau, safety=safety, inside=inside, force_N=force_N,
                                  force_p=force_p, blocks=blocks)[0]

    def run_host_many(self, jobs, tau=TAU, safety=2.0, inside=True, force_N=None, force_p=None, blocks=4):
        """A stream of host-buffer products: ``jobs`` is a list of (A_h, B_h, C_h) float64 CPU tensors of one shape
        (pinned for overlap; C_h None to allocate); returns [(C_h, info), ...], each equal to ``run``'s bit for bit.

        A single product cannot overlap its input copies with its compute (the statistics need all of A and B), but
        a stream can: with two device slots the H2D copies of job i + 1 run on their own stream while job i computes,
        and job i's row blocks of C go back on a third stream (PCIe carries both directions at once).  Job i + 1's
        copies are issued before job i's one blocking read of (N, p).  Before returning, the device error word of the
        INT8 products is read: a bounded wait that ran out raises OzkError instead of returning invalid C."""
        if not jobs:
            return []
        m, k = jobs[0][0].shape
        n = jobs[0][1].shape[1]
        for A_h, B_h, _ in jobs:
            assert A_h.dtype == torch.float64 and B_h.dtype == torch.float64
            assert tuple(A_h.shape) == (m, k) and tuple(B_h.shape) == (k, n), "all jobs must have one shape"
        io = self._host_slots(m, n, k, min(2, len(jobs)))
        slots, h2d, d2h = io["slots"], io["h2d"], io["d2h"]
        self._shape_check(slots[0]["A"], slots[0]["B"], slots[0]["C"])
        req = _Request(float(tau), float(safety), bool(inside), None if force_N is None else int(force_N),
                       None if force_p is None else int(force_p))
        compute = torch.cuda.current_stream()
        h2d.wait_stream(compute)
        d2h.wait_stream(compute)
        outs = [C_h if C_h is not None else torch.empty((m, n), dtype=torch.float64, pin_memory=True)
                for _, _, C_h in jobs]
        loaded = [torch.cuda.Event() for _ in slots]
        released = [None] * len(slots)       # per slot: (inputs consumed, output copied) events of its last job

        def load(i):
            s = i % len(slots)
            if released[s] is not None:
                h2d.wait_event(released[s][0])
            with torch.cuda.stream(h2d):
                slots[s]["A"].copy_(jobs[i][0], non_blocking=True)
                slots[s]["B"].copy_(jobs[i][1], non_blocking=True)
            loaded[s].record(h2d)

        block_rows = ((-(-m // blocks) + 127) // 128) * 128        # whole 128-row tiles per block
        ws = self.buffers(m, n, k, req.force_N or DEFAULT_PLANES)
        load(0)
        results = []
        for i, C_h in enumerate(outs):
            s = i % len(slots)
            A, B, C = slots[s]["A"], slots[s]["B"], slots[s]["C"]
            if i + 1 < len(jobs):
                load(i + 1)
            compute.wait_event(loaded[s])
            if released[s] is not None:
                compute.wait_event(released[s][1])
            self._decide(A, B, ws, req)
            self.launches += self._decide_launches(req)
            dec, _, _ = ws.fetch()
            if dec.native:
                torch.matmul(A, B, out=C)
                spans = [(0, m)]
                info = {"fallback": True, "preq": dec.p_req}
            else:
                self.buffers(m, n, k, dec.N)
                spans = [(r0, min(m, r0 + block_rows)) for r0 in range(0, m, block_rows)]
                info = {"N": dec.N, "p": dec.p, "preq": dec.p_req, "blocks": len(spans)}
            for bi, (r0, r1) in enumerate(spans):
                if not dec.native:
                    self._launch_core(A, B, ws, dec.N, C, r0, r1, with_B=bi == 0)
                done = torch.cuda.Event()
                done.record(compute)
                d2h.wait_event(done)
                with torch.cuda.stream(d2h):
                    C_h[r0:r1].copy_(C[r0:r1], non_blocking=True)
            consumed, copied = torch.cuda.Event(), torch.cuda.Event()
            consumed.record(compute)
            copied.record(d2h)
            released[s] = (consumed, copied)
            results.append((C_h, info))
        compute.wait_stream(d2h)
        compute.wait_stream(h2d)
        ws.fetch(compute)                      # synchronises; raises if a product's bounded wait ran out
        return results


__all__ = ["OzakiCRT", "Workspace", "Decision", "DEV", "MODS", "NMAX", "NEG", "pmax_bits"]
