"""C row-block sharding of the FP64-on-INT8 GEMM over the ranks of a torch.distributed process group.

The reference engine runs on one GPU only (dl1683/matrix-numbers code/ozaki_engine.py:443, :531).  Output rows are
independent once the statistics are global, so rank g owns rows [g m/G, (g+1) m/G) of A and C and B is present on
every rank (or broadcast from one rank first, ``b_root``).  One call makes these collective steps, in this order on
every rank:

  1. all_reduce(MAX) of the per-column max |A| bit patterns (k int64)  -> the global inside scaling gamma;
  2. all_gather of the row statistics (r, sA, nA; 20 bytes per row)     -> every rank builds the same probe set
     (64 random rows + the 32 globally hardest rows) and the same nu_A;
  3. all_reduce(SUM) of the probe product D (96 x 96 doubles; each rank fills the probe rows it owns, zeros elsewhere)
     -> every rank makes the same decision (N, p) from the same numbers;
then each rank splits its A rows and B into residue planes, runs the N INT8 products and reconstructs its C rows --
no further communication.  The result equals the single-GPU product bit for bit (same gamma, r, c, N, p, and the CRT
stage is exact).

Compute is delegated to an ``ops`` object: ``CudaOps`` (default) calls libozaki_b200.so on the rank's GPU; the CPU
tests substitute an implementation with the same interface to check the orchestration over gloo ranks.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, ptr


class CudaOps:
    """Per-rank compute on the current CUDA device through the C ABI (include/ozaki_b200.h)."""

    def __init__(self):
        from .engine import OzakiCRT
        self.engine = OzakiCRT()
        self.lib = self.engine.lib
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._glob = {}

    @property
    def launches(self):
        return self.engine.launches

    def _stream(self):
        return torch.cuda.current_stream().cuda_stream

    def buffers(self, rows, n, k, N):
        return self.engine.buffers(rows, n, k, N)

    def colmax(self, A):
        rows, k = A.shape
        out = torch.empty(k, dtype=torch.int64, device=A.device)
        check(self.lib.ozk_stats_colmax(ptr(A), rows, k, ptr(out), self._stream()), "ozk_stats_colmax")
        self.engine.launches += 1
        return out

    def stats_finish(self, A, B, colmax, inside):
        rows, k = A.shape
        n = B.shape[1]
        b = self.engine.buffers(rows, n, k, 20)
        check(self.lib.ozk_stats_finish(ptr(A), ptr(B), rows, n, k, 1 if inside else 0, ptr(colmax), ptr(b["gam"]),
                                        ptr(b["r"]), ptr(b["c"]), ptr(b["sA"]), ptr(b["nA"]), ptr(b["sB"]), ptr(b["nB"]),
                                        ptr(b["flag"]), ptr(b["ws_stats"]), b["ws_stats"].numel(), self._stream()),
              "ozk_stats_finish")
        self.engine.launches += 5
        return {"gam": b["gam"], "r": b["r"], "sA": b["sA"], "nA": b["nA"], "c": b["c"], "sB": b["sB"], "nB": b["nB"],
                "flag": b["flag"], "_b": b}

    def global_rows(self, m, device):
        g = self._glob.get(m)
        if g is None:
            g = {"r": torch.empty(m, dtype=torch.int32, device=device),
                 "sA": torch.empty(m, dtype=torch.float64, device=device),
                 "nA": torch.empty(m, dtype=torch.float64, device=device)}
            self._glob[m] = g
        return g

    def rule_prepare(self, st, glob, m, n, k, Ir, Jr, force_N, force_p):
        b = st["_b"]
        ws = b.setdefault("ws_rule_global_" + str(m), torch.empty(max(1, self.lib.ozk_rule_workspace_bytes(m, n, k)),
                                                                    dtype=torch.uint8, device=self.device))
        check(self.lib.ozk_rule_prepare(ptr(glob["r"]), ptr(st["c"]), ptr(glob["sA"]), ptr(glob["nA"]), ptr(st["sB"]),
                                        ptr(st["nB"]), ptr(st["flag"]), m, n, k, ptr(Ir), Ir.numel(), ptr(Jr), Jr.numel(),
                                        int(force_N or 0), -1 if force_p is None else int(force_p), ptr(b["dec"]),
                                        ptr(b["pdev"]), ptr(b["aux"]), ptr(ws), ws.numel(), self._stream()),
              "ozk_rule_prepare")
        self.engine.launches += 1
        return {"ws": ws, "b": b, "m": m, "n": n, "k": k}

    def rule_probe(self, h, A, B, row_begin):
        rows = A.shape[0]
        ws = h["ws"]
        check(self.lib.ozk_rule_probe(ptr(A), ptr(B), row_begin, rows, h["m"], h["n"], h["k"], ptr(ws), ws.numel(),
                                      self._stream()), "ozk_rule_probe")
        self.engine.launches += 2
        off = self.lib.ozk_rule_probe_offset(h["m"], h["n"], h["k"])
        return ws[off:off + 96 * 96 * 8].view(torch.float64)

    def rule_finish(self, h, st, glob, tau, safety):
        b = h["b"]
        check(self.lib.ozk_rule_finish(ptr(glob["r"]), ptr(st["c"]), ptr(glob["sA"]), ptr(st["sB"]), h["m"], h["n"],
                                       h["k"], float(tau), float(safety), ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]),
                                       ptr(h["ws"]), h["ws"].numel(), self._stream()), "ozk_rule_finish")
        self.engine.launches += 1
        ctl, aux = self.engine._read_ctl(b)
        return ctl[0], ctl[1], ctl[2], ctl[3], aux

    def core(self, A, B, st, N, p, C):
        rows, k = A.shape
        n = B.shape[1]
        b = self.engine.buffers(rows, n, k, N)
        if b is not st["_b"]:          # grown: copy the statistics into the new buffers
            for x in ("gam", "r", "c", "sA", "nA", "sB", "nB", "flag"):
                b[x].copy_(st[x])
        b["pdev"].fill_(p)
        self.engine.core(A, B, b, N, C)
        return C

    def native(self, A, B, C):
        torch.matmul(A, B, out=C)
        return C


class DistributedOzakiCRT:
    """``run(A_local, B, C_local)``: this rank's rows of C = A B, with the plane count and scalings of the whole
    product.  Every rank must call ``run`` with the same shapes and arguments (A_local: equal row counts)."""

    def __init__(self, group=None, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ops = ops if ops is not None else CudaOps()
        self.probe = {}

    @property
    def engine(self):
        return self.ops.engine

    @property
    def launches(self):
        return self.ops.launches

    def _probe_sets(self, m, n, seed, device):
        key = (m, n, seed, str(device))
        if key not in self.probe:
            rs = np.random.RandomState(seed)
            Ir = rs.choice(m, min(64, m), replace=False)
            Jr = rs.choice(n, min(64, n), replace=False)
            self.probe[key] = (torch.as_tensor(Ir, dtype=torch.int64, device=device),
                               torch.as_tensor(Jr, dtype=torch.int64, device=device))
        return self.probe[key]

    def run(self, A, B, C=None, tau=2.0 ** -52, force_N=None, inside=True, seed=0, force_p=None, safety=2.0,
            b_root=None, config=None):
        if config is not None:
            force_N, force_p = int(config["N"]), config.get("p")
        rows, k = A.shape
        n = B.shape[1]
        assert B.shape[0] == k and rows % 4 == 0 and n % 32 == 0 and k % 32 == 0, "shape rule (per rank)"
        m = rows * self.world
        row_begin = rows * self.rank
        if C is None:
            C = torch.empty((rows, n), dtype=torch.float64, device=A.device)
        if b_root is not None:
            dist.broadcast(B, src=b_root, group=self.group)
        # 1. global column max of |A|
        cm = self.ops.colmax(A)
        dist.all_reduce(cm, op=dist.ReduceOp.MAX, group=self.group)
        st = self.ops.stats_finish(A, B, cm, inside)
        # 2. row statistics of all ranks
        glob = self.ops.global_rows(m, A.device)
        dist.all_gather_into_tensor(glob["r"], st["r"].contiguous(), group=self.group)
        dist.all_gather_into_tensor(glob["sA"], st["sA"].contiguous(), group=self.group)
        dist.all_gather_into_tensor(glob["nA"], st["nA"].contiguous(), group=self.group)
        # 3. probe product summed over the row blocks, then the same decision everywhere
        Ir, Jr = self._probe_sets(m, n, seed, A.device)
        h = self.ops.rule_prepare(st, glob, m, n, k, Ir, Jr, force_N, force_p)
        D = self.ops.rule_probe(h, A, B, row_begin)
        dist.all_reduce(D, op=dist.ReduceOp.SUM, group=self.group)
        N, p, fb, preq, aux = self.ops.rule_finish(h, st, glob, tau, safety)
        if fb or N == 0:
            self.ops.native(A, B, C)
            return C, {"fallback": True, "preq": preq}
        self.ops.core(A, B, st, N, p, C)
        return C, {"N": N, "p": p, "preq": preq, "rows": [row_begin, row_begin + rows], "world": self.world}


__all__ = ["DistributedOzakiCRT", "CudaOps", "_lib"]
