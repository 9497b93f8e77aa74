"""The FP64-on-INT8 GEMM over the ranks of a torch.distributed process group, as a 2-D grid of C blocks.

The reference engine runs on one GPU only (dl1683/matrix-numbers code/ozaki_engine.py:443, :531).  Blocks of C are
independent once the statistics are global, so the ranks form an R x S grid: rank g = a S + b holds the row block a
of A (m/R rows, all of k) and the column block b of B (k x n/S, stored contiguously) and computes the block (a, b)
of C.  S = 1 is the plain row-block split (B on every rank); S > 1 also divides the B-side work (its statistics and
residue planes), which otherwise every rank would repeat for the whole of B.  One call makes these collective steps,
in this order on every rank:

  1. all_reduce(MAX) of the per-column max |A| and of the per-row max |B| bit patterns (2 x k int64)
     -> every rank computes the same inside scaling gamma and non-finite flag;
  2. all_gather of the row statistics (r, sA, nA) and of the column statistics (c, sB, nB)
     -> every rank builds the same probe set (64 random + the 32 globally hardest rows / columns) and the same nu;
  3. all_reduce(SUM) of the probe product D (96 x 96 doubles; each rank fills the entries whose probe row and probe
     column it holds, zeros elsewhere) -> every rank makes the same decision (N, p) from the same numbers;
then each rank splits its A rows and B columns into residue planes, runs the N INT8 products and reconstructs its C
block -- no further communication.  With ``certify=True`` step 3 is the full-matrix certificate instead of the probe:
each rank bounds every entry of its own block (the bound of entry (i, j) needs only row i's and column j's
statistics and the global gamma), one all_reduce(MIN) of the blocks' minimum xmax (float64 bit patterns, which order
like the values) gives the minimum over all of C, and one all_reduce(SUM) the uncertified count; every rank then makes
the certified-mode decision from the same numbers.  The result equals the single-GPU product bit for bit (same gamma, r, c, N, p;
the CRT stage is exact).

Where the operands start.  ``run`` takes pre-placed blocks (each rank already holds its rows of A and its columns of
B).  Two more entry points move the operands over NCCL inside the call:

* ``run_broadcast_b`` -- A's row block a lives on the ranks of grid row a and C's blocks on their owners; B lives on
  one root rank and is sent as FP64: whole to every rank on a row-block grid (S = 1), column block b to the ranks of
  grid column b on an R x S grid (one communicator per column group, the root in each; the root's egress stays one
  copy of B, and every rank splits only its n / S columns of B instead of all of them).  Sending the FP64 operand
  moves fewer bytes than its N residue planes would (N k n, N = 16-20).  The sends run on their own communicators
  while the statistics proceed: the root computes B's row maxima and column statistics from its own copy and
  broadcasts those vectors, every rank computes its rows' statistics, and B is waited for only before the probe
  product.
* ``run_from_root`` -- A, B (and C) live on the root only (row-block grid): B's broadcast starts, A's row blocks are
  scattered, the statistics overlap the broadcast as above, and (with ``gather=True``) the row blocks of C are
  gathered back into the root's C.

From host memory, ``run_host_many`` streams products whose operands start in pinned host buffers: with
``shares=True`` each rank loads only its share of its blocks (1 / S of A's row block, 1 / R of B's column block, so
that every byte of A and B crosses PCIe once, spread over all ranks' links), ``gather_shares`` assembles the blocks
with one all_gather per grid row and column, and the next job's loads and the previous job's C block overlap the
product.

Every collective is NCCL's (no peer-memory loads, no TMA multicast): the exchanges are plain operand moves and small
statistics vectors, with no computation to fuse them with.  ``events`` (a list) receives (name, CUDA event) marks
after each phase, for per-stage timing on each rank.

Compute is delegated to an ``ops`` object: ``CudaOps`` (default) calls libozaki_b200.so on the rank's GPU; the CPU
tests substitute an implementation with the same interface to check the orchestration over gloo ranks.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, ptr


def default_grid(world: int):
    """R x S with S = 2 from 4 ranks on (the B-side work halves), else a plain row split."""
    if world >= 4 and world % 2 == 0:
        return world // 2, 2
    return world, 1


class CudaOps:
    """Per-rank compute on the current CUDA device through the C ABI (include/ozaki_b200.h)."""

    def __init__(self):
        from .engine import OzakiCRT
        self.engine = OzakiCRT()
        self.timed = True                                     # phases can be marked with CUDA events
        self.lib = self.engine.lib
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._glob = {}
        self._ws = {}

    @property
    def launches(self):
        return self.engine.launches

    def _stream(self):
        return torch.cuda.current_stream().cuda_stream

    def colmax(self, A):
        rows, k = A.shape
        out = torch.empty(k, dtype=torch.int64, device=A.device)
        check(self.lib.ozk_stats_colmax(ptr(A), rows, k, ptr(out), self._stream()), "ozk_stats_colmax")
        self.engine.launches += 1
        return out

    def rowmax(self, B):
        k, cols = B.shape
        out = torch.empty(k, dtype=torch.int64, device=B.device)
        check(self.lib.ozk_stats_rowmax(ptr(B), k, cols, ptr(out), self._stream()), "ozk_stats_rowmax")
        self.engine.launches += 1
        return out

    def local_stats(self, A, B, colmax, rowmax, inside, cols=None):
        """gamma from the global maxima, then this rank's row statistics of A and column statistics of B.  With
        B None (``cols`` columns) the column statistics are left to the caller (they arrive from the rank that
        holds B)."""
        rows, k = A.shape
        cols = B.shape[1] if B is not None else cols
        b = self.engine.buffers(rows, cols, k, 20)
        st = self._stream()
        check(self.lib.ozk_stats_gamma(ptr(colmax), ptr(rowmax), k, 1 if inside else 0, ptr(b["gam"]), ptr(b["flag"]),
                                       st), "ozk_stats_gamma")
        check(self.lib.ozk_stats_rows(ptr(A), rows, k, ptr(b["gam"]), ptr(b["r"]), ptr(b["sA"]), ptr(b["nA"]), st),
              "ozk_stats_rows")
        self.engine.launches += 2
        if B is not None:
            check(self.lib.ozk_stats_cols(ptr(B), k, cols, ptr(b["gam"]), ptr(b["c"]), ptr(b["sB"]), ptr(b["nB"]),
                                          ptr(b["ws_stats"]), b["ws_stats"].numel(), st), "ozk_stats_cols")
            self.engine.launches += 2
        return {"gam": b["gam"], "r": b["r"], "sA": b["sA"], "nA": b["nA"], "c": b["c"], "sB": b["sB"], "nB": b["nB"],
                "flag": b["flag"], "_b": b}

    def col_stats(self, B, st, colmax, rowmax, inside):
        """Column statistics (c, sB, nB) of all of B (k x n) with this rank's gamma (``st["gam"]``, from the global
        maxima): the root's share of ``run_broadcast_b``."""
        k, n = B.shape
        out = self._glob.get(("cols", k, n))
        if out is None:
            out = {"c": torch.empty(n, dtype=torch.int32, device=B.device),
                   "sB": torch.empty(n, dtype=torch.float64, device=B.device),
                   "nB": torch.empty(n, dtype=torch.float64, device=B.device),
                   "ws": torch.empty(max(1, self.lib.ozk_stats_cols_workspace_bytes(k, n)), dtype=torch.uint8,
                                     device=B.device)}
            self._glob[("cols", k, n)] = out
        check(self.lib.ozk_stats_cols(ptr(B), k, n, ptr(st["gam"]), ptr(out["c"]), ptr(out["sB"]), ptr(out["nB"]),
                                      ptr(out["ws"]), out["ws"].numel(), self._stream()), "ozk_stats_cols")
        self.engine.launches += 2
        return out

    def global_stats(self, m, n, device):
        g = self._glob.get((m, n))
        if g is None:
            g = {"r": torch.empty(m, dtype=torch.int32, device=device),
                 "sA": torch.empty(m, dtype=torch.float64, device=device),
                 "nA": torch.empty(m, dtype=torch.float64, device=device),
                 "c": torch.empty(n, dtype=torch.int32, device=device),
                 "sB": torch.empty(n, dtype=torch.float64, device=device),
                 "nB": torch.empty(n, dtype=torch.float64, device=device)}
            self._glob[(m, n)] = g
        return g

    def rule_prepare(self, st, glob, m, n, k, Ir, Jr, force_N, force_p):
        b = st["_b"]
        key = (m, n, k)
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.empty(max(1, self.lib.ozk_rule_workspace_bytes(m, n, k)), dtype=torch.uint8, device=self.device)
            self._ws = {key: ws}
        check(self.lib.ozk_rule_prepare(ptr(glob["r"]), ptr(glob["c"]), ptr(glob["sA"]), ptr(glob["nA"]),
                                        ptr(glob["sB"]), ptr(glob["nB"]), ptr(st["flag"]), m, n, k, ptr(Ir), Ir.numel(),
                                        ptr(Jr), Jr.numel(), int(force_N or 0), -1 if force_p is None else int(force_p),
                                        ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]), ptr(ws), ws.numel(),
                                        self._stream()), "ozk_rule_prepare")
        self.engine.launches += 1 if force_N else 2
        return {"ws": ws, "b": b, "m": m, "n": n, "k": k}

    def rule_probe(self, h, A, B, row_begin, col_begin):
        ws = h["ws"]
        check(self.lib.ozk_rule_probe_block(ptr(A), ptr(B), row_begin, A.shape[0], col_begin, B.shape[1], h["m"],
                                            h["n"], h["k"], ptr(ws), ws.numel(), self._stream()), "ozk_rule_probe_block")
        self.engine.launches += 2
        off = self.lib.ozk_rule_probe_offset(h["m"], h["n"], h["k"])
        return ws[off:off + 96 * 96 * 8].view(torch.float64)

    def rule_finish(self, h, glob, tau, safety):
        b = h["b"]
        check(self.lib.ozk_rule_finish(ptr(glob["r"]), ptr(glob["c"]), ptr(glob["sA"]), ptr(glob["sB"]), h["m"], h["n"],
                                       h["k"], float(tau), float(safety), ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]),
                                       ptr(h["ws"]), h["ws"].numel(), self._stream()), "ozk_rule_finish")
        self.engine.launches += 2
        dec, _, aux = b.fetch()
        return dec.N, dec.p, int(dec.fallback), dec.p_req, aux

    def certificate_block(self, A, B, st, tau, safety):
        """This block's minimum xmax (float64 bit pattern as int64, -1 when no entry has D > 0) and its uncertified
        entry count, both as 1-element device tensors (csrc/certificate.cu)."""
        from .certificate import certificate_device
        w = certificate_device(self.engine, A, B, st["gam"], st["r"], st["c"], st["sA"], st["sB"], tau, safety)
        self._cert = w
        return w["xmin"].view(torch.int64).clone(), w["unc"].clone()

    def rule_certified(self, st, glob, m, n, k, xmin_bits):
        """The certified-mode decision from the global minimum (``ozk_rule_certified``); (N, p, fallback, p_req)."""
        b = st["_b"]
        xm = xmin_bits.view(torch.float64)
        check(self.lib.ozk_rule_certified(ptr(glob["nA"]), ptr(glob["nB"]), ptr(st["flag"]), m, n, k, ptr(xm),
                                          ptr(b["dec"]), ptr(b["pdev"]), ptr(b["aux"]), self._stream()),
              "ozk_rule_certified")
        self.engine.launches += 1
        dec, _, _ = b.fetch()
        if int(self._cert["err"].item()):
            raise _lib.OzkError(f"ozk_certificate: device error flag {int(self._cert['err'].item()):#x}")
        return dec.N, dec.p, int(dec.fallback), dec.p_req

    def core(self, A, B, st, N, p, C):
        rows, k = A.shape
        cols = B.shape[1]
        b = self.engine.buffers(rows, cols, k, N)
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
    """``run(A_block, B_block, C_block)``: this rank's block of C = A B, with the plane count and scalings of the
    whole product.  Rank g = a S + b passes rows [a m/R, (a+1) m/R) of A and columns [b n/S, (b+1) n/S) of B (as a
    contiguous k x n/S matrix); every rank must call ``run`` with the same block shapes and arguments.
    ``grid=(R, S)`` (default ``default_grid(world)``).  The constructor, the first ``run_broadcast_b`` for a root and
    the first ``gather_shares`` (or ``run_host_many(shares=True)``) create extra communicators with
    ``torch.distributed.new_group``, which every process of the default group must call: with a sub-group, construct
    the object (and make those first calls) on every process, in the same order."""

    def __init__(self, group=None, ops=None, grid=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.R, self.S = grid if grid is not None else default_grid(self.world)
        assert self.R * self.S == self.world, "grid must cover the ranks"
        self.a, self.b = divmod(self.rank, self.S)
        self.ops = ops if ops is not None else CudaOps()
        self.probe = {}
        self._recv = {}                                       # receive buffers of the operand moves, per name
        self.last_b = None
        # a second communicator over the same ranks for the bulk operand moves (B's broadcast), so that the small
        # statistics collectives run beside it instead of queueing behind it; created here, on every rank alike
        ranks = dist.get_process_group_ranks(group) if group is not None else list(range(self.world))
        self.bulk = dist.new_group(ranks=ranks)

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

    def _gather(self, x, total, stride, count):
        """all_gather of an equally sized per-rank vector; keeps the blocks of ranks 0, stride, 2 stride, ... (one per
        row block when stride = S, one per column block when stride = 1 and count = S)."""
        parts = torch.empty(self.world * x.numel(), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(parts, x.contiguous(), group=self.group)
        parts = parts.view(self.world, x.numel())
        return parts[0:stride * count:stride].reshape(total)

    def _mark(self, events, name):
        if events is not None and getattr(self.ops, "timed", False):
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append((name, e))

    def _buffer(self, name, shape, dtype, device):
        """A receive buffer kept between calls (replaced when the shape changes)."""
        t = self._recv.get(name)
        if t is None or tuple(t.shape) != tuple(shape) or t.dtype != dtype or t.device != device:
            t = self._recv[name] = torch.empty(shape, dtype=dtype, device=device)
        return t

    def _header(self, values, root, device):
        """Broadcast a few int64 sizes from the root (the other ranks pass placeholders)."""
        h = torch.tensor(values, dtype=torch.int64, device=device)
        dist.broadcast(h, src=root, group=self.group)
        return [int(x) for x in h.tolist()]

    def _device_of(self, *tensors):
        for t in tensors:
            if t is not None:
                return t.device
        return getattr(self.ops, "device", torch.device("cpu"))

    def _column_groups(self, root):
        """Per column block b, the communicator over the root and the ranks of grid column b (the bulk communicator
        when S = 1).  Created on first use for a root, by every rank in the same order (new_group is collective)."""
        if self.S == 1:
            return [self.bulk]
        groups = self.__dict__.setdefault("_colgroups", {})
        if root not in groups:
            base = dist.get_process_group_ranks(self.group) if self.group is not None else list(range(self.world))
            groups[root] = [dist.new_group(ranks=sorted({base[root]} | {base[a * self.S + b] for a in range(self.R)}))
                            for b in range(self.S)]
        return groups[root]

    def run_broadcast_b(self, A, B=None, C=None, root=0, events=None, **kw):
        """This rank's block of C = A B when B lives only on rank ``root``: B (k x n FP64) is sent from the root
        over NCCL, then the blocks are multiplied as in ``run``.  Rank g = a S + b passes A's row block a (rows x k,
        rows = m / R); on the root B is the whole k x n matrix or, for S > 1, the list of its S contiguous column
        blocks (k x n / S each; a whole B is cut into such blocks first); elsewhere it is ignored.  On a row-block
        grid (S = 1) B is broadcast whole; with S > 1 column block b goes to the ranks of grid column b only (the
        root's egress is still one copy of B; every rank receives, splits and multiplies n / S columns)."""
        is_root = self.rank == root
        parts = None
        if is_root:
            parts = list(B) if isinstance(B, (list, tuple)) else [B]
            for t in parts:
                assert t.is_contiguous() and t.dtype == torch.float64
        dev = self._device_of(A, *(parts or []))
        k = A.shape[1]
        hdr = [parts[0].shape[0], sum(t.shape[1] for t in parts), len(parts)] if is_root else [0, 0, 0]
        k_b, n, nparts = self._header(hdr, root, dev)
        assert k_b == k, "A's and B's inner dimensions differ"
        assert n % self.S == 0, "n must divide into equal column blocks"
        cols = n // self.S
        if is_root and self.S > 1 and nparts == 1:
            whole = parts[0]
            parts = []
            for b in range(self.S):
                blk = self._buffer(f"Bc{b}", (k, cols), torch.float64, dev)
                blk.copy_(whole[:, b * cols:(b + 1) * cols])
                parts.append(blk)
        if is_root:
            assert len(parts) == self.S and all(tuple(t.shape) == (k, cols) for t in parts), "B's column blocks"
        groups = self._column_groups(root)
        self._mark(events, "start")
        works = []
        Bl = parts[self.b] if is_root else self._buffer("B", (k, cols), torch.float64, dev)
        for b in range(self.S):
            if is_root:
                works.append(dist.broadcast(parts[b], src=root, group=groups[b], async_op=True))
            elif b == self.b:
                works.append(dist.broadcast(Bl, src=root, group=groups[b], async_op=True))
        self.last_b = Bl                      # this rank's block of B (kept for callers that reuse it)
        return self._run_b_on_root(A, Bl, parts, n, C, root, works, events, **kw)

    def run_from_root(self, A=None, B=None, C=None, root=0, gather=True, events=None, **kw):
        """C = A B with A (m x k) and B (k x n) only on rank ``root``: A's row blocks are scattered, B broadcast,
        each rank multiplies its block, and with ``gather`` the row blocks of C are gathered into the root's C
        (allocated when None).  Returns (C on the root -- this rank's row block elsewhere or without gather, info).
        Needs a row-block grid (S = 1) and m divisible by the number of ranks."""
        assert self.S == 1, "run_from_root needs a row-block grid (S = 1)"
        dev = self._device_of(A, B, C)
        m, k, n = self._header(list(A.shape) + [B.shape[1]] if self.rank == root else [0, 0, 0], root, dev)
        assert m % self.R == 0, "m must divide into equal row blocks"
        rows = m // self.R
        Ab = self._buffer("A", (rows, k), torch.float64, dev)
        Bl = B if self.rank == root else self._buffer("B", (k, n), torch.float64, dev)
        Cb = self._buffer("C", (rows, n), torch.float64, dev)
        if self.rank == root:
            assert A.is_contiguous() and B.is_contiguous() and A.dtype == B.dtype == torch.float64
            if C is None and gather:
                C = torch.empty((m, n), dtype=torch.float64, device=dev)
        self._mark(events, "start")
        work = dist.broadcast(Bl, src=root, group=self.bulk, async_op=True)
        dist.scatter(Ab, list(A.split(rows)) if self.rank == root else None, src=root, group=self.group)
        self._mark(events, "scatter A")
        _, info = self._run_b_on_root(Ab, Bl, [B] if self.rank == root else None, n, Cb, root, [work], events, **kw)
        if not gather:
            return Cb, info
        dist.gather(Cb, list(C.split(rows)) if self.rank == root else None, dst=root, group=self.group)
        self._mark(events, "gather C")
        return (C if self.rank == root else Cb), info

    def _run_b_on_root(self, A, Bl, B_parts, n, C, root, pending, events, tau=2.0 ** -52, force_N=None, inside=True,
                       seed=0, force_p=None, safety=2.0, config=None, certify=False):
        """``run`` while this rank's block of B (``Bl``, k x n / S) is still arriving from ``root`` (``pending``:
        the handles of the sends on the bulk communicators).  The root computes B's row maxima and column
        statistics from its own copy (``B_parts``: B's column blocks, in order) while the sends run and broadcasts
        the column statistics (3 n values); every rank computes its rows' statistics meanwhile, and waits for B
        only before the probe product.  Same collectives in the same order on every rank; the decision and C equal
        ``run``'s bit for bit."""
        if config is not None:
            force_N, force_p = int(config["N"]), config.get("p")
        rows, k = A.shape
        cols = n // self.S
        assert Bl.shape == (k, cols) and rows % 4 == 0 and cols % 32 == 0 and k % 32 == 0, "shape rule (per rank)"
        m = rows * self.R
        row_begin, col_begin = rows * self.a, cols * self.b
        is_root = self.rank == root
        if C is None:
            C = torch.empty((rows, cols), dtype=torch.float64, device=A.device)
        # 1. global maxima: B's row maxima from the root only (zeros, the identity of MAX on the non-negative bit
        #    patterns, elsewhere)
        cm = self.ops.colmax(A)
        if is_root:
            rm = self.ops.rowmax(B_parts[0])
            for part in B_parts[1:]:
                rm = torch.maximum(rm, self.ops.rowmax(part))
        else:
            rm = torch.zeros_like(cm)
        mx = torch.cat([cm, rm])
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=self.group)
        self._mark(events, "maxima + all_reduce")
        # 2. rows' statistics everywhere; all of B's column statistics on the root, then broadcast (each rank keeps
        #    its block's slice for the split)
        st = self.ops.local_stats(A, None, mx[:k], mx[k:], inside, cols=cols)
        glob = self.ops.global_stats(m, n, A.device)
        for x in ("r", "sA", "nA"):
            glob[x].copy_(self._gather(st[x], m, self.S, self.R))
        if is_root:
            c0 = 0
            for part in B_parts:
                cs = self.ops.col_stats(part, st, mx[:k], mx[k:], inside)
                w = part.shape[1]
                for x in ("c", "sB", "nB"):
                    glob[x][c0:c0 + w].copy_(cs[x])
                c0 += w
        for x in ("c", "sB", "nB"):
            dist.broadcast(glob[x], src=root, group=self.group)
            st[x].copy_(glob[x][col_begin:col_begin + cols])
        self._mark(events, "statistics + all_gather")
        for w in pending:
            w.wait()
        self._mark(events, "broadcast B (rest)")
        return self._decide_and_core(A, Bl, C, st, glob, m, n, k, row_begin, col_begin, tau, force_N, seed, force_p,
                                     safety, certify, events)

    def _grid_groups(self):
        """(communicator of this rank's grid row, of its grid column); None for a row or column of one rank.
        Created on first use: every rank creates all of them in the same order (new_group is collective)."""
        gg = self.__dict__.get("_gridgroups")
        if gg is None:
            base = dist.get_process_group_ranks(self.group) if self.group is not None else list(range(self.world))
            rowg = [dist.new_group(ranks=[base[a * self.S + q] for q in range(self.S)]) if self.S > 1 else None
                    for a in range(self.R)]
            colg = [dist.new_group(ranks=[base[a * self.S + b] for a in range(self.R)]) if self.R > 1 else None
                    for b in range(self.S)]
            gg = self._gridgroups = (rowg[self.a], colg[self.b])
        return gg

    def gather_shares(self, A_share, B_share, A=None, B=None):
        """This rank's blocks from the shares of its grid row and grid column.  Rank (a, b) holds rows
        [b rows / S, (b + 1) rows / S) of A's row block a and rows [a k / R, (a + 1) k / R) of B's column block b
        (k x n / S); one all_gather over the grid row gives the row block (rows x k), one over the grid column the
        column block (k x n / S), so that every byte of A and B is loaded onto the GPUs once.  Every rank calls it
        with shares of the same shapes.  Returns (A_block, B_block), written into A, B when given."""
        rowg, colg = self._grid_groups()
        rs, k = A_share.shape
        ks, cols = B_share.shape
        assert ks * self.R == k, "B's share must hold k / R rows of its column block"
        if A is None:
            A = A_share if rowg is None else torch.empty((rs * self.S, k), dtype=A_share.dtype, device=A_share.device)
        if B is None:
            B = B_share if colg is None else torch.empty((k, cols), dtype=B_share.dtype, device=B_share.device)
        assert tuple(A.shape) == (rs * self.S, k) and tuple(B.shape) == (k, cols), "block buffers of the wrong shape"
        for full, share, g in ((A, A_share, rowg), (B, B_share, colg)):
            if g is None:
                if full.data_ptr() != share.data_ptr():
                    full.copy_(share)
            else:
                dist.all_gather_into_tensor(full, share.contiguous(), group=g)
        return A, B

    def run(self, A, B, C=None, tau=2.0 ** -52, force_N=None, inside=True, seed=0, force_p=None, safety=2.0,
            config=None, certify=False, events=None):
        if config is not None:
            force_N, force_p = int(config["N"]), config.get("p")
        rows, k = A.shape
        cols = B.shape[1]
        assert B.shape[0] == k and rows % 4 == 0 and cols % 32 == 0 and k % 32 == 0, "shape rule (per rank)"
        m, n = rows * self.R, cols * self.S
        row_begin, col_begin = rows * self.a, cols * self.b
        if C is None:
            C = torch.empty((rows, cols), dtype=torch.float64, device=A.device)
        # 1. global maxima -> gamma, flag; local statistics
        cm = self.ops.colmax(A)
        rm = self.ops.rowmax(B)
        mx = torch.cat([cm, rm])
        dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=self.group)
        self._mark(events, "maxima + all_reduce")
        st = self.ops.local_stats(A, B, mx[:k], mx[k:], inside)
        # 2. statistics of all rows and columns
        glob = self.ops.global_stats(m, n, A.device)
        for x in ("r", "sA", "nA"):
            glob[x].copy_(self._gather(st[x], m, self.S, self.R))
        for x in ("c", "sB", "nB"):
            glob[x].copy_(self._gather(st[x], n, 1, self.S))
        self._mark(events, "statistics + all_gather")
        return self._decide_and_core(A, B, C, st, glob, m, n, k, row_begin, col_begin, tau, force_N, seed, force_p,
                                     safety, certify, events)

    def _decide_and_core(self, A, B, C, st, glob, m, n, k, row_begin, col_begin, tau, force_N, seed, force_p, safety,
                         certify, events):
        """Steps 3 (probe or certificate, the same decision on every rank) and the local core."""
        rows, cols = A.shape[0], B.shape[1]
        if certify and force_N is None:
            # 3'. full-matrix certificate: minimum over the blocks, then the same decision everywhere
            xb, unc = self.ops.certificate_block(A, B, st, tau, safety)
            none = torch.full_like(xb, torch.iinfo(torch.int64).max)
            xr = torch.where(xb == -1, none, xb)
            dist.all_reduce(xr, op=dist.ReduceOp.MIN, group=self.group)
            dist.all_reduce(unc, op=dist.ReduceOp.SUM, group=self.group)
            xr = torch.where(xr == none, torch.full_like(xr, -1), xr)
            N, p, fb, preq = self.ops.rule_certified(st, glob, m, n, k, xr)
            if fb or N == 0:
                self.ops.native(A, B, C)
                return C, {"fallback": True, "preq": preq, "certified": True}
            self.ops.core(A, B, st, N, p, C)
            return C, {"N": N, "p": p, "preq": preq, "certified": True, "uncertified_entries": int(unc.item()),
                       "rows": [row_begin, row_begin + rows], "cols": [col_begin, col_begin + cols],
                       "grid": [self.R, self.S], "world": self.world}
        # 3. probe product summed over the blocks, then the same decision everywhere
        Ir, Jr = self._probe_sets(m, n, seed, A.device)
        h = self.ops.rule_prepare(st, glob, m, n, k, Ir, Jr, force_N, force_p)
        D = self.ops.rule_probe(h, A, B, row_begin, col_begin)
        dist.all_reduce(D, op=dist.ReduceOp.SUM, group=self.group)
        N, p, fb, preq, aux = self.ops.rule_finish(h, glob, tau, safety)
        self._mark(events, "rule (probe + all_reduce + host read)")
        if fb or N == 0:
            self.ops.native(A, B, C)
            return C, {"fallback": True, "preq": preq}
        self.ops.core(A, B, st, N, p, C)
        self._mark(events, "core")
        return C, {"N": N, "p": p, "preq": preq, "rows": [row_begin, row_begin + rows],
                   "cols": [col_begin, col_begin + cols], "grid": [self.R, self.S], "world": self.world}


    def run_host_many(self, jobs, shares=False, **kw):
        """A stream of host-buffer products on this rank: ``jobs`` is a list of (A_rows_h, B_cols_h, C_block_h)
        pinned float64 CPU tensors of one shape (C_block_h None to allocate), the same list length and keyword
        arguments (those of ``run``) on every rank.  Two device slots: the H2D copies of job i + 1 run on their own
        stream while job i computes (its collectives included) and its C block goes back on a third stream.
        ``shares=True``: A_rows_h and B_cols_h are this rank's shares as ``gather_shares`` defines them (rows / S of
        A's row block, k / R rows of B's column block), so that each byte of A and B crosses PCIe once, on one rank;
        the blocks are gathered over NCCL within the grid row and column before each product.
        Returns [(C_block_h, info), ...]; each equals a ``run`` on the same blocks bit for bit.  Synchronises at the
        end and raises ``OzkError`` if a kernel of these products reported a device-side error."""
        if not jobs:
            return []
        rows, k = jobs[0][0].shape
        ks, cols = jobs[0][1].shape
        split_a = shares and self.S > 1
        split_b = shares and self.R > 1
        if shares:
            rows, k = rows * self.S, ks * self.R
            assert jobs[0][0].shape[1] == k, "A's share must hold all k columns"
        dev = torch.device("cuda", torch.cuda.current_device())
        key = (rows, cols, k, split_a, split_b)
        io = self.__dict__.setdefault("_host_many", {})
        dv = io.get(key)
        if dv is None:
            io.clear()
            shapes = [("A", (rows, k)), ("B", (k, cols)), ("C", (rows, cols))]
            if split_a:
                shapes.append(("As", (rows // self.S, k)))
            if split_b:
                shapes.append(("Bs", (k // self.R, cols)))
            dv = {"slots": [{x: torch.empty(sh, dtype=torch.float64, device=dev) for x, sh in shapes}
                            for _ in range(2)],
                  "cin": torch.cuda.Stream(), "cout": torch.cuda.Stream()}
            io[key] = dv
        slots, cin, cout = dv["slots"], dv["cin"], dv["cout"]
        cur = torch.cuda.current_stream()
        cin.wait_stream(cur)
        cout.wait_stream(cur)
        in_done = [torch.cuda.Event(), torch.cuda.Event()]
        used = [None, None]
        outs = [C_h if C_h is not None else torch.empty((rows, cols), dtype=torch.float64, pin_memory=True)
                for _, _, C_h in jobs]

        def h2d(i):
            s = i % 2
            if used[s] is not None:
                cin.wait_event(used[s][0])
            with torch.cuda.stream(cin):
                slots[s]["As" if split_a else "A"].copy_(jobs[i][0], non_blocking=True)
                slots[s]["Bs" if split_b else "B"].copy_(jobs[i][1], non_blocking=True)
            in_done[s].record(cin)

        h2d(0)
        results = []
        for i in range(len(jobs)):
            s = i % 2
            if i + 1 < len(jobs):
                h2d(i + 1)
            cur.wait_event(in_done[s])
            if used[s] is not None:
                cur.wait_event(used[s][1])
            if shares:
                # the gathers run on the current stream's order, before the product (the next H2D into this slot's
                # shares waits for the event recorded after the product)
                self.gather_shares(slots[s]["As"] if split_a else slots[s]["A"],
                                   slots[s]["Bs"] if split_b else slots[s]["B"], slots[s]["A"], slots[s]["B"])
            C, info = self.run(slots[s]["A"], slots[s]["B"], slots[s]["C"], **kw)
            cdone, odone = torch.cuda.Event(), torch.cuda.Event()
            cdone.record(cur)
            cout.wait_event(cdone)
            with torch.cuda.stream(cout):
                outs[i].copy_(C, non_blocking=True)
            odone.record(cout)
            used[s] = (cdone, odone)
            results.append((outs[i], info))
        cur.wait_stream(cout)
        cur.wait_stream(cin)
        cur.synchronize()
        self.engine.check_errors()           # raises if a split, product or reconstruction reported a device error
        return results


__all__ = ["DistributedOzakiCRT", "CudaOps", "default_grid", "_lib"]
