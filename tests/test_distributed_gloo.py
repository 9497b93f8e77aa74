"""The multi-GPU C block orchestration (matrix_numbers_b200.distributed) over gloo ranks on the CPU.

The per-rank compute is supplied by ``OracleOps`` (the CPU oracle behind the ops interface of ``CudaOps``), so these
tests check the collective steps and the index bookkeeping: the assembled C of 2 ranks (row blocks or column blocks)
and of a 2 x 2 grid of 4 ranks must equal the single-process product bit for bit, and every rank must reach the same
(N, p).  A failing rank must end the others' next collective
with an error instead of a hang (host-side failure injection; no GPU involved)."""
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """CPU stand-in for CudaOps: same interface, oracle arithmetic (test infrastructure)."""

    def __init__(self, oracle):
        self.O = oracle
        self.launches = 0
        self.device = torch.device("cpu")

    def colmax(self, A):
        return torch.from_numpy(self.O.colmax(A.numpy()).copy())

    def rowmax(self, B):
        return torch.from_numpy(self.O.rowmax(B.numpy()).copy())

    def local_stats(self, A, B, colmax, rowmax, inside, cols=None):
        # B None: column statistics come from the rank that holds B (placeholders of the right size here)
        Bn = B.numpy() if B is not None else np.zeros((A.shape[1], cols))
        st = self.O.stats_given_maxima(A.numpy(), Bn, colmax.numpy(), rowmax.numpy(), inside)
        out = {x: torch.from_numpy(np.ascontiguousarray(st[x])) for x in ("gam", "r", "sA", "nA", "c", "sB", "nB")}
        out["flag"] = torch.tensor([st["flag"]], dtype=torch.int32)
        out["_np"] = st
        return out

    def col_stats(self, B, st, colmax, rowmax, inside):
        # gamma depends on the maxima only: a placeholder row of A gives B's column statistics under the global gamma
        o = self.O.stats_given_maxima(np.zeros((1, B.shape[0])), B.numpy(), colmax.numpy(), rowmax.numpy(), inside)
        return {x: torch.from_numpy(np.ascontiguousarray(o[x])) for x in ("c", "sB", "nB")}

    def global_stats(self, m, n, device):
        return {"r": torch.empty(m, dtype=torch.int32), "sA": torch.empty(m, dtype=torch.float64),
                "nA": torch.empty(m, dtype=torch.float64), "c": torch.empty(n, dtype=torch.int32),
                "sB": torch.empty(n, dtype=torch.float64), "nB": torch.empty(n, dtype=torch.float64)}

    def rule_prepare(self, st, glob, m, n, k, Ir, Jr, force_N, force_p):
        g = {x: glob[x].numpy() for x in ("r", "sA", "nA", "c", "sB", "nB")}
        g["flag"] = int(st["flag"][0])
        I = np.concatenate([Ir.numpy(), self.O.hard_top(g["r"], g["sA"], k)])
        J = np.concatenate([Jr.numpy(), self.O.hard_top(g["c"], g["sB"], k)])
        return {"g": g, "I": I, "J": J, "m": m, "n": n, "k": k, "force_N": force_N, "force_p": force_p}

    def rule_probe(self, h, A, B, row_begin, col_begin):
        # this rank's entries of D = |A_I| |B_J| (probe row and column inside its block), zeros elsewhere
        rows, cols = A.shape[0], B.shape[1]
        D = np.zeros((96, 96))
        I, J = h["I"], h["J"]
        jb = [b for b, j in enumerate(J) if col_begin <= j < col_begin + cols]
        for a, i in enumerate(I):
            if row_begin <= i < row_begin + rows and jb:
                D[a, jb] = self.O.probe_D(A.numpy(), B.numpy(), [i - row_begin], [J[b] - col_begin for b in jb])[0]
        h["Dt"] = torch.from_numpy(D.reshape(-1))
        return h["Dt"]

    def rule_finish(self, h, glob, tau, safety):
        I, J = h["I"], h["J"]
        D = h["Dt"].numpy().reshape(96, 96)[:len(I), :len(J)]
        ru = self.O.rule(h["g"], h["m"], h["n"], h["k"], I, J, D, tau, safety, h["force_N"])
        N, p, fb = ru["N"] or 0, ru["p"], int(ru["fallback"])
        if h["force_N"] and h["force_p"] is not None:
            fb = int(p < h["force_p"])
            p = min(p, h["force_p"])
            N = 0 if fb else N
        return N, p, fb, ru["p_req"], [ru["nuA"], ru["nuB"], ru["worst_ratio_E_over_D"], len(set(I)), len(set(J)), 0, 0, 0]

    def certificate_block(self, A, B, st, tau, safety):
        xb, unc = self.O.certificate_xmin(A.numpy(), B.numpy(), st["_np"], tau, safety)
        return torch.tensor([xb], dtype=torch.int64), torch.tensor([unc], dtype=torch.int64)

    def rule_certified(self, st, glob, m, n, k, xmin_bits):
        N, p, fb, preq = self.O.rule_certified(glob["nA"].numpy(), glob["nB"].numpy(), int(st["flag"][0]), k,
                                               int(xmin_bits[0]))
        return N, p, int(fb), preq

    def core(self, A, B, st, N, p, C):
        C.copy_(torch.from_numpy(self.O.core(A.numpy(), B.numpy(), st["_np"], N, p)))
        return C

    def native(self, A, B, C):
        torch.matmul(A, B, out=C)
        return C


GRIDS = {"ok": (2, 1), "cols": (1, 2), "grid4": (2, 2), "cert": (2, 1), "cert4": (2, 2), "bcastB4": (2, 2), "bcastB8": (4, 2),
         "sharesR": (2, 1), "sharesS": (1, 2), "shares8": (4, 2)}


def _worker(rank, world, port, outdir, mode):
    try:
        sys.path.insert(0, ROOT)
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import datetime

        import torch.distributed as dist

        import __graft_entry__
        import oracle as O
        pkg = __graft_entry__.load_package()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=8))
        from matrix_numbers_b200.distributed import DistributedOzakiCRT
        m, k, n = 128, 256, 128
        A, B = pkg.make_inputs(m, k, n, 2.0, seed=31)
        R, S = GRIDS[mode] if mode in GRIDS else (world, 1)
        a, b = divmod(rank, S)
        rows, cols = m // R, n // S
        Al = torch.from_numpy(np.ascontiguousarray(A[a * rows:(a + 1) * rows]))
        Bt = torch.from_numpy(np.ascontiguousarray(B[:, b * cols:(b + 1) * cols]))
        D = DistributedOzakiCRT(ops=OracleOps(O), grid=(R, S))
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the first collective")
        if mode in ("bcastB", "bcastB4", "bcastB8", "root"):
            # the operands start on rank 1 (the root): B only (A's rows on their owners), or A and B both
            root = 1
            Bfull = torch.from_numpy(B) if rank == root else None
            if mode in ("bcastB", "bcastB4", "bcastB8"):
                C, info = D.run_broadcast_b(Al, Bfull, root=root)
                # on the grid the root may also hold B as its column blocks
                Bparts = [torch.from_numpy(np.ascontiguousarray(B[:, q * cols:(q + 1) * cols])) for q in range(S)]
                C2, info2 = D.run_broadcast_b(Al, Bparts if (mode != "bcastB" and rank == root) else Bfull, root=root,
                                              force_N=22)
            else:
                Afull = torch.from_numpy(A) if rank == root else None
                C, info = D.run_from_root(Afull, Bfull, root=root)
                C2, info2 = D.run_from_root(Afull, Bfull, root=root, force_N=22)
                if rank != root:                 # every rank holds its row block; the root holds all of C
                    C, C2 = torch.zeros(m, n, dtype=torch.float64), torch.zeros(m, n, dtype=torch.float64)
                Cb, _ = D.run_from_root(Afull, Bfull, root=root, gather=False)
                np.save(os.path.join(outdir, f"Cblock_{rank}.npy"), Cb.numpy())
        elif mode.startswith("shares"):
            # each rank holds 1 / S of A's row block and 1 / R of B's column block; the grid row and column gather
            sr, sk = rows // S, k // R
            As = torch.from_numpy(np.ascontiguousarray(A[a * rows + b * sr:a * rows + (b + 1) * sr]))
            Bs = torch.from_numpy(np.ascontiguousarray(B[a * sk:(a + 1) * sk, b * cols:(b + 1) * cols]))
            Ab, Bb = D.gather_shares(As, Bs)
            assert torch.equal(Ab, Al) and torch.equal(Bb, Bt), "gathered blocks differ from the blocks"
            try:                                    # a share of the wrong height fails before any collective
                D.gather_shares(As, Bs[:-1])
                raise RuntimeError("a B share of k / R - 1 rows was accepted")
            except AssertionError:
                pass
            try:                                    # so does a block buffer of the wrong shape
                D.gather_shares(As, Bs, torch.empty(rows + 4, k, dtype=torch.float64), None)
                raise RuntimeError("an A block buffer of rows + 4 rows was accepted")
            except AssertionError:
                pass
            Ab2, Bb2 = torch.empty_like(Al), torch.empty_like(Bt)
            D.gather_shares(As, Bs, Ab2, Bb2)
            assert torch.equal(Ab2, Al) and torch.equal(Bb2, Bt), "gather into given buffers"
            C, info = D.run(Ab, Bb)
            C2, info2 = D.run(Ab2, Bb2, force_N=22)
        else:
            C, info = D.run(Al, Bt, certify=mode.startswith("cert"))
            C2, info2 = D.run(Al, Bt, force_N=22)
        np.save(os.path.join(outdir, f"C_{rank}.npy"), C.numpy())
        np.save(os.path.join(outdir, f"C22_{rank}.npy"), C2.numpy())
        with open(os.path.join(outdir, f"info_{rank}.txt"), "w") as f:
            f.write(repr((info["N"], info["p"], info["preq"], info2["N"], info2["p"])))
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"error_{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())


def _spawn(world, mode, tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_worker, args=(world, port, str(tmp_path), mode), nprocs=world, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    alive = [p.is_alive() for p in ctx.processes]
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    return alive


@pytest.mark.parametrize("mode,world", [("ok", 2), ("cols", 2), ("grid4", 4), ("sharesR", 2), ("sharesS", 2),
                                        ("shares8", 8)])
def test_blocks_equal_single_process(oracle, tmp_path, pkg, mode, world):
    """Pre-placed blocks (ok, cols, grid4), or blocks assembled by gather_shares from each rank's share of them
    (shares*: the host-buffer path's loads), then the grid product."""
    alive = _spawn(world, mode, tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    R, S = GRIDS[mode]
    A, B = pkg.make_inputs(128, 256, 128, 2.0, seed=31)

    def assemble(name):
        return np.concatenate([np.concatenate([np.load(os.path.join(tmp_path, f"{name}_{a * S + b}.npy"))
                                               for b in range(S)], axis=1) for a in range(R)])
    Cref, iref = oracle.run(A, B)
    np.testing.assert_array_equal(assemble("C").view(np.uint64), Cref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(world)]
    assert all(i == infos[0] for i in infos)
    assert infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])
    C22ref, i22 = oracle.run(A, B, force_N=22)
    np.testing.assert_array_equal(assemble("C22").view(np.uint64), C22ref.view(np.uint64))
    assert infos[0][3:] == (22, i22["p"])


@pytest.mark.parametrize("mode,world", [("cert", 2), ("cert4", 4)])
def test_certified_blocks_equal_single_process(oracle, tmp_path, pkg, mode, world):
    """Certified mode over the grid: the blocks' minimum bound, reduced with MIN, gives the same decision and the
    same C as the whole-matrix certificate of the single-process oracle."""
    alive = _spawn(world, mode, tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    R, S = GRIDS[mode]
    A, B = pkg.make_inputs(128, 256, 128, 2.0, seed=31)
    C = np.concatenate([np.concatenate([np.load(os.path.join(tmp_path, f"C_{a * S + b}.npy")) for b in range(S)], axis=1)
                        for a in range(R)])
    Cref, iref = oracle.run_certified(A, B)
    assert Cref is not None
    np.testing.assert_array_equal(C.view(np.uint64), Cref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(world)]
    assert all(i == infos[0] for i in infos)
    assert infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])


def test_broadcast_b_from_root_equals_single_process(oracle, tmp_path, pkg):
    """A's and C's row blocks on their owners, B only on the root (rank 1): B is broadcast inside the call."""
    alive = _spawn(2, "bcastB", tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    A, B = pkg.make_inputs(128, 256, 128, 2.0, seed=31)
    Cref, iref = oracle.run(A, B)
    C = np.concatenate([np.load(os.path.join(tmp_path, f"C_{r}.npy")) for r in range(2)])
    np.testing.assert_array_equal(C.view(np.uint64), Cref.view(np.uint64))
    C22ref, i22 = oracle.run(A, B, force_N=22)
    C22 = np.concatenate([np.load(os.path.join(tmp_path, f"C22_{r}.npy")) for r in range(2)])
    np.testing.assert_array_equal(C22.view(np.uint64), C22ref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(2)]
    assert infos[0] == infos[1] and infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])


@pytest.mark.parametrize("mode,world", [("bcastB4", 4), ("bcastB8", 8)])
def test_broadcast_b_on_grid_equals_single_process(oracle, tmp_path, pkg, mode, world):
    """B only on the root (rank 1) of a 2 x 2 or 4 x 2 grid: column block b of B goes to grid column b only (through
    one communicator per column group, the root in both), the root computes all of B's column statistics; every rank
    multiplies A's row block a by B's column block b."""
    R, S = GRIDS[mode]
    alive = _spawn(world, mode, tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    A, B = pkg.make_inputs(128, 256, 128, 2.0, seed=31)

    def assemble(name):
        return np.concatenate([np.concatenate([np.load(os.path.join(tmp_path, f"{name}_{a * S + b}.npy"))
                                               for b in range(S)], axis=1) for a in range(R)])
    Cref, iref = oracle.run(A, B)
    np.testing.assert_array_equal(assemble("C").view(np.uint64), Cref.view(np.uint64))
    C22ref, i22 = oracle.run(A, B, force_N=22)
    np.testing.assert_array_equal(assemble("C22").view(np.uint64), C22ref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(world)]
    assert all(i == infos[0] for i in infos) and infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])


def test_run_from_root_scatter_broadcast_gather(oracle, tmp_path, pkg):
    """A and B only on the root (rank 1): A scattered by row blocks, B broadcast, C gathered into the root's C; and
    without the gather every rank keeps its row block."""
    alive = _spawn(2, "root", tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    A, B = pkg.make_inputs(128, 256, 128, 2.0, seed=31)
    Cref, iref = oracle.run(A, B)
    np.testing.assert_array_equal(np.load(os.path.join(tmp_path, "C_1.npy")).view(np.uint64), Cref.view(np.uint64))
    C22ref, _ = oracle.run(A, B, force_N=22)
    np.testing.assert_array_equal(np.load(os.path.join(tmp_path, "C22_1.npy")).view(np.uint64),
                                  C22ref.view(np.uint64))
    blocks = np.concatenate([np.load(os.path.join(tmp_path, f"Cblock_{r}.npy")) for r in range(2)])
    np.testing.assert_array_equal(blocks.view(np.uint64), Cref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(2)]
    assert infos[0] == infos[1] and infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])


def test_failed_rank_ends_peers_collective_with_error(tmp_path):
    alive = _spawn(2, "fail", tmp_path)
    assert not any(alive), "a rank hung after its peer failed"
    assert os.path.exists(os.path.join(tmp_path, "error_1.txt"))
    # rank 0 must have seen an error from its collective (timeout or closed connection), not a hang
    assert os.path.exists(os.path.join(tmp_path, "error_0.txt"))
