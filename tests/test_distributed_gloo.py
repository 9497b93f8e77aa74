"""The multi-GPU C row-block orchestration (matrix_numbers_b200.distributed) over gloo ranks on the CPU.

The per-rank compute is supplied by ``OracleOps`` (the CPU oracle behind the ops interface of ``CudaOps``), so these
tests check the collective steps and the index bookkeeping: the gathered C of 2 ranks must equal the single-process
product bit for bit, and every rank must reach the same (N, p).  A failing rank must end the others' next collective
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

    def colmax(self, A):
        return torch.from_numpy(self.O.colmax(A.numpy()).copy())

    def stats_finish(self, A, B, colmax, inside):
        st = self.O.stats_given_colmax(A.numpy(), B.numpy(), colmax.numpy(), inside)
        out = {x: torch.from_numpy(np.ascontiguousarray(st[x])) for x in ("gam", "r", "sA", "nA", "c", "sB", "nB")}
        out["flag"] = torch.tensor([st["flag"]], dtype=torch.int32)
        out["_np"] = st
        return out

    def global_rows(self, m, device):
        return {"r": torch.empty(m, dtype=torch.int32), "sA": torch.empty(m, dtype=torch.float64),
                "nA": torch.empty(m, dtype=torch.float64)}

    def rule_prepare(self, st, glob, m, n, k, Ir, Jr, force_N, force_p):
        g = {"r": glob["r"].numpy(), "sA": glob["sA"].numpy(), "nA": glob["nA"].numpy(),
             "c": st["c"].numpy(), "sB": st["sB"].numpy(), "nB": st["nB"].numpy(), "flag": int(st["flag"][0])}
        I = np.concatenate([Ir.numpy(), self.O.hard_top(g["r"], g["sA"], k)])
        J = np.concatenate([Jr.numpy(), self.O.hard_top(g["c"], g["sB"], k)])
        return {"g": g, "I": I, "J": J, "m": m, "n": n, "k": k, "force_N": force_N, "force_p": force_p}

    def rule_probe(self, h, A, B, row_begin):
        # this rank's probe rows of D = |A_I| |B_J|, zeros for the rows other ranks own (summed by all_reduce)
        rows = A.shape[0]
        D = np.zeros((96, 96))
        I, J = h["I"], h["J"]
        for a, i in enumerate(I):
            if row_begin <= i < row_begin + rows:
                D[a, :len(J)] = self.O.probe_D(A.numpy(), B.numpy(), [i - row_begin], J)[0]
        h["Dt"] = torch.from_numpy(D.reshape(-1))
        return h["Dt"]

    def rule_finish(self, h, st, glob, tau, safety):
        I, J = h["I"], h["J"]
        D = h["Dt"].numpy().reshape(96, 96)[:len(I), :len(J)]
        ru = self.O.rule(h["g"], h["m"], h["n"], h["k"], I, J, D, tau, safety, h["force_N"])
        N, p, fb = ru["N"] or 0, ru["p"], int(ru["fallback"])
        if h["force_N"] and h["force_p"] is not None:
            fb = int(p < h["force_p"])
            p = min(p, h["force_p"])
            N = 0 if fb else N
        return N, p, fb, ru["p_req"], [ru["nuA"], ru["nuB"], ru["worst_ratio_E_over_D"], len(set(I)), len(set(J)), 0, 0, 0]

    def core(self, A, B, st, N, p, C):
        C.copy_(torch.from_numpy(self.O.core(A.numpy(), B.numpy(), st["_np"], N, p)))
        return C

    def native(self, A, B, C):
        torch.matmul(A, B, out=C)
        return C


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
        m, k, n = 128, 256, 96
        A, B = pkg.make_inputs(m, k, n, 2.0, seed=31)
        rows = m // world
        Al = torch.from_numpy(np.ascontiguousarray(A[rank * rows:(rank + 1) * rows]))
        Bt = torch.from_numpy(B)
        D = DistributedOzakiCRT(ops=OracleOps(O))
        if mode == "fail" and rank == 1:
            raise RuntimeError("injected failure on rank 1 before the first collective")
        C, info = D.run(Al, Bt)
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


def test_row_blocks_equal_single_process(oracle, tmp_path, pkg):
    alive = _spawn(2, "ok", tmp_path)
    assert not any(alive)
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    A, B = pkg.make_inputs(128, 256, 96, 2.0, seed=31)
    Cref, iref = oracle.run(A, B)
    C = np.concatenate([np.load(os.path.join(tmp_path, f"C_{r}.npy")) for r in range(2)])
    np.testing.assert_array_equal(C.view(np.uint64), Cref.view(np.uint64))
    infos = [eval(open(os.path.join(tmp_path, f"info_{r}.txt")).read()) for r in range(2)]
    assert infos[0] == infos[1]
    assert infos[0][:3] == (iref["N"], iref["p"], iref["p_req"])
    C22ref, i22 = oracle.run(A, B, force_N=22)
    C22 = np.concatenate([np.load(os.path.join(tmp_path, f"C22_{r}.npy")) for r in range(2)])
    np.testing.assert_array_equal(C22.view(np.uint64), C22ref.view(np.uint64))
    assert infos[0][3:] == (22, i22["p"])


def test_failed_rank_ends_peers_collective_with_error(tmp_path):
    alive = _spawn(2, "fail", tmp_path)
    assert not any(alive), "a rank hung after its peer failed"
    assert os.path.exists(os.path.join(tmp_path, "error_1.txt"))
    # rank 0 must have seen an error from its collective (timeout or closed connection), not a hang
    assert os.path.exists(os.path.join(tmp_path, "error_0.txt"))
