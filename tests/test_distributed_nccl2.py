"""DistributedOzakiCRT over NCCL on two GPUs (skipped when the machine has fewer): the pre-placed grid of C blocks, B
broadcast from one rank inside the call, A, B on one rank with scatter / broadcast / gather, and host buffers of which
each rank loads only its share (run_host_many(shares=True)); and on four GPUs (a 2 x 2 grid) B's column blocks sent
from one rank to their grid columns, and the host-share path.  Every C must equal the single-GPU product bit
for bit, and every rank must decide the same (N, p).  The ranks are spawned child processes, one per GPU; the process
group has a short timeout so that a failure ends the test instead of hanging it."""
import os
import socket
import sys
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHAPE = (512, 768, 384)                        # m, k, n


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _host_shares(pkg, D, A, B, rank):
    """DistributedOzakiCRT.run_host_many(shares=True) over three jobs (B, -B, B): rank (a, b) passes rows / S rows
    of A's row block a and k / R rows of B's column block b from pinned host memory.  The second product must be the
    negation of the first (the symmetric lift and the rounding are odd), the third equal to the first."""
    import torch
    R, S = D.R, D.S
    a, b = divmod(rank, S)
    m, k = A.shape
    n = B.shape[1]
    br, bc = m // R, n // S
    sr, sk = br // S, k // R
    Ah = torch.from_numpy(np.ascontiguousarray(A[a * br + b * sr:a * br + (b + 1) * sr])).pin_memory()
    Bh = torch.from_numpy(np.ascontiguousarray(B[a * sk:(a + 1) * sk, b * bc:(b + 1) * bc])).pin_memory()
    Bn = torch.from_numpy(np.ascontiguousarray(-B[a * sk:(a + 1) * sk, b * bc:(b + 1) * bc])).pin_memory()
    res = D.run_host_many([(Ah, Bh, None), (Ah, Bn, None), (Ah, Bh, None)], shares=True)
    C0, C1, C2 = (x[0].numpy() for x in res)
    assert np.array_equal(C1.view(np.uint64), (-C0).view(np.uint64)), "second job (negated B)"
    assert np.array_equal(C2.view(np.uint64), C0.view(np.uint64)), "third job (slot reuse)"
    info = res[0][1]
    return C0.copy(), (info["N"], info["p"], info["preq"])


def _worker(rank, world, port, outdir):
    try:
        sys.path.insert(0, ROOT)
        import datetime

        import torch
        import torch.distributed as dist

        import __graft_entry__
        pkg = __graft_entry__.load_package()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from matrix_numbers_b200.distributed import DistributedOzakiCRT
        m, k, n = SHAPE
        A, B = pkg.make_inputs(m, k, n, 2.0, seed=44)
        rows = m // world
        A_rows = torch.from_numpy(np.ascontiguousarray(A[rank * rows:(rank + 1) * rows])).to(dev)
        B_full = torch.from_numpy(B).to(dev)
        D = DistributedOzakiCRT(grid=(world, 1))
        out = {}
        C, info = D.run(A_rows, B_full)
        out["pre"] = (C.cpu().numpy(), (info["N"], info["p"], info["preq"]))
        root = world - 1
        C, info = D.run_broadcast_b(A_rows, B_full if rank == root else None, root=root)
        out["bcast"] = (C.cpu().numpy(), (info["N"], info["p"], info["preq"]))
        A_full = torch.from_numpy(A).to(dev)
        C, info = D.run_from_root(A_full if rank == root else None, B_full if rank == root else None, root=root)
        out["root"] = (C.cpu().numpy(), (info["N"], info["p"], info["preq"]))
        # a 1 x 2 grid: B's column blocks from the root to their grid columns (the root's own column included)
        D12 = DistributedOzakiCRT(grid=(1, world))
        cols = n // world
        parts = [B_full[:, q * cols:(q + 1) * cols].contiguous() for q in range(world)]
        C, info = D12.run_broadcast_b(A_full, parts if rank == root else None, root=root)
        out["cols"] = (C.cpu().numpy(), (info["N"], info["p"], info["preq"]))
        # host buffers, each rank loading only its share of its blocks, on both grids
        for name, Dx in (("hostR", D), ("hostS", D12)):
            out[name] = _host_shares(pkg, Dx, A, B, rank)
        torch.cuda.synchronize()
        D.engine.check_errors()
        for name, (Cn, dec) in out.items():
            np.save(os.path.join(outdir, f"{name}_{rank}.npy"), Cn)
            with open(os.path.join(outdir, f"{name}_{rank}.txt"), "w") as f:
                f.write(repr(dec))
        if rank == 0:
            E = pkg.OzakiCRT()
            Cs, i_s = E.run(A_full, B_full)
            np.save(os.path.join(outdir, "single.npy"), Cs.cpu().numpy())
            with open(os.path.join(outdir, "single.txt"), "w") as f:
                f.write(repr((i_s["N"], i_s["p"], i_s["p_req"])))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"error_{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())


def test_two_ranks_nccl_bit_exact(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=240)
    alive = [p.is_alive() for p in ctx.processes]
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert not any(alive), "a rank did not finish"
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    single = np.load(os.path.join(tmp_path, "single.npy")).view(np.uint64)
    want = eval(open(os.path.join(tmp_path, "single.txt")).read())
    for name in ("pre", "bcast", "hostR"):
        C = np.concatenate([np.load(os.path.join(tmp_path, f"{name}_{r}.npy")) for r in range(world)])
        np.testing.assert_array_equal(C.view(np.uint64), single, err_msg=name)
    np.testing.assert_array_equal(np.load(os.path.join(tmp_path, f"root_{world - 1}.npy")).view(np.uint64), single)
    for name in ("cols", "hostS"):
        C = np.concatenate([np.load(os.path.join(tmp_path, f"{name}_{r}.npy")) for r in range(world)], axis=1)
        np.testing.assert_array_equal(C.view(np.uint64), single, err_msg=name)
    for name in ("pre", "bcast", "root", "cols", "hostR", "hostS"):
        for r in range(world):
            assert eval(open(os.path.join(tmp_path, f"{name}_{r}.txt")).read()) == want, (name, r)


def _worker_grid(rank, world, port, outdir):
    """2 x 2 grid, B only on rank 0 as its two column blocks: column block b is sent to grid column b."""
    try:
        sys.path.insert(0, ROOT)
        import datetime

        import torch
        import torch.distributed as dist

        import __graft_entry__
        pkg = __graft_entry__.load_package()
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        from matrix_numbers_b200.distributed import DistributedOzakiCRT
        m, k, n = SHAPE
        A, B = pkg.make_inputs(m, k, n, 2.0, seed=44)
        R, S = 2, 2
        a, b = divmod(rank, S)
        rows, cols = m // R, n // S
        A_rows = torch.from_numpy(np.ascontiguousarray(A[a * rows:(a + 1) * rows])).to(dev)
        parts = [torch.from_numpy(np.ascontiguousarray(B[:, q * cols:(q + 1) * cols])).to(dev) for q in range(S)]
        D = DistributedOzakiCRT(grid=(R, S))
        C, info = D.run_broadcast_b(A_rows, parts if rank == 0 else None, root=0)
        C2, info2 = D.run_broadcast_b(A_rows, torch.from_numpy(B).to(dev) if rank == 0 else None, root=0)
        C3, dec3 = _host_shares(pkg, D, A, B, rank)
        torch.cuda.synchronize()
        D.engine.check_errors()
        np.save(os.path.join(outdir, f"grid_{rank}.npy"), C.cpu().numpy())
        np.save(os.path.join(outdir, f"grid2_{rank}.npy"), C2.cpu().numpy())
        np.save(os.path.join(outdir, f"grid3_{rank}.npy"), C3)
        with open(os.path.join(outdir, f"grid_{rank}.txt"), "w") as f:
            f.write(repr(((info["N"], info["p"], info["preq"]), (info2["N"], info2["p"], info2["preq"]), dec3)))
        if rank == 0:
            E = pkg.OzakiCRT()
            Cs, i_s = E.run(torch.from_numpy(A).to(dev), torch.from_numpy(B).to(dev))
            np.save(os.path.join(outdir, "single.npy"), Cs.cpu().numpy())
            with open(os.path.join(outdir, "single.txt"), "w") as f:
                f.write(repr((i_s["N"], i_s["p"], i_s["p_req"])))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:
        with open(os.path.join(outdir, f"error_{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())


def test_four_ranks_grid_broadcast_bit_exact(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if not torch.cuda.is_available() or torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    world = 4
    ctx = mp.start_processes(_worker_grid, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=240)
    alive = [p.is_alive() for p in ctx.processes]
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    assert not any(alive), "a rank did not finish"
    errs = [f for f in os.listdir(tmp_path) if f.startswith("error_")]
    assert not errs, open(os.path.join(tmp_path, errs[0])).read()
    single = np.load(os.path.join(tmp_path, "single.npy")).view(np.uint64)
    want = eval(open(os.path.join(tmp_path, "single.txt")).read())
    for name in ("grid", "grid2", "grid3"):
        C = np.concatenate([np.concatenate([np.load(os.path.join(tmp_path, f"{name}_{a * 2 + b}.npy"))
                                            for b in range(2)], axis=1) for a in range(2)])
        np.testing.assert_array_equal(C.view(np.uint64), single, err_msg=name)
    for r in range(world):
        got = eval(open(os.path.join(tmp_path, f"grid_{r}.txt")).read())
        assert got[0] == want and got[1] == want and got[2] == want, (r, got, want)
