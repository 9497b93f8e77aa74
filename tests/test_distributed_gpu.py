"""DistributedOzakiCRT on the GPU through NCCL with one rank (the CUDA ops and the collectives of the multi-GPU
path; the multi-rank bookkeeping is covered by tests/test_distributed_gloo.py).  The block result must equal the
single-engine product bit for bit."""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_distributed_one_rank_nccl(pkg, engine):
    import torch
    import torch.distributed as dist
    from matrix_numbers_b200.distributed import DistributedOzakiCRT
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", 0))
    try:
        A, B = pkg.make_inputs(256, 512, 384, 2.0, seed=8)
        Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        D = DistributedOzakiCRT(grid=(1, 1))
        C, info = D.run(Ad, Bd)
        Cr, ir = engine.run(Ad, Bd)
        assert (info["N"], info["p"], info["preq"]) == (ir["N"], ir["p"], ir["p_req"])
        assert torch.equal(C, Cr)
        C2, i2 = D.run(Ad, Bd, force_N=20)
        C2r, _ = engine.run(Ad, Bd, force_N=20)
        assert i2["N"] == 20 and torch.equal(C2, C2r)
        C3, i3c = D.run(Ad, Bd, certify=True)
        C3r, i3r = engine.run(Ad, Bd, certify=True)
        assert i3c["certified"] and (i3c["N"], i3c["p"], i3c["preq"]) == (i3r["N"], i3r["p"], i3r["p_req"])
        assert i3c["uncertified_entries"] == i3r["uncertified_entries"] and torch.equal(C3, C3r)
        jobs, want = [], []
        for seed in range(3):
            A2, B2 = pkg.make_inputs(256, 512, 384, 1.0 + seed, seed=20 + seed)
            jobs.append((torch.from_numpy(A2).pin_memory(), torch.from_numpy(B2).pin_memory(), None))
            want.append(D.run(torch.from_numpy(A2).cuda(), torch.from_numpy(B2).cuda(), certify=seed == 1))
        got = D.run_host_many(jobs[:1], certify=False) + D.run_host_many(jobs[1:2], certify=True) + \
            D.run_host_many(jobs[2:], certify=False)
        for (Cg, ig), (Cw, iw) in zip(got, want):
            assert (ig["N"], ig["p"]) == (iw["N"], iw["p"])
            assert torch.equal(Cg, Cw.cpu())
        many = D.run_host_many([jobs[0], jobs[2], jobs[0]])
        assert torch.equal(many[0][0], want[0][0].cpu()) and torch.equal(many[1][0], want[2][0].cpu())
        assert torch.equal(many[2][0], want[0][0].cpu())
        Bn = Bd.clone()
        Bn[3, 4] = float("nan")
        _, i3 = D.run(Ad, Bn)
        assert i3.get("fallback")
    finally:
        dist.destroy_process_group()
