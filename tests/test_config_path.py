"""Configuration-table fast path: ``run(..., config=pick_config(...), graph=True)`` runs statistics, the forced rule
(no probe product), the core and the decision copy as one CUDA graph with one synchronisation.  Its results equal the
eager forced run and the CPU oracle bit for bit; a configuration the data cannot honour falls back to native FP64
like the reference's (ozaki_engine.py:1486-1497)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,n,phi", [(128, 384, 96, 1.0), (256, 1024, 512, 0.5), (64, 2048, 64, 2.0)])
def test_config_graph_matches_oracle(pkg, oracle, engine, m, k, n, phi):
    import torch
    A, B = pkg.make_inputs(m, k, n, phi, seed=m + k)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    cfg = pkg.pick_config(pkg.make_config_table(), k, 2.0 ** -50)
    Cref, iref = oracle.run(A, B, force_N=cfg["N"], force_p=cfg["p"])
    C = torch.empty(m, n, dtype=torch.float64, device="cuda")
    for _ in range(3):                                       # capture, then replays
        C.fill_(0.0)
        C2, info = engine.run(Ad, Bd, C, config=cfg, graph=True)
        assert C2 is C and not info.get("fallback")
        assert (info["N"], info["p"]) == (cfg["N"], cfg["p"]) == (iref["N"], iref["p"])
        assert np.array_equal(C.cpu().numpy(), Cref)
    Ce, _ = engine.run(Ad, Bd, config=cfg)
    assert torch.equal(Ce, C)


def test_config_graph_rejected_and_nonfinite(pkg, engine):
    import torch
    A, B = pkg.make_inputs(128, 256, 64, 1.0, seed=2)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty(128, 64, dtype=torch.float64, device="cuda")
    _, info = engine.run(Ad, Bd, C, config={"N": 8, "p": 200}, graph=True)
    assert info.get("fallback")
    assert torch.equal(C, Ad @ Bd)
    Bd[3, 5] = float("nan")
    _, info = engine.run(Ad, Bd, C, config={"N": 16, "p": 40}, graph=True)
    assert info.get("fallback")
    assert torch.equal(torch.isnan(C), torch.isnan(Ad @ Bd))
