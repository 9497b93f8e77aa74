"""Parity at the benchmark configurations themselves (the shapes and generators the headline numbers are quoted on),
as the reference's own ``cmd_check`` runs at its benchmark sizes (code/ozaki_engine.py:1769-1847).

* c1 (1024^3, phi 0.5, seed 0): the whole eager ``run`` against ``oracle.run`` -- plane count N, p, p_req, probe
  sizes and every entry of C bit for bit; the timed (graph) path gives the same C.
* c2 (4096^3) and c4 (32768 x 8192 x 32768): N, p and p_req against the oracle's rule on the same full statistics
  and probe product, and a 256 x 256 block of C against ``oracle.core`` on those rows and columns with the global
  statistics.
* c3 (16384^3, phi 2): the same decision check, and 16 sampled rows (2048 columns each) bit for bit.
* c5 (2048 x 262144 x 2048, alternating signs, N forced to 16): the decision at full size and a sampled block; and a
  reduced c5 (m = n = 64, k = 262144) whose whole ``run`` equals ``oracle.run``.  k > 131071 lies beyond the
  reference's own limit (:1316), so the oracle's int64 products are the only check there.

Bar: N, p, p_req exact; C bit-exact (exact CRT + the reference's rounding).  Each large test builds its own engine and
frees it, so the device never holds more than one configuration's planes."""
import gc

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_mod(engine):
    import torch
    return torch


def _inputs(pkg, name, m=None, n=None):
    m0, k, n0, phi, alt, force_N, _ = pkg.CONFIGS[name]
    A, B = pkg.make_inputs(m or m0, k, n or n0, phi, 0, alt)
    return A, B, force_N


def _oracle_decision(oracle, A, B, force_N=None):
    """The oracle's statistics over all of A and B, its probe sets and probe product, and its rule."""
    m, k = A.shape
    n = B.shape[1]
    st = oracle.stats(A, B, True)
    I, J = oracle.probe_sets(st, m, n, k, 0)
    D = oracle.probe_D(A, B, I, J) if not force_N else np.zeros((len(I), len(J)))
    return st, oracle.rule(st, m, n, k, I, J, D, force_N=force_N)


def _block_of_oracle(oracle, A, B, st, rows, cols, N, p):
    """oracle.core on rows x cols with the global statistics (gamma of the whole product; r, c of the rows and
    columns): equal to those entries of the whole product."""
    sub = {"gam": st["gam"], "r": st["r"][rows], "c": st["c"][cols]}
    return oracle.core(np.ascontiguousarray(A[rows]), np.ascontiguousarray(B[:, cols]), sub, N, p)


def _bits(x):
    return np.ascontiguousarray(x).view(np.uint64)


def _free(torch, *objs):
    del objs
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def test_c1_whole_product_bit_exact(pkg, oracle, torch_mod):
    torch = torch_mod
    A, B, _ = _inputs(pkg, "c1")
    E = pkg.OzakiCRT()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = E.run(Ad, Bd)
    Cref, iref = oracle.run(A, B)
    assert (info["N"], info["p"], info["p_req"], info["probe"]) == (iref["N"], iref["p"], iref["p_req"], iref["probe"])
    np.testing.assert_array_equal(_bits(C.cpu().numpy()), _bits(Cref))
    Cg = torch.empty_like(C)
    E.run(Ad, Bd, C=Cg, graph=True)
    _, ig = E.run(Ad, Bd, C=Cg, graph=True)
    torch.cuda.synchronize()
    assert (ig["N"], ig["p"], ig["preq"]) == (info["N"], info["p"], info["p_req"])
    assert torch.equal(C, Cg)
    E.check_errors()
    _free(torch, E, Ad, Bd, C, Cg)


@pytest.mark.parametrize("name,block", [("c2", (slice(1024, 1280), slice(2048, 2304))),
                                        ("c4", (slice(20480, 20736), slice(7936, 8192)))])
def test_decision_and_block_bit_exact(pkg, oracle, torch_mod, name, block):
    torch = torch_mod
    A, B, _ = _inputs(pkg, name)
    st, ru = _oracle_decision(oracle, A, B)
    assert not ru["fallback"]
    E = pkg.OzakiCRT()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = E.run(Ad, Bd)
    assert (info["N"], info["p"], info["p_req"]) == (ru["N"], ru["p"], ru["p_req"]), (info, ru)
    rows, cols = block
    want = _block_of_oracle(oracle, A, B, st, rows, cols, ru["N"], ru["p"])
    np.testing.assert_array_equal(_bits(C[rows, cols].cpu().numpy()), _bits(want))
    # the timed path decides the same
    Cg = torch.empty_like(C)
    _, ig = E.run(Ad, Bd, C=Cg, graph=True)
    assert (ig["N"], ig["p"], ig["preq"]) == (ru["N"], ru["p"], ru["p_req"])
    assert torch.equal(Cg[rows, cols], C[rows, cols])
    E.check_errors()
    _free(torch, E, Ad, Bd, C, Cg)


def test_c3_decision_and_sampled_rows_bit_exact(pkg, oracle, torch_mod):
    torch = torch_mod
    A, B, _ = _inputs(pkg, "c3")
    st, ru = _oracle_decision(oracle, A, B)
    assert not ru["fallback"] and 18 <= ru["N"] <= 20
    E = pkg.OzakiCRT()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty((A.shape[0], B.shape[1]), dtype=torch.float64, device="cuda")
    _, ig = E.run(Ad, Bd, C=C, graph=True)               # the benchmark's call
    assert (ig["N"], ig["p"], ig["preq"]) == (ru["N"], ru["p"], ru["p_req"]), (ig, ru)
    rows = np.random.default_rng(3).choice(A.shape[0], 16, replace=False)
    rows.sort()
    cols = slice(6144, 8192)
    want = _block_of_oracle(oracle, A, B, st, rows, cols, ru["N"], ru["p"])
    got = C[torch.as_tensor(rows, device="cuda")][:, cols].cpu().numpy()
    np.testing.assert_array_equal(_bits(got), _bits(want))
    E.check_errors()
    _free(torch, E, Ad, Bd, C)


def test_c5_forced_planes_decision_and_block_bit_exact(pkg, oracle, torch_mod):
    torch = torch_mod
    A, B, force_N = _inputs(pkg, "c5")
    assert force_N == 16 and A.shape[1] == 262144
    st, ru = _oracle_decision(oracle, A, B, force_N=force_N)
    E = pkg.OzakiCRT()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C = torch.empty((A.shape[0], B.shape[1]), dtype=torch.float64, device="cuda")
    _, ig = E.run(Ad, Bd, C=C, graph=True, force_N=force_N)
    assert (ig["N"], ig["p"]) == (ru["N"], ru["p"]), (ig, ru)
    rows, cols = slice(1000, 1008), slice(512, 576)
    want = _block_of_oracle(oracle, A, B, st, rows, cols, ru["N"], ru["p"])
    np.testing.assert_array_equal(_bits(C[rows, cols].cpu().numpy()), _bits(want))
    E.check_errors()
    _free(torch, E, Ad, Bd, C)


def test_c5_reduced_whole_run_bit_exact(pkg, oracle, torch_mod):
    torch = torch_mod
    A, B, force_N = _inputs(pkg, "c5", m=64, n=64)
    E = pkg.OzakiCRT()
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = E.run(Ad, Bd, force_N=force_N)
    Cref, iref = oracle.run(A, B, force_N=force_N)
    assert (info["N"], info["p"]) == (iref["N"], iref["p"]) == (16, iref["p"])
    np.testing.assert_array_equal(_bits(C.cpu().numpy()), _bits(Cref))
    Cg = torch.empty_like(C)
    E.run(Ad, Bd, C=Cg, graph=True, force_N=force_N)
    torch.cuda.synchronize()
    assert torch.equal(C, Cg)
    E.check_errors()
    _free(torch, E, Ad, Bd, C, Cg)
