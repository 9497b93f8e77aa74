"""Persistent fixed operand mode (PersistA, reference code/ozaki_engine.py:2417-2466): A encoded once at (N, p) with
inside scaling off, then products with several B.  Bit-exact against the CPU restatement (oracle.persist_product),
and, when p stays safe, against the ordinary engine run with inside scaling off and the same forced (N, p)."""
import numpy as np
import pytest


def inputs(pkg, m, k, n, phi, seed):
    A, B0 = pkg.make_inputs(m, k, n, phi, seed=seed)
    Bs = [pkg.make_inputs(4, k, n, phi, seed=seed + 1 + j)[1] for j in range(2)]
    return A, B0, Bs


def test_oracle_persist_equals_forced_run(pkg, oracle):
    A, B0, Bs = inputs(pkg, 32, 96, 64, 1.0, 5)
    _, info = oracle.run(A, B0, inside=False)
    N, p = info["N"], info["p"]
    for B in Bs:
        C, d = oracle.persist_product(A, B, N, p)
        if not d["fallback"]:
            Cr, _ = oracle.run(A, B, inside=False, force_N=N, force_p=p)
            assert np.array_equal(C, Cr)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,phi", [(128, 512, 256, 1.0), (64, 1024, 96, 2.0)])
def test_persist_products(pkg, oracle, engine, m, k, n, phi):
    import torch
    A, B0, Bs = inputs(pkg, m, k, n, phi, 11)
    Ad, B0d = torch.from_numpy(A).cuda(), torch.from_numpy(B0).cuda()
    P = pkg.PersistA(engine, Ad, B0d, n)
    _, info = oracle.run(A, B0, inside=False)
    assert (P.N, P.p) == (info["N"], info["p"])
    P.encode()
    C = torch.empty(m, n, dtype=torch.float64, device="cuda")
    for B in [B0] + Bs:
        Bd = torch.from_numpy(B).cuda()
        want, d = oracle.persist_product(A, B, P.N, P.p)
        for _ in range(2):                                  # capture, then replay
            P.product(Bd, C)
            torch.cuda.synchronize()
            assert np.array_equal(C.cpu().numpy(), want)
        N, pB, fb = P.last_decision()
        assert (pB, fb) == (d["p_B"], d["fallback"])
        if not fb:
            Cr = torch.empty_like(C)
            engine.run(Ad, Bd, C=Cr, inside=False, config={"N": P.N, "p": P.p})
            assert torch.equal(Cr, C)


@pytest.mark.gpu
def test_persist_unsafe_B_lowers_p_like_the_reference(pkg, oracle, engine):
    import torch
    m, k, n = 64, 512, 64
    A, _, _ = inputs(pkg, m, k, n, 2.0, 3)
    rng = np.random.default_rng(1)
    B0 = rng.uniform(-1e-3, 1e-3, (k, n))
    B0[np.arange(n) % k, np.arange(n)] = 1.0                 # one dominant entry per column: small column norms
    flat = np.where(rng.random((k, n)) < 0.5, -0.75, 0.75)   # maximal column norms
    Ad, B0d = torch.from_numpy(A).cuda(), torch.from_numpy(B0).cuda()
    P = pkg.PersistA(engine, Ad, B0d, n)
    P.encode()
    want, d = oracle.persist_product(A, flat, P.N, P.p)
    assert d["fallback"] and d["p_B"] < P.p                 # the case this test is about
    C = torch.empty(m, n, dtype=torch.float64, device="cuda")
    P.product(torch.from_numpy(flat).cuda(), C)
    torch.cuda.synchronize()
    assert P.last_decision()[1:] == (d["p_B"], True)
    assert np.array_equal(C.cpu().numpy(), want)
