"""Exact integer product chains in INT8 residue form (matrix_numbers_b200.chain, csrc/chain.cu).

CPU: the fixed-base plane count is the fewest moduli of MODS whose product exceeds 2 R, and the oracle's residue-form
chain (reduce after every product, symmetric range in between) agrees with exact Python-integer products modulo every
modulus.  GPU: the symmetric map of the product planes, and whole chains of 2-4 matrices against the oracle -- the
final planes bit for bit, the reconstructed result as the correctly rounded double of the exact integer product."""
import math

import numpy as np
import pytest


def _ints(rs, shape, b):
    H = 2 ** b - 1
    return rs.randint(-H, H + 1, size=shape, dtype=np.int64) if b < 63 else None


def test_planes_for_is_minimal(pkg):
    mods = pkg.MODS
    for R in [1, 255, 2 ** 40, 3 ** 50, 2 ** 120 + 7, 2 ** 200]:
        N = pkg.planes_for(R)
        assert math.prod(mods[:N]) > 2 * R
        assert N == 1 or math.prod(mods[:N - 1]) <= 2 * R
    assert pkg.planes_for(math.prod(mods)) is None
    assert pkg.chain_bound([3, 5, 7], [32, 64]) == 3 * 5 * 7 * 32 * 64


@pytest.mark.parametrize("q,b,dims", [(2, 20, (64, 96, 32)), (3, 9, (32, 64, 96, 64)), (4, 5, (32, 32, 64, 32, 64))])
def test_oracle_residue_chain_matches_exact(oracle, q, b, dims):
    rs = np.random.RandomState(q * 100 + b)
    mats = [_ints(rs, (dims[s], dims[s + 1]), b) for s in range(q)]
    exact = oracle.chain_exact(mats)
    R = (2 ** b - 1) ** q * math.prod(dims[1:-1])
    assert int(np.max(np.abs(exact))) <= R
    N = 12
    planes = oracle.chain_residues(mats, N)
    for t in range(N):
        np.testing.assert_array_equal(planes[t].astype(np.int64), np.mod(exact, oracle.MODS[t]).astype(np.int64))


# ------------------------------------------------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_residue_symmetric(pkg, engine):
    import torch
    L, ptr = pkg._lib.lib(), pkg._lib.ptr
    N, elems = 32, 4096
    rs = np.random.RandomState(3)
    X = np.stack([rs.randint(0, m, size=elems) for m in pkg.MODS[:N]]).astype(np.uint8)
    X[:, 0], X[:, 1] = 0, 1                                  # the ends of every range
    for t, m in enumerate(pkg.MODS[:N]):
        X[t, 8:12] = [m - 1, (m + 1) // 2, (m + 1) // 2 - 1, m // 2]
    Xd = torch.from_numpy(X).cuda()
    out = torch.empty((N, elems), dtype=torch.int8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    pkg._lib.check(L.ozk_residue_symmetric(ptr(Xd), N, elems, ptr(out), s), "ozk_residue_symmetric")
    pkg._lib.check(L.ozk_residue_symmetric(ptr(Xd), N, elems, ptr(Xd), s), "ozk_residue_symmetric in place")
    mods = np.array(pkg.MODS[:N])[:, None]
    want = np.where(X.astype(np.int64) >= (mods + 1) // 2, X.astype(np.int64) - mods, X.astype(np.int64))
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.int64), want)
    np.testing.assert_array_equal(Xd.cpu().numpy().view(np.int8).astype(np.int64), want)
    assert L.ozk_residue_symmetric(ptr(Xd), N, 24, ptr(out), s) == -1          # not a multiple of 16


@pytest.mark.gpu
@pytest.mark.parametrize("q,b,dims", [(2, 52, (64, 128, 96)), (2, 1, (32, 32, 64)), (3, 20, (64, 96, 128, 64)),
                                      (4, 8, (32, 128, 64, 96, 128)), (3, 30, (128, 256, 64, 160))])
def test_chain_exact(pkg, oracle, engine, q, b, dims):
    import torch
    rs = np.random.RandomState(q * 1000 + b)
    H = 2 ** b - 1
    mats = [rs.randint(-H, H + 1, size=(dims[s], dims[s + 1]), dtype=np.int64) for s in range(q)]
    mats[0][0, :] = H                                        # a row and a column at the bound
    mats[-1][:, 0] = H if q % 2 else -H
    dev = [torch.from_numpy(A.astype(np.float64)).cuda() for A in mats]
    ch = pkg.ResidueChain()
    C, info = ch.product(dev, return_residues=True)
    exact = oracle.chain_exact(mats)
    R = pkg.chain_bound([int(np.abs(A).max()) for A in mats], dims[1:-1])
    assert info["N"] == pkg.planes_for(R) and info["gemms"] == (q - 1) * info["N"]
    X = info["residues"].cpu().numpy()
    np.testing.assert_array_equal(X, oracle.chain_residues(mats, info["N"]))
    want = np.array([[float(v) for v in row] for row in exact])           # correctly rounded (Python int -> float)
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint64), want.view(np.uint64))
    # the reference's model bound H^q k^(q-1) gives at least as many planes and the same value
    C2, i2 = ch.product(dev, b=b)
    assert i2["N"] >= info["N"] and torch.equal(C, C2)


@pytest.mark.gpu
def test_chain_large_exact_in_fp64(pkg, engine):
    """n = 2048, q = 3, 7-bit entries: every entry and partial sum is below 2^53, so the FP64 product on the GPU is the
    exact value -- a size-independent check of the residue chain at a size the object-array oracle cannot reach."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(11)
    mats = [torch.randint(-127, 128, (2048, 2048), generator=g, device="cuda").double() for _ in range(3)]
    C, info = pkg.ResidueChain().product(mats)
    ref = (mats[0] @ mats[1]) @ mats[2]
    assert float(ref.abs().max()) < 2.0 ** 53
    assert torch.equal(C, ref)
    assert info["N"] == pkg.planes_for(pkg.chain_bound([127] * 3, [2048, 2048]))


@pytest.mark.gpu
def test_chain_rejects(pkg, engine):
    import torch
    A = torch.ones(32, 32, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        pkg.ResidueChain().product([A * 0.5, A])             # not integers
    big = torch.full((32, 32), 2.0 ** 52, dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError):
        pkg.ResidueChain().product([big] * 6)                # beyond the 32 moduli
    with pytest.raises(ValueError):
        pkg.ResidueChain().product([A])
