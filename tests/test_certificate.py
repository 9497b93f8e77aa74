"""Full-matrix certificate (reference full_certificate, code/ozaki_engine.py:1542-1583): the tcgen05 FP16 kernel with
the bound reduced in its epilogue, against the numpy restatement of the reference arithmetic (oracle.full_certificate).

The FP16 operands are bit-identical to the reference's; the product is summed in FP32 on the tensor cores in a
different order than cuBLAS (and than the oracle's float64 sum), so D agrees to within the FP32 accumulation error,
which the certificate's 8 k 2^-24 derating covers: D must stay below the exact sum of |A||B| on every entry."""
import numpy as np
import pytest


def test_oracle_certificate_is_a_lower_bound(pkg, oracle):
    A, B = pkg.make_inputs(48, 256, 64, 2.0, seed=9)
    B[:, 3] = 0.0
    st = oracle.stats(A, B, True)
    cert = oracle.full_certificate(A, B, st)
    exact = np.abs(A) @ np.abs(B)
    assert np.all(cert["D"][exact > 0] <= exact[exact > 0])
    assert cert["uncertified"] == 48                      # the zero column
    assert np.all(cert["D"][:, 3] == 0)


def test_fast_bound_is_below_the_formula():
    """The certificate kernel skips an entry when an FP32 lower bound of its xmax is at or above the running minimum
    (csrc/certificate.cu, fast_term): with the row and column scalings cancelled, L = c8 v s / (4 s^2 + k4 v).
    Over the whole range where the kernel uses it (2^r, 2^c in [2^-200, 2^200], row and column terms in
    [2^-59, 2^60], v in [2^-48, 2^31], tau and safety in [2^-100, 2^100]) L must stay below the reference's FP64
    chain, with the reciprocal one ulp high (the worst case of rcp.approx.f32), and within 2^-7 of it on ordinary
    data (so that it does skip)."""
    rng = np.random.default_rng(1)
    f32 = np.float32
    checked = 0
    for trial in range(120):
        n = 4000
        ext = trial % 4
        r = rng.integers(-200, 201, n) if ext else rng.integers(-5, 6, n)
        c = rng.integers(-200, 201, n) if ext else rng.integers(-5, 6, n)
        a = np.exp2(rng.uniform(-59, 60, n)) if ext == 1 else np.exp2(rng.uniform(-1, 12, n))
        b = np.exp2(rng.uniform(-59, 60, n)) if ext == 2 else np.exp2(rng.uniform(-1, 12, n))
        v32 = (np.exp2(rng.uniform(-48, 31, n)) if ext == 3 else rng.uniform(1, 4096, n)).astype(f32)
        v = v32.astype(np.float64)
        k = int(rng.choice([32, 4096, 65536, 262144]))
        tau = 2.0 ** rng.uniform(-100, 100) if ext else 2.0 ** -52
        safety = 2.0 ** rng.uniform(-100, 100) if ext else float(rng.choice([2.0, 3.0, 0.75]))
        derate = 1.0 - 8.0 * k * 2.0 ** -24
        kap = tau * derate / safety
        c8, k4 = 8.0 * kap * (1 - 2.0 ** -8), 4.0 * k * kap
        if not (2.0 ** -110 <= c8 <= 2.0 ** 110 and 2.0 ** -110 <= k4 <= 2.0 ** 110):
            continue                                          # the kernel's host code disables the bound there
        rI, cJ = np.ldexp(1.0, r), np.ldexp(1.0, c)
        sA, sB = a * rI, b * cJ
        with np.errstate(all="ignore"):
            D = ((v * derate) * rI) * cJ
            thr = (tau * D) / safety
            F1 = 0.5 * (rI * sB + cJ * sA)
            F2 = ((0.25 * k) * rI) * cJ
            x = (2.0 * thr) / (F1 + np.sqrt(F1 * F1 + (4.0 * F2) * thr))
            s = (sA / rI).astype(f32) + (sB / cJ).astype(f32)
            den = (s * s) * f32(4.0) + f32(k4) * v32
            q = (v32 * s) * np.nextafter(f32(1.0) / den, f32(np.inf))
            L = q * f32(c8)
        used = (L >= 2.0 ** -100) & np.isfinite(L) & (q >= f32(2.0 ** -126))
        ratio = L[used].astype(np.float64) / x[used]
        assert ratio.max() < 1.0
        if ext == 0:
            assert ratio.min() > 1.0 - 2.0 ** -7
        checked += int(used.sum())
    assert checked > 200000


def test_fast_bound_small_terms_large_kappa():
    """The corner where the bound's quotient q = v s / den leaves FP32's normal range: k4 = 4 k kap at the top of the
    allowed range (2^110), row and column terms from 2^-59 up.  q is then subnormal or zero; the kernel does not skip
    on a subnormal q, and every entry it would skip on has L below the reference's FP64 xmax."""
    f32 = np.float32
    rng = np.random.default_rng(5)
    k = 262144
    derate = 1.0 - 8.0 * k * 2.0 ** -24
    tau = 2.0 ** -52
    safety = tau * derate / 2.0 ** 90                     # kap = 2^90: k4 = 2^110, c8 ~ 2^93
    kap = tau * derate / safety
    c8, k4 = 8.0 * kap * (1 - 2.0 ** -8), 4.0 * k * kap
    assert 2.0 ** -110 <= c8 <= 2.0 ** 110 and k4 <= 2.0 ** 110
    n = 100000
    subnormal_seen = 0
    for e in range(-59, 61, 4):
        a = np.exp2(e + rng.uniform(-1, 0, n))
        b = np.exp2(rng.uniform(-59, e, n))
        v32 = np.exp2(rng.uniform(-48, 31, n)).astype(f32)
        v = v32.astype(np.float64)
        with np.errstate(all="ignore"):
            D = v * derate
            thr = (tau * D) / safety
            F1 = 0.5 * (b + a)
            F2 = 0.25 * k
            x = (2.0 * thr) / (F1 + np.sqrt(F1 * F1 + (4.0 * F2) * thr))
            s = a.astype(f32) + b.astype(f32)
            den = (s * s) * f32(4.0) + f32(k4) * v32
            q = (v32 * s) * np.nextafter(f32(1.0) / den, f32(np.inf))
            L = q * f32(c8)
        subnormal_seen += int(((q > 0) & (q < f32(2.0 ** -126))).sum())
        used = (L >= 2.0 ** -100) & np.isfinite(L) & (q >= f32(2.0 ** -126))
        assert np.all(L[used].astype(np.float64) < x[used])
    assert subnormal_seen > 0


def _dev_stats(torch, E, Ad, Bd):
    m, k = Ad.shape
    b = E.buffers(m, Bd.shape[1], k, 20)
    E.stats(Ad, Bd, b, True)
    return b


def _tol(k):
    return 3.0 * (k + 2) * 2.0 ** -24


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,phi,safety", [(4096, 64, 4096, 0.5, 2.0), (2048, 96, 1024, 2.0, 3.0),
                                              (260, 544, 96, 1.0, 3.0), (128, 32, 256, 3.0, 0.75)])
def test_certificate_min_is_exact_over_its_own_D(pkg, engine, m, k, n, phi, safety):
    """The kernel skips entries whose xmax provably cannot lower the running minimum.  Its minimum must equal, bit for
    bit, the minimum of the reference formula (:1565-1569) evaluated exactly over the kernel's own D (written out
    through D_out), in the reference's operation order; the uncertified count is the number of entries with D <= 0.
    4096 x 4096 gives 512 tiles, several per CTA, so the minimum published between tiles is exercised; safety 3 and
    0.75 are not powers of two."""
    import torch
    from matrix_numbers_b200.certificate import certificate_device
    tau = 2.0 ** -52
    A, B = pkg.make_inputs(m, k, n, phi, seed=3 * m + n)
    A[1, :] = 0.0
    B[:, 2] = 0.0
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    b = _dev_stats(torch, engine, Ad, Bd)
    Dd = torch.empty(m, n, dtype=torch.float64, device="cuda")
    w = certificate_device(engine, Ad, Bd, b["gam"], b["r"], b["c"], b["sA"], b["sB"], tau=tau, safety=safety, D_out=Dd)
    torch.cuda.synchronize()
    assert int(w["err"].item()) == 0
    D = Dd.cpu().numpy()
    rI = np.ldexp(1.0, b["r"].cpu().numpy().astype(np.int64))[:, None]
    cJ = np.ldexp(1.0, b["c"].cpu().numpy().astype(np.int64))[None, :]
    sA = b["sA"].cpu().numpy()[:, None]
    sB = b["sB"].cpu().numpy()[None, :]
    with np.errstate(all="ignore"):
        thr = (tau * D) / safety
        F1 = 0.5 * (rI * sB + cJ * sA)
        F2 = ((0.25 * k) * rI) * cJ
        x = (2.0 * thr) / (F1 + np.sqrt(F1 * F1 + (4.0 * F2) * thr))
    pos = D > 0
    assert int(w["unc"].item()) == int((~pos).sum()) >= n + m - 1
    cand = x[pos & ~np.isnan(x)].view(np.uint64)
    want = int(cand.min()) if cand.size else 2 ** 64 - 1
    got = int(w["xmin"].view(torch.int64).item()) & (2 ** 64 - 1)
    assert got == want, (got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,phi", [(128, 256, 256, 1.0), (260, 544, 96, 2.0), (512, 2048, 384, 0.5),
                                       (64, 96, 512, 3.0)])
def test_certificate_kernel_vs_oracle(pkg, oracle, engine, m, k, n, phi):
    import torch
    from matrix_numbers_b200.certificate import certificate_device, required_p
    A, B = pkg.make_inputs(m, k, n, phi, seed=m + n)
    A[5, :] = 0.0
    B[:, 7] = 0.0
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    b = _dev_stats(torch, engine, Ad, Bd)
    st = oracle.stats(A, B, True)
    Dd = torch.empty(m, n, dtype=torch.float64, device="cuda")
    w = certificate_device(engine, Ad, Bd, b["gam"], b["r"], b["c"], b["sA"], b["sB"], D_out=Dd)
    torch.cuda.synchronize()
    assert int(w["err"].item()) == 0
    ref = oracle.full_certificate(A, B, st)
    D = Dd.cpu().numpy()
    exact = np.abs(A) @ np.abs(B)
    pos = ref["D"] > 0
    assert np.array_equal(D > 0, pos)
    assert int(w["unc"].item()) == ref["uncertified"] == int((~pos).sum())
    rel = np.abs(D[pos] - ref["D"][pos]) / ref["D"][pos]
    assert rel.max() <= _tol(k)
    # a lower bound of the exact sum wherever the reference's arithmetic gives one: its FP16 rounding of magnitudes in
    # the subnormal range (below 2^-14) can round up by far more than the (1 - 2^-10) pre-scaling (at phi = 3 one
    # entry of the restatement exceeds the exact sum by 0.8%); there the kernel must agree with the restatement
    ok_ref = ref["D"][pos] <= exact[pos]
    assert np.all(D[pos][ok_ref] <= exact[pos][ok_ref] * (1 + 2.0 ** -40))
    assert ok_ref.mean() > 0.99
    preq, need = required_p(int(w["xmin"].view(torch.int64).item()))
    assert abs(need - ref["need"]) <= _tol(k)
    frac = ref["need"] + 1e-9 - np.floor(ref["need"] + 1e-9)
    if _tol(k) < frac < 1 - _tol(k):                         # not within the tolerance of an integer boundary
        assert preq == ref["preq"]


@pytest.mark.gpu
def test_full_certificate_api(pkg, oracle, engine):
    import torch
    m, k, n = 256, 1024, 256
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=4)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = engine.run(Ad, Bd)
    cert = pkg.full_certificate(engine, Ad, Bd, info)
    assert set(cert) == {"N_full", "preq_full", "preq_sampled", "uncertified_entries", "cost_ms", "N_sampled",
                         "sampled_config_fully_certified"}
    ref = oracle.full_certificate(A, B, oracle.stats(A, B, True))
    assert abs(cert["preq_full"] - ref["preq"]) <= 1
    assert cert["uncertified_entries"] == ref["uncertified"] == 0
    assert cert["preq_sampled"] == info["p_req"] and cert["N_sampled"] == info["N"]
    assert cert["preq_full"] >= info["p_req"] - 1          # every probe entry is one of the certified entries
    Nf = cert["N_full"]
    assert Nf is not None and pkg.pmax_bits(Nf, info["nuA"], info["nuB"], k) >= cert["preq_full"]
    assert Nf == 6 or pkg.pmax_bits(Nf - 1, info["nuA"], info["nuB"], k) < cert["preq_full"]
    assert cert["sampled_config_fully_certified"] == (info["N"] >= Nf)


@pytest.mark.gpu
@pytest.mark.parametrize("m,k,n,phi", [(256, 1024, 256, 2.0), (128, 512, 384, 0.5)])
def test_run_certified(pkg, oracle, engine, m, k, n, phi):
    """The certified rule in the timed path: N from the certificate of every entry, core bit-exact."""
    import torch
    A, B = pkg.make_inputs(m, k, n, phi, seed=k + n)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = engine.run(Ad, Bd, certify=True)
    assert info["certified"] and not info.get("fallback")
    st = oracle.stats(A, B, True)
    ref = oracle.full_certificate(A, B, st)
    assert abs(info["p_req"] - ref["preq"]) <= 1
    N, p = info["N"], info["p"]
    assert p == oracle.pmax_bits(N, info["nuA"], info["nuB"], k) >= info["p_req"]
    assert N == 6 or oracle.pmax_bits(N - 1, info["nuA"], info["nuB"], k) < info["p_req"]
    assert np.array_equal(C.cpu().numpy(), oracle.core(A, B, st, N, p))
    _, sampled = engine.run(Ad, Bd)
    assert N >= sampled["N"] - 1                              # the certificate covers the probe entries too
    Cg = torch.empty_like(C)
    for _ in range(2):
        _, ig = engine.run(Ad, Bd, Cg, graph=True, certify=True)
        assert (ig["N"], ig["p"], ig["preq"]) == (N, p, info["p_req"]) and ig["certified"]
        assert torch.equal(Cg, C)
