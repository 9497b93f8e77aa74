"""The reference's contract and control tests (ozaki_engine.py cmd_config :1586-1615, cmd_check :1769-1840, cmd_instr
controls :2144-2158) on this engine: configurations from the data-independent table meet their guaranteed sigma on
the G / X / W families; the Lemma L1 audit shows no violation with the true bound and catches a bound shrunk 100x;
every entry of the dynamic-rule result is at least as close to the N = 32 result as native DGEMM is; a NaN input on
the timed path is reported as a fallback."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N1024 = 1024


def family(pkg, fam):
    if fam == "W":
        return pkg.make_inputs_w(N1024)
    phi = {"G": 0.5, "X": 2.0}[fam]
    return pkg.make_inputs(N1024, N1024, N1024, phi, seed=0)


@pytest.mark.parametrize("fam", ["G", "X", "W"])
@pytest.mark.parametrize("sigma_t", [2.0 ** -40, 2.0 ** -50])
def test_config_contract(pkg, engine, fam, sigma_t):
    import torch
    A, B = family(pkg, fam)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    cfg = pkg.pick_config(pkg.make_config_table(), N1024, sigma_t)
    Cn = Ad @ Bd
    S = pkg.Sample(Ad, Bd, Cn)
    C, info = engine.run(Ad, Bd, C=torch.empty_like(Cn), config=cfg)
    assert not info.get("fallback")
    h = info["stats"]
    Cs = C[S.tri][:, S.tci].cpu().numpy()
    err = np.abs(Cs - S.ref)
    lim = cfg["sigma"] * N1024 * np.exp2(np.asarray(h["r"], np.float64)[S.ri][:, None]
                                         + np.asarray(h["c"], np.float64)[S.ci][None, :]) \
        + 2.0 ** -53 * (np.abs(Cs) + np.abs(S.ref)) * (1 + 1e-9)
    assert int((err > lim).sum()) == 0, float((err / lim).max())


def test_audit_controls(pkg, engine):
    import torch
    A, B = family(pkg, "G")
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    S = pkg.Sample(Ad, Bd, Ad @ Bd)
    C, info = engine.run(Ad, Bd, force_N=8)          # p ~ 21: the quantisation error dominates the final rounding
    assert pkg.audit_bound(S, info, N1024, C)["violations"] == 0
    assert pkg.audit_bound(S, info, N1024, C, scale=0.01)["violations"] > 0


@pytest.mark.parametrize("fam", ["G", "X", "W"])
def test_full_matrix_not_worse_than_native(pkg, engine, fam):
    import torch
    A, B = family(pkg, fam)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    C, info = engine.run(Ad, Bd)
    C32, _ = engine.run(Ad, Bd, force_N=32)
    Cn = Ad @ Bd
    Dm = torch.abs(Ad) @ torch.abs(Bd)
    pos = Dm > 0
    den = Dm.clamp_min(1e-300)
    e2 = float(((C - C32).abs() / den)[pos].max())
    e2n = float(((Cn - C32).abs() / den)[pos].max())
    e1 = float((C - C32).abs().max() / C32.abs().max())
    e1n = float((Cn - C32).abs().max() / C32.abs().max())
    assert e2 <= e2n and e1 <= e1n, (e2, e2n, e1, e1n)


def test_timed_path_fallback_flag(pkg, engine):
    import torch
    A, B = family(pkg, "G")
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    Cx = torch.empty(N1024, N1024, dtype=torch.float64, device="cuda")
    _, i_ok = engine.run(Ad, Bd, C=Cx, graph=True)
    An = Ad.clone()
    An[3, 5] = float("nan")
    _, i_nan = engine.run(An, Bd, C=Cx, graph=True)
    assert not i_ok.get("fallback") and i_nan.get("fallback")


def test_error_conventions(pkg, engine):
    """The reference's error conventions (ozaki_engine.py:1315-1316 asserts; a RuntimeError from the GPU layer):
    shape violations and wrong dtypes raise AssertionError before any launch, eagerly and on the timed path;
    zero-sized problems are rejected by the C ABI's argument checks as a RuntimeError."""
    import torch
    A, B = pkg.make_inputs(64, 128, 64, 0.5, seed=4)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    bad = [(Ad[:, :120].contiguous(), Bd[:120]),             # k % 32 != 0
           (Ad, Bd[:, :48].contiguous()),                     # n % 32 != 0
           (Ad[:62].contiguous(), Bd),                        # m % 4 != 0
           (Ad.float(), Bd),                                  # not float64
           (Ad.t(), Bd),                                      # not contiguous (and k differs)
           (Ad, Bd[:96])]                                     # inner dimensions differ
    for a, b in bad:
        with pytest.raises(AssertionError):
            engine.run(a, b)
        with pytest.raises(AssertionError):
            engine.run(a, b, C=torch.empty(a.shape[0], b.shape[1], dtype=torch.float64, device="cuda"), graph=True)
    with pytest.raises(AssertionError):
        engine.run(Ad, Bd, C=torch.empty(64, 32, dtype=torch.float64, device="cuda"))   # C of the wrong shape
    with pytest.raises(RuntimeError):
        engine.run(Ad[:0], Bd)                                                        # m = 0
    C, info = engine.run(Ad, Bd)                                 # the engine is still usable afterwards
    Cr, _ = engine.run(Ad, Bd)
    assert torch.equal(C, Cr)
