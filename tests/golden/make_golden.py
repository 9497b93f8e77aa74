"""Generate the golden vectors that pin the CPU oracle (oracle/) to the reference engine.

Run where a checkout of the reference (read-only is enough) is at $OZAKI_REFERENCE:

    OZAKI_REFERENCE=<path of the dl1683/matrix-numbers checkout> python tests/golden/make_golden.py

It imports the reference's ``code/ozaki_engine.py`` on the CPU (no GPU needed; ENGINE_OUT is pointed at a temp
dir) and records, from the reference's OWN functions:

* ``selftest_golden.npz`` / ``selftest_golden.json`` -- the 6 input sets of the reference's ``cmd_selftest``
  (ozaki_engine.py:1682-1704; regenerated here from ``np.random.RandomState(5)`` in the same call order), their
  ``np_stats`` (ozaki_engine.py:1635-1650), the (N, p) pairs the selftest uses (N in 8/14/20/30, p = pmax_bits and
  max(pmax_bits - 9, 6), ozaki_engine.py:1719-1722) and the bit-exact ``expected_core`` result for each pair
  (ozaki_engine.py:1653-1679), stored as SHA-256 digests of the float64 bytes plus a few full arrays;
* ``rule_golden.json`` -- N, p, p_req, probe sizes and worst E/D of the reference's host rule ``choose``
  (ozaki_engine.py:1250-1307) and the dec vector of its device rule ``_rule_device`` (ozaki_engine.py:1372-1426),
  both run on CPU torch tensors, for seeded inputs of the BASELINE generator;
* ``tables_golden.json`` -- ``pmax_bits`` on a grid, ``_pow2tab`` digest, ``_limbs_for``, the float products of
  the moduli, ``make_config_table`` and ``pick_config`` answers (ozaki_engine.py:1104-1147, :1511-1539).

The fixtures are small and committed; the reference itself never has to be present when the tests run.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("OZAKI_REFERENCE", "")


def load_reference():
    if not REF or not os.path.isdir(os.path.join(REF, "code")):
        raise SystemExit("set OZAKI_REFERENCE to the path of a dl1683/matrix-numbers checkout")
    os.environ["ENGINE_OUT"] = tempfile.mkdtemp(prefix="ozaki_ref_out_")
    sys.path.insert(0, os.path.join(REF, "code"))
    import ozaki_engine as oe  # noqa: E402  (the reference, imported read-only)
    return oe


def selftest_inputs():
    """The 6 input sets of the reference's cmd_selftest, in its RandomState(5) call order
    (ozaki_engine.py:1686-1704)."""
    rng = np.random.RandomState(5)

    def gen(kind, m, k, n):
        if kind == "gauss":
            A, B = rng.randn(m, k), rng.randn(k, n)
        elif kind == "graded":
            A = (rng.rand(m, k) - 0.5) * np.exp(2 * rng.randn(m, k))
            B = (rng.rand(k, n) - 0.5) * np.exp(2 * rng.randn(k, n))
        else:
            A, B = rng.randn(m, k), rng.randn(k, n)
            A *= 2.0 ** rng.randint(-90, 90, size=(m, k)) * (rng.rand(m, k) > 0.25)
            B *= 2.0 ** rng.randint(-90, 90, size=(k, n)) * (rng.rand(k, n) > 0.25)
            A[0, :3] = [1.0, -2.0 ** -40, 5e-324 * 3]
            B[:3, 0] = [-1.0, 2.0 ** 30, 1.0]
        return np.ascontiguousarray(A), np.ascontiguousarray(B)

    out = []
    for (m, k, n) in ((64, 64, 64), (32, 96, 64)):
        for kind in ("gauss", "graded", "wide"):
            A, B = gen(kind, m, k, n)
            out.append(((m, k, n), kind, A, B))
    return out


def baseline_inputs(m, k, n, phi, seed=0, alt_sign=False):
    """The BASELINE generator: entries (U(0,1) - 0.5) * exp(phi * N(0,1)), numpy default_rng(seed), A before B,
    U before N; alt_sign makes row i of A |A_il| (-1)^l and B = |B| (fully alternating dot products)."""
    g = np.random.default_rng(seed)
    A = (g.random((m, k)) - 0.5) * np.exp(phi * g.standard_normal((m, k)))
    B = (g.random((k, n)) - 0.5) * np.exp(phi * g.standard_normal((k, n)))
    if alt_sign:
        A = np.abs(A) * np.where(np.arange(k) % 2 == 0, 1.0, -1.0)[None, :]
        B = np.abs(B)
    return np.ascontiguousarray(A), np.ascontiguousarray(B)


RULE_CASES = [
    # (m, k, n, phi, seed, alt_sign, row_scale)   row_scale: multiply row i of A by 2^(s_i), s_i in [-20, 20]
    (128, 128, 128, 0.5, 0, False, False),
    (128, 128, 128, 2.0, 1, False, False),
    (96, 256, 160, 1.0, 2, False, False),
    (200, 64, 136, 0.5, 3, False, True),
    (48, 96, 40, 2.0, 4, False, False),
    (160, 192, 96, 1.0, 5, True, False),
    (256, 320, 256, 2.0, 6, False, True),
    (64, 1024, 64, 0.5, 7, False, False),
]


def rule_inputs(case):
    m, k, n, phi, seed, alt, rs = case
    A, B = baseline_inputs(m, k, n, phi, seed, alt)
    if rs:
        s = np.random.default_rng(1000 + seed).integers(-20, 21, size=m)
        A = np.ascontiguousarray(A * np.exp2(s.astype(np.float64))[:, None])
    return A, B


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    oe = load_reference()
    import torch

    # ---------------------------------------------------------------- selftest cases: stats + exact core
    recs = []
    full = {}
    for ci, ((m, k, n), kind, A, B) in enumerate(selftest_inputs()):
        st = oe.np_stats(A, B, True)
        nuA, nuB = math.sqrt(float(st["nA"].max())), math.sqrt(float(st["nB"].max()))
        rec = {"case": ci, "shape": [m, k, n], "kind": kind, "A_sha": digest(A), "B_sha": digest(B),
               "stats": {x: st[x].tolist() for x in ("gam", "r", "c", "sA", "sB", "nA", "nB")}, "cores": []}
        for N in (8, 14, 20, 30):
            pm = oe.pmax_bits(N, nuA, nuB, k)
            for p in sorted({pm, max(pm - 9, 6)}):
                C = oe.expected_core(A, B, st["gam"], st["r"], st["c"], p)
                rec["cores"].append({"N": N, "p": int(p), "sha": digest(C)})
                if N == 14 and p == pm:
                    full[f"C_{ci}_N{N}_p{p}"] = C
        recs.append(rec)
        print("selftest case", ci, kind, (m, k, n), [(c["N"], c["p"]) for c in rec["cores"]], flush=True)
    ref_self = json.load(open(os.path.join(REF, "results", "engine", "selftest.json")))
    shipped = [(tuple(c["shape"]), c["kind"], c["N"], c["p"]) for c in ref_self["cases"] if "N" in c]
    ours = [((r["shape"][0], r["shape"][1], r["shape"][2]), r["kind"], c["N"], c["p"]) for r in recs for c in r["cores"]]
    json.dump({"cases": recs, "shipped_selftest_np_pairs": [list(map(list, [s[0]])) + list(s[1:]) for s in shipped],
               "np_pairs_match_shipped_selftest": sorted(ours) == sorted(shipped)},
              open(os.path.join(HERE, "selftest_golden.json"), "w"), indent=0)
    np.savez_compressed(os.path.join(HERE, "selftest_golden.npz"), **full)
    print("(N,p) pairs equal to the shipped selftest.json:", sorted(ours) == sorted(shipped), flush=True)

    # ---------------------------------------------------------------- host and device rule on CPU tensors
    oe.DEV = "cpu"
    torch.cuda.current_stream = lambda *a, **kw: types.SimpleNamespace(synchronize=lambda: None)
    rules = []
    for case in RULE_CASES:
        m, k, n = case[0], case[1], case[2]
        A, B = rule_inputs(case)
        st = oe.np_stats(A, B, True)
        bi = torch.tensor(np.concatenate([st["r"], st["c"], [0]]).astype(np.int32))
        bd = torch.tensor(np.concatenate([st["sA"], st["nA"], st["sB"], st["nB"]]))
        b = {"bi": bi, "bd": bd, "hi": torch.empty_like(bi), "hd": torch.empty_like(bd),
             "r": bi[:m], "c": bi[m:m + n], "flag": bi[m + n:], "sA": bd[:m], "nA": bd[m:2 * m],
             "sB": bd[2 * m:2 * m + n], "nB": bd[2 * m + n:], "dec": torch.zeros(4, dtype=torch.int32),
             "pdev": torch.zeros(1, dtype=torch.int32)}
        At, Bt = torch.from_numpy(A), torch.from_numpy(B)
        rec = {"case": list(case), "A_sha": digest(A), "B_sha": digest(B)}
        for seed in (0, 3):
            N, p, info, _ = oe.OzakiCRT.choose(None, At, Bt, b, tau=2.0 ** -52, force_N=None, seed=seed)
            rec[f"host_seed{seed}"] = {"N": N, "p": p, "p_req": info.get("p_req"), "probe": info.get("probe"),
                                       "worst_ratio_E_over_D": info.get("worst_ratio_E_over_D"),
                                       "nuA": info.get("nuA"), "nuB": info.get("nuB"),
                                       "fallback": bool(info.get("fallback", False))}
        for tau in (2.0 ** -40, 2.0 ** -60):
            N, p, info, _ = oe.OzakiCRT.choose(None, At, Bt, b, tau=tau, force_N=None, seed=0)
            rec[f"host_tau{int(-math.log2(tau))}"] = {"N": N, "p": p, "p_req": info.get("p_req"),
                                                      "fallback": bool(info.get("fallback", False))}
        if m >= 32 and n >= 32:
            dev_self = types.SimpleNamespace(probe={}, Mvec=torch.tensor(
                [float(math.prod(oe.MODS[:N_])) for N_ in range(6, oe.NMAX + 1)], dtype=torch.float64))
            oe.OzakiCRT._rule_device(dev_self, At, Bt, b, 2.0 ** -52, 2.0)
            rec["device_dec"] = b["dec"].tolist()
            oe.OzakiCRT._rule_device(dev_self, At, Bt, b, 2.0 ** -52, 2.0, force_N=16, force_p=40)
            rec["device_dec_forced_16_40"] = b["dec"].tolist()
        rules.append(rec)
        print("rule case", case, rec["host_seed0"], rec.get("device_dec"), flush=True)
    json.dump({"cases": rules}, open(os.path.join(HERE, "rule_golden.json"), "w"), indent=0)

    # ---------------------------------------------------------------- tables
    grid = []
    for N in range(6, 33):
        for (nuA, nuB, k) in ((0.5, 0.5, 64), (3.7, 11.2, 1024), (64.0, 64.0, 4096), (181.02, 90.5, 16384),
                              (1e-3, 2.5, 262144), (0.0, 0.0, 128), (512.0, 512.0, 262144)):
            grid.append([N, nuA, nuB, k, oe.pmax_bits(N, nuA, nuB, k)])
    tab_path = os.path.join(tempfile.mkdtemp(), "config_table.json")
    tab = oe.make_config_table(tab_path, ks=(1024, 2048, 4096, 8192, 16384, 262144))
    picks = []
    for k in (1000, 1024, 4096, 5000, 16384, 262144):
        for sig in (2.0 ** -40, 2.0 ** -50, 2.0 ** -53):
            picks.append([k, sig, oe.pick_config(tab, k, sig)])
    tables = {"pmax_grid": grid, "pow2tab_sha": digest(oe._pow2tab()), "limbs": [oe._limbs_for(N) for N in range(1, 33)],
              "Mfloat": [float(math.prod(oe.MODS[:N])) for N in range(1, 33)], "mods": oe.MODS,
              "config_entries": tab["entries"], "picks": picks,
              "worst_case_p": [[N, k, oe.worst_case_p(N, k)] for N in (6, 12, 16, 20, 32) for k in (1024, 262144)]}
    json.dump(tables, open(os.path.join(HERE, "tables_golden.json"), "w"), indent=0)
    print("tables written", flush=True)


if __name__ == "__main__":
    main()
