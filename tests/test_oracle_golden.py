"""The CPU oracle (oracle/) against golden vectors produced by the reference itself (tests/golden/make_golden.py):
np_stats, expected_core (bit-exact CRT results), pmax_bits, choose and _rule_device of dl1683/matrix-numbers
code/ozaki_engine.py.  CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest

from make_golden import RULE_CASES, rule_inputs, selftest_inputs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SELF = json.load(open(os.path.join(HERE, "selftest_golden.json")))
RULE = json.load(open(os.path.join(HERE, "rule_golden.json")))
TABLES = json.load(open(os.path.join(HERE, "tables_golden.json")))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_golden_fixture_matches_shipped_selftest():
    # the (N, p) pairs regenerated from the reference equal the ones in its shipped results/engine/selftest.json
    assert SELF["np_pairs_match_shipped_selftest"]


@pytest.mark.parametrize("ci", range(6))
def test_inputs_regenerate(ci):
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    rec = SELF["cases"][ci]
    assert [m, k, n] == rec["shape"] and kind == rec["kind"]
    assert sha(A) == rec["A_sha"] and sha(B) == rec["B_sha"]


@pytest.mark.parametrize("ci", range(6))
def test_stats_vs_np_stats(oracle, ci):
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    rec = SELF["cases"][ci]["stats"]
    st = oracle.stats(A, B, True)
    for x in ("gam", "r", "c"):
        assert np.array_equal(st[x], np.array(rec[x])), x
    for x in ("sA", "sB", "nA", "nB"):
        np.testing.assert_allclose(st[x], np.array(rec[x]), rtol=1e-13, atol=0)
    assert st["flag"] == 0


@pytest.mark.parametrize("ci", range(6))
def test_core_bit_exact_vs_expected_core(oracle, ci):
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    rec = SELF["cases"][ci]
    st = oracle.stats(A, B, True)
    full = np.load(os.path.join(HERE, "selftest_golden.npz"))
    for c in rec["cores"]:
        C = oracle.core(A, B, st, c["N"], c["p"])
        key = f"C_{ci}_N{c['N']}_p{c['p']}"
        if key in full:
            np.testing.assert_array_equal(C.view(np.uint64), full[key].view(np.uint64))
        assert sha(C) == c["sha"], (kind, c)


def test_pmax_table(oracle):
    for N, a, b, k, p in TABLES["pmax_grid"]:
        assert oracle.pmax_bits(N, a, b, k) == p, (N, a, b, k)
    assert [oracle.limbs_for(N) for N in range(1, 33)] == TABLES["limbs"]
    assert [oracle.modulus_product(N) for N in range(1, 33)] == TABLES["Mfloat"]


@pytest.mark.parametrize("ci", range(len(RULE_CASES)))
def test_host_rule_vs_reference_choose(oracle, ci):
    case = RULE_CASES[ci]
    rec = RULE["cases"][ci]
    m, k, n = case[:3]
    A, B = rule_inputs(case)
    assert sha(A) == rec["A_sha"] and sha(B) == rec["B_sha"]
    st = oracle.stats(A, B, True)
    for seed in (0, 3):
        I, J = oracle.probe_sets(st, m, n, k, seed)
        D = oracle.probe_D(A, B, I, J)
        got = oracle.rule(st, m, n, k, I, J, D)
        ref = rec[f"host_seed{seed}"]
        assert (got["N"], got["p"], got["p_req"], [len(I), len(J)]) == (ref["N"], ref["p"], ref["p_req"], ref["probe"])
        assert got["worst_ratio_E_over_D"] == pytest.approx(ref["worst_ratio_E_over_D"], rel=1e-12)
        assert got["nuA"] == pytest.approx(ref["nuA"], rel=1e-14) and got["nuB"] == pytest.approx(ref["nuB"], rel=1e-14)
    for tau in (40, 60):
        I, J = oracle.probe_sets(st, m, n, k, 0)
        got = oracle.rule(st, m, n, k, I, J, oracle.probe_D(A, B, I, J), tau=2.0 ** -tau)
        ref = rec[f"host_tau{tau}"]
        assert (got["N"], got["p"], got["p_req"], got["fallback"]) == (ref["N"], ref["p"], ref["p_req"], ref["fallback"])
    if "device_dec" in rec:
        # the reference's device rule agrees with its host rule on these inputs
        I, J = oracle.probe_sets(st, m, n, k, 0)
        got = oracle.rule(st, m, n, k, I, J, oracle.probe_D(A, B, I, J))
        assert rec["device_dec"] == [got["N"], got["p"], 0, got["p_req"]]


def test_forced_rule_matches_reference_device_rule(oracle):
    for ci, case in enumerate(RULE_CASES):
        rec = RULE["cases"][ci]
        if "device_dec_forced_16_40" not in rec:
            continue
        m, k, n = case[:3]
        A, B = rule_inputs(case)
        st = oracle.stats(A, B, True)
        got = oracle.rule(st, m, n, k, [], [], np.zeros((0, 0)), force_N=16)
        pv = got["p"]
        fb = int(pv < 40)
        assert rec["device_dec_forced_16_40"] == [0 if fb else 16, min(pv, 40), fb, 0]


def test_exact_sample_is_correctly_rounded(oracle):
    rng = np.random.default_rng(3)
    A = rng.standard_normal((3, 200)) * np.exp2(rng.integers(-30, 30, (3, 200)))
    B = rng.standard_normal((200, 4))
    from fractions import Fraction
    S = oracle.exact_sample(A, B)
    for i in range(3):
        for j in range(4):
            exact = sum(Fraction(float(a)) * Fraction(float(b)) for a, b in zip(A[i], B[:, j]))
            assert S[i, j] == float(exact)
