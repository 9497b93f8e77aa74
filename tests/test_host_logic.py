"""Host-side logic of the package (no GPU): constants, range bounds, configuration table, probe sets, input
generator, and the C ABI of libozaki_b200.so (it loads without a device and exports every declared symbol)."""
import ctypes
import hashlib
import json
import math
import os
import re

import numpy as np
import pytest

from make_golden import baseline_inputs

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TABLES = json.load(open(os.path.join(HERE, "tables_golden.json")))
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_moduli(pkg):
    assert pkg.MODS == TABLES["mods"]
    assert all(math.gcd(a, b) == 1 for i, a in enumerate(pkg.MODS) for b in pkg.MODS[i + 1:])
    lib = pkg._lib.lib()
    assert [lib.ozk_modulus(t) for t in range(32)] == pkg.MODS
    assert lib.ozk_modulus(32) == 0 and lib.ozk_modulus(-1) == 0


def test_library_tables_match_reference(pkg):
    assert [pkg.limbs_for(N) for N in range(1, 33)] == TABLES["limbs"]
    assert [pkg.modulus_product(N) for N in range(1, 33)] == TABLES["Mfloat"]
    for N, a, b, k, p in TABLES["pmax_grid"]:
        assert pkg.pmax_bits(N, a, b, k) == p
    assert hashlib.sha256(pkg._pow2tab().tobytes()).hexdigest() == TABLES["pow2tab_sha"]
    for N, k, p in TABLES["worst_case_p"]:
        assert pkg.worst_case_p(N, k) == p


def test_config_table_and_pick(pkg):
    tab = pkg.make_config_table(ks=(1024, 2048, 4096, 8192, 16384, 262144))
    assert tab["entries"] == TABLES["config_entries"]
    for k, sig, want in TABLES["picks"]:
        assert pkg.pick_config(tab, k, sig) == want


def test_bound_matrix_formula(pkg):
    r = np.array([3, -2, 0])
    c = np.array([1, 4])
    sA = np.array([2.0, 5.0, 1.5])
    sB = np.array([7.0, 0.25])
    E = pkg.bound_matrix(r, c, sA, sB, 64, 20, np.array([0, 2]), np.array([1]))
    want = 0.5 * 2.0 ** (3 - 20) * 0.25 + 0.5 * 2.0 ** (4 - 20) * 2.0 + 0.25 * 64 * 2.0 ** (3 + 4 - 40)
    assert E[0, 0] == want and E.shape == (2, 1)


def test_input_generator_matches_golden_generator(pkg):
    for (m, k, n, phi, seed, alt) in ((64, 96, 32, 0.5, 0, False), (40, 64, 96, 2.0, 5, True)):
        A, B = pkg.make_inputs(m, k, n, phi, seed, alt)
        A2, B2 = baseline_inputs(m, k, n, phi, seed, alt)
        assert np.array_equal(A, A2) and np.array_equal(B, B2)


def test_input_generator_chunking_is_stream_equivalent(pkg):
    # the chunked fill draws the same stream as one draw
    A, B = pkg.make_inputs(4096 + 7, 4096, 32, 1.0, seed=2)   # > 2^24 / k rows: several chunks
    g = np.random.default_rng(2)
    U = g.random((4096 + 7, 4096))
    Z = g.standard_normal((4096 + 7, 4096))
    assert np.array_equal(A, (U - 0.5) * np.exp(1.0 * Z))


def _declared_functions():
    src = open(os.path.join(ROOT, "include", "ozaki_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ozk_[a-z0-9_]+)\s*\(", src)))


def test_capi_exports_every_declared_symbol(pkg):
    declared = _declared_functions()
    assert len(declared) >= 17
    L = ctypes.CDLL(pkg._lib.LIB_PATH)
    missing = [f for f in declared if not hasattr(L, f)]
    assert not missing, missing
    assert sorted(pkg._lib.exported_names()) == declared


def test_capi_host_calls_without_device(pkg):
    lib = pkg._lib.lib()
    assert lib.ozk_version() >= 100
    assert pkg._lib.error_string(0) == "ok"
    assert "invalid argument" in pkg._lib.error_string(-1)
    assert lib.ozk_stats_workspace_bytes(64, 64, 64) > 0
    assert lib.ozk_stats_workspace_bytes(0, 64, 64) == 0
    # argument validation happens before any device work: null pointers are rejected with OZK_ERR_ARG
    assert lib.ozk_split_a(None, None, None, None, 4, 32, 16, None, None, None) == -1
    assert lib.ozk_gemm_residues(None, None, 4, 32, 32, 16, None, None, None) == -1
    assert lib.ozk_reconstruct(None, None, None, None, 4, 32, 16, None, None, None) == -1
    assert lib.ozk_wait_selftest(0, 10**6, None, None, None) == -1
    assert lib.ozk_wait_selftest(2, 10**6, 16, 16, None) == -1           # role outside {0, 1}
    assert lib.ozk_wait_selftest(0, 999, 16, 16, None) == -1             # limit below 1 us
    assert lib.ozk_wait_selftest(1, 5 * 10**9, 16, 16, None) == -1       # limit above the GEMM's 4 s
    assert lib.ozk_wait_selftest(0, 10**6, 16, 20, None) == -1           # waited_ns not 8-byte aligned
    with pytest.raises(pkg._lib.OzkError):
        pkg._lib.check(-5, "probe")


def test_oracle_probe_sets_follow_reference(oracle):
    # RandomState(seed).choice without replacement, rows then columns
    Ir, Jr = oracle.probe_random(300, 200, seed=0)
    rs = np.random.RandomState(0)
    assert np.array_equal(Ir, rs.choice(300, 64, replace=False))
    assert np.array_equal(Jr, rs.choice(200, 64, replace=False))
    Ir, Jr = oracle.probe_random(40, 32, seed=1)
    assert len(Ir) == 40 and len(Jr) == 32


def test_correctly_rounded_products_are_exact(pkg):
    """The accuracy sample's reference values (Dekker products + fsum) equal the exact rational dot product rounded
    once, including a cancelling case."""
    from fractions import Fraction
    A, B = pkg.make_inputs(6, 200, 5, 2.0, seed=13)
    B[:, 4] = A[0] * 3.0                       # column 4: row 0's dot product has no cancellation...
    A[1] = -A[0]                               # ...and row 1's is its exact negative
    got = pkg.correctly_rounded_products(A, B)
    for i in range(A.shape[0]):
        for j in range(B.shape[1]):
            exact = sum(Fraction(float(a)) * Fraction(float(b)) for a, b in zip(A[i], B[:, j]))
            assert got[i, j] == float(exact), (i, j)
    assert got[1, 4] == -got[0, 4]
