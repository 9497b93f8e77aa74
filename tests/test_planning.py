"""Planning helpers (coprime_ip, int8_crt, the residue-chain cost model) against the reference's own outputs
(tests/golden/planning_golden.json, made by tests/golden/make_planning_golden.py from code/digit_gemm.py)."""
import json
import math
import os

import pytest

GOLD = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "planning_golden.json")))


@pytest.fixture(scope="module")
def planning(pkg):
    import importlib
    return importlib.import_module(pkg.__name__ + ".planning")


@pytest.mark.parametrize("case", GOLD["int8_crt"], ids=lambda c: f"b{c['b']}_k{c['k']}")
def test_int8_crt(planning, case):
    mods, n = planning.int8_crt(case["b"], case["k"])
    assert (mods, n) == (case["mods"], case["n"])
    assert math.prod(mods) > 2 * case["k"] * (2 ** case["b"] - 1) ** 2
    assert all(math.gcd(a, b) == 1 for i, a in enumerate(mods) for b in mods[i + 1:])


@pytest.mark.parametrize("case", GOLD["coprime_ip"], ids=lambda c: f"t{c['target']}")
def test_coprime_ip(planning, case):
    cands = [tuple(c) for c in case["cands"]]
    assert planning.coprime_ip(cands, case["target"]) == (case["mods"], case["cost"])


def test_chain_cost_model(planning):
    assert planning.chain_cost_model() == GOLD["chain"]
