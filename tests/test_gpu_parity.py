"""Parity of every stage of libozaki_b200.so (through its C ABI) with the CPU oracle, and of the drop-in entry point
with the reference's golden results.  Integer work (statistics exponents, residue planes, per-modulus products,
plane count, p, p_req) must be bit-exact; the reconstructed C is bit-exact too (exact CRT + the reference's
rounding).  Floating-point sums of the statistics are compared with rtol 1e-13 (summation order differs)."""
import hashlib
import json
import os

import numpy as np
import pytest

from make_golden import RULE_CASES, rule_inputs, selftest_inputs

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
SELF = json.load(open(os.path.join(HERE, "selftest_golden.json")))
RULE = json.load(open(os.path.join(HERE, "rule_golden.json")))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def torch_mod():
    import torch
    return torch


def T(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def dev_stats(pkg, torch, A, B, inside=True):
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    m, k = A.shape
    n = B.shape[1]
    out = {"gam": torch.empty(k, dtype=torch.int32, device="cuda"), "r": torch.empty(m, dtype=torch.int32, device="cuda"),
           "c": torch.empty(n + 3, dtype=torch.int32, device="cuda")[:n],
           "sA": torch.empty(m, dtype=torch.float64, device="cuda"), "nA": torch.empty(m, dtype=torch.float64, device="cuda"),
           "sB": torch.empty(n, dtype=torch.float64, device="cuda"), "nB": torch.empty(n, dtype=torch.float64, device="cuda"),
           "flag": torch.empty(1, dtype=torch.int32, device="cuda")}
    ws = torch.empty(L.ozk_stats_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    rc = L.ozk_stats(ptr(A), ptr(B), m, n, k, int(inside), *(ptr(out[x]) for x in ("gam", "r", "c", "sA", "nA", "sB", "nB", "flag")),
                     ptr(ws), ws.numel(), torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(rc, "ozk_stats")
    torch.cuda.synchronize()
    return out


def host(d):
    return {k: v.cpu().numpy() for k, v in d.items()}


def assert_stats_equal(got, ref, rtol=1e-13):
    for x in ("gam", "r", "c"):
        assert np.array_equal(got[x], ref[x]), x
    for x in ("sA", "sB", "nA", "nB"):
        np.testing.assert_allclose(got[x], ref[x], rtol=rtol, atol=0, err_msg=x)
    assert int(got["flag"][0]) == int(ref["flag"])


# ------------------------------------------------------------------------------------------------ statistics
@pytest.mark.parametrize("ci", range(6))
def test_stats_selftest_cases(pkg, oracle, torch_mod, ci):
    torch = torch_mod
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    got = host(dev_stats(pkg, torch, T(torch, A), T(torch, B)))
    assert_stats_equal(got, oracle.stats(A, B, True))
    rec = SELF["cases"][ci]["stats"]
    for x in ("gam", "r", "c"):
        assert np.array_equal(got[x], np.array(rec[x]))


@pytest.mark.parametrize("shape,phi,inside", [((256, 1024, 512), 2.0, True), ((96, 4096, 160), 0.5, True),
                                              ((128, 640, 64), 1.0, False)])
def test_stats_random(pkg, oracle, torch_mod, shape, phi, inside):
    torch = torch_mod
    m, k, n = shape
    A, B = pkg.make_inputs(m, k, n, phi, seed=21)
    A[3, :] = 0.0          # an all-zero row and column
    B[:, 5] = 0.0
    got = host(dev_stats(pkg, torch, T(torch, A), T(torch, B), inside))
    assert_stats_equal(got, oracle.stats(A, B, inside))


def test_stats_extreme_exponents(pkg, oracle, torch_mod):
    """Entries across the whole double range: subnormal rows and columns, 2^-1070 next to 2^1014 in one row, zeros.
    The scaled values |x| 2^gamma then leave the normal range, so the statistics' general path runs beside the fast
    one (csrc/stats.cu, RunStats.add_abs); both must agree with the oracle, with inside scaling on and off."""
    torch = torch_mod
    rng = np.random.default_rng(7)
    m, k, n = 64, 256, 96

    def mat(r, c):
        x = rng.uniform(1.0, 2.0, (r, c)) * np.ldexp(1.0, rng.integers(-1070, 1015, (r, c)))
        x *= rng.choice([-1.0, 1.0], (r, c))
        x[rng.random((r, c)) < 0.1] = 0.0
        return x

    A, B = mat(m, k), mat(k, n)
    A[0] = np.ldexp(rng.uniform(1.0, 2.0, k), rng.integers(-1074, -1023, k))     # subnormal row
    A[1] = np.ldexp(rng.uniform(1.0, 2.0, k), rng.integers(990, 1020, k))        # huge row
    A[2] = 0.0
    B[:, 0] = np.ldexp(rng.uniform(1.0, 2.0, k), rng.integers(-1074, -1023, k))  # subnormal column
    B[:, 1] = -np.ldexp(rng.uniform(1.0, 2.0, k), rng.integers(990, 1020, k))    # huge column
    A[:, 3] = np.ldexp(rng.uniform(1.0, 2.0, m), rng.integers(-1074, -1060, m))  # gamma_3 above 1023
    B[3, :] = np.ldexp(rng.uniform(1.0, 2.0, n), rng.integers(1005, 1015, n))
    assert np.all(np.isfinite(A)) and np.all(np.isfinite(B))
    for inside in (True, False):
        got = host(dev_stats(pkg, torch, T(torch, A), T(torch, B), inside))
        assert_stats_equal(got, oracle.stats(A, B, inside))


def test_stats_nonfinite_flag(pkg, torch_mod):
    torch = torch_mod
    A, B = pkg.make_inputs(64, 64, 64, 1.0, seed=1)
    B[7, 9] = np.inf
    got = host(dev_stats(pkg, torch, T(torch, A), T(torch, B)))
    assert int(got["flag"][0]) == 1
    A[1, 1] = np.nan
    B[7, 9] = 1.0
    assert int(host(dev_stats(pkg, torch, T(torch, A), T(torch, B)))["flag"][0]) == 1


def test_stats_reproducible(pkg, torch_mod):
    torch = torch_mod
    A, B = pkg.make_inputs(512, 2048, 512, 2.0, seed=4)
    Ad, Bd = T(torch, A), T(torch, B)
    s1, s2 = host(dev_stats(pkg, torch, Ad, Bd)), host(dev_stats(pkg, torch, Ad, Bd))
    for x in s1:
        assert np.array_equal(s1[x], s2[x]), x


# ------------------------------------------------------------------------------------------------ the rule
def dev_rule(pkg, torch, A, B, st, Ir, Jr, tau=2.0 ** -52, safety=2.0, force_N=0, force_p=-1):
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    m, k = A.shape
    n = B.shape[1]
    ctl = torch.zeros(8, dtype=torch.int32, device="cuda")
    aux = torch.zeros(8, dtype=torch.float64, device="cuda")
    ws = torch.empty(L.ozk_rule_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    Irt = torch.as_tensor(np.asarray(Ir, dtype=np.int64), device="cuda")
    Jrt = torch.as_tensor(np.asarray(Jr, dtype=np.int64), device="cuda")
    rc = L.ozk_rule(ptr(A), ptr(B), m, n, k, ptr(st["r"]), ptr(st["c"]), ptr(st["sA"]), ptr(st["nA"]), ptr(st["sB"]),
                    ptr(st["nB"]), ptr(st["flag"]), ptr(Irt), len(Ir), ptr(Jrt), len(Jr), tau, safety, force_N, force_p,
                    ptr(ctl[0:4]), ptr(ctl[5:6]), ptr(aux), ptr(ws), ws.numel(), torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(rc, "ozk_rule")
    torch.cuda.synchronize()
    c = ctl.cpu().tolist()
    return {"N": c[0] or None, "p": c[1], "fallback": bool(c[2]), "p_req": c[3], "pdev": c[5]}, aux.cpu().tolist()


@pytest.mark.parametrize("ci", range(len(RULE_CASES)))
def test_rule_vs_oracle_and_reference(pkg, oracle, torch_mod, ci):
    torch = torch_mod
    case = RULE_CASES[ci]
    m, k, n = case[:3]
    A, B = rule_inputs(case)
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    for seed in (0, 3):
        Ir, Jr = oracle.probe_random(m, n, seed)
        got, aux = dev_rule(pkg, torch, Ad, Bd, st, Ir, Jr)
        I, J = oracle.probe_sets(sto, m, n, k, seed)
        want = oracle.rule(sto, m, n, k, I, J, oracle.probe_D(A, B, I, J))
        assert (got["N"], got["p"], got["p_req"], got["fallback"]) == (want["N"], want["p"], want["p_req"], want["fallback"])
        assert got["pdev"] == got["p"]
        assert [int(aux[3]), int(aux[4])] == [len(I), len(J)]
        assert aux[0] == pytest.approx(want["nuA"], rel=1e-14) and aux[1] == pytest.approx(want["nuB"], rel=1e-14)
        assert aux[2] == pytest.approx(want["worst_ratio_E_over_D"], rel=1e-12)
        ref = RULE["cases"][ci][f"host_seed{seed}"]       # the reference's own choose()
        assert (got["N"], got["p"], got["p_req"]) == (ref["N"], ref["p"], ref["p_req"])
    for tau in (40, 60):
        Ir, Jr = oracle.probe_random(m, n, 0)
        got, _ = dev_rule(pkg, torch, Ad, Bd, st, Ir, Jr, tau=2.0 ** -tau)
        ref = RULE["cases"][ci][f"host_tau{tau}"]
        assert (got["N"], got["p"], got["p_req"], got["fallback"]) == (ref["N"], ref["p"], ref["p_req"], ref["fallback"])


def test_rule_forced_and_nonfinite(pkg, oracle, torch_mod):
    torch = torch_mod
    A, B = rule_inputs(RULE_CASES[0])
    m, k, n = RULE_CASES[0][:3]
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    pv = oracle.rule(oracle.stats(A, B), m, n, k, [], [], np.zeros((0, 0)), force_N=16)["p"]
    got, _ = dev_rule(pkg, torch, Ad, Bd, st, [], [], force_N=16)
    assert (got["N"], got["p"], got["fallback"]) == (16, pv, False)
    got, _ = dev_rule(pkg, torch, Ad, Bd, st, [], [], force_N=16, force_p=40)
    assert (got["N"], got["p"], got["fallback"]) == (16, 40, False)
    got, _ = dev_rule(pkg, torch, Ad, Bd, st, [], [], force_N=16, force_p=pv + 1)
    assert (got["N"], got["p"], got["fallback"]) == (None, pv, True)
    assert RULE["cases"][0]["device_dec_forced_16_40"] == [16, 40, 0, 0]
    B2 = B.copy()
    B2[0, 0] = np.inf
    B2d = T(torch, B2)
    st2 = dev_stats(pkg, torch, Ad, B2d)
    Ir, Jr = oracle.probe_random(m, n, 0)
    got, _ = dev_rule(pkg, torch, Ad, B2d, st2, Ir, Jr)
    assert got["fallback"] and got["N"] is None


# ------------------------------------------------------------------------------------------------ residue split
def dev_split(pkg, torch, A, B, st, p, N):
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    m, k = A.shape
    n = B.shape[1]
    pd = torch.tensor([p], dtype=torch.int32, device="cuda")
    Ar = torch.empty((N, m, k), dtype=torch.int8, device="cuda")
    Br = torch.empty((N, n, k), dtype=torch.int8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    pkg._lib.check(L.ozk_split_a(ptr(A), ptr(st["r"]), ptr(st["gam"]), ptr(pd), m, k, N, ptr(Ar), ptr(err), s),
                   "split_a")
    pkg._lib.check(L.ozk_split_b(ptr(B), ptr(st["c"]), ptr(st["gam"]), ptr(pd), k, n, N, ptr(Br), ptr(err), s),
                   "split_b")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return Ar.cpu().numpy(), Br.cpu().numpy()


@pytest.mark.parametrize("ci", range(6))
def test_split_selftest_cases(pkg, oracle, torch_mod, ci):
    torch = torch_mod
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    for c in SELF["cases"][ci]["cores"]:
        N, p = c["N"], c["p"]
        Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, N)
        assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, N)), (N, p)
        assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, N)), (N, p)


@pytest.mark.parametrize("p", [6, 31, 58, 69, 80, 99, 121, 159])
def test_split_all_digit_widths(pkg, oracle, torch_mod, p):
    torch = torch_mod
    A, B = pkg.make_inputs(64, 256, 96, 2.0, seed=p)
    A[0, :4] = [5e-324, -5e-324 * 7, 2.0 ** -1070, -1.0]     # subnormals and exact powers of two
    A[1, :] = 0.0
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, 32)
    assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, 32))
    assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, 32))


# ragged work division: row-block counts that leave a partial task, fewer l-blocks than chunks per task, every
# plane-count boundary of the 16-modulus row tiles, both byte-string widths
@pytest.mark.parametrize("m,k,n,N,p", [(12, 96, 32, 6, 40), (20, 64, 64, 8, 58), (36, 32, 96, 9, 60),
                                       (12, 160, 32, 16, 70), (44, 96, 32, 17, 67), (8, 224, 64, 24, 90),
                                       (28, 96, 32, 25, 119), (12, 96, 64, 20, 120), (16, 32, 32, 31, 150),
                                       (24, 64, 32, 3, 50), (16, 96, 64, 1, 45), (40, 160, 96, 13, 104)])
def test_split_ragged(pkg, oracle, torch_mod, m, k, n, N, p):
    torch = torch_mod
    A, B = pkg.make_inputs(m, k, n, 1.5, seed=m + k + N)
    A[0, 0], B[1, 0] = -0.0, -3e-320
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, N)
    assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, N))
    assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, N))


# moduli 16 .. N-1 for 16 < N <= 20 come from the packed tail (8 chunks x 2 moduli or 4 chunks x 4 moduli per MMA
# row tile): every N around it, a last A task with fewer than 8 chunks, one and several l-blocks per B column group
@pytest.mark.parametrize("m,k,n,N", [(52, 96, 64, 17), (20, 32, 96, 18), (36, 160, 32, 19), (12, 224, 64, 20),
                                     (28, 96, 32, 21), (1028, 128, 160, 18), (44, 64, 288, 20)])
def test_split_packed_tail(pkg, oracle, torch_mod, m, k, n, N):
    torch = torch_mod
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=3 * m + N)
    A[0, 1], B[2, 0] = -5e-324, -0.0
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    for p in (58, 67, 119):
        Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, N)
        assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, N)), p
        assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, N)), p


# many tiles per CTA of the tensor-core split (its load ring and both string buffers wrap around several times),
# narrow and wide digit ranges (p <= 100 and 101 <= p <= 119)
@pytest.mark.parametrize("N,p", [(18, 67), (20, 110), (16, 58)])
def test_split_many_tiles(pkg, oracle, torch_mod, N, p):
    torch = torch_mod
    m, k, n = 2048, 1536, 1024
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=N + p)
    A[5, 7], B[9, 3] = -0.0, 4e-310
    Ad, Bd = T(torch, A), T(torch, B)
    st = dev_stats(pkg, torch, Ad, Bd)
    sto = oracle.stats(A, B, True)
    Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, N)
    assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, N))
    assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, N))


# B 8 bytes off a 16-byte boundary: ozk_split_b keeps the general kernel for it (the tensor-core split loads B by TMA,
# which needs a 16-byte aligned base), A still takes the tensor-core path; both bit-exact
def test_split_unaligned_B_uses_general_kernel(pkg, oracle, torch_mod):
    torch = torch_mod
    m, k, n, N, p = 96, 256, 64, 18, 67
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=5)
    Ad = T(torch, A)
    store = torch.empty(k * n + 1, dtype=torch.float64, device="cuda")
    Bd = store[1:].view(k, n)
    Bd.copy_(T(torch, B))
    assert Bd.data_ptr() % 16 == 8
    st = dev_stats(pkg, torch, Ad, T(torch, B))             # the statistics entry points want aligned operands
    sto = oracle.stats(A, B, True)
    Ar, Br = dev_split(pkg, torch, Ad, Bd, st, p, N)
    assert np.array_equal(Ar, oracle.split_A(A, sto["r"], sto["gam"], p, N))
    assert np.array_equal(Br, oracle.split_B(B, sto["c"], sto["gam"], p, N))


# ------------------------------------------------------------------------------------------------ INT8 products
def rand_planes(rng, N, rows, k):
    return rng.integers(-128, 128, size=(N, rows, k), dtype=np.int64).astype(np.int8)


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (132, 288, 96), (256, 512, 1024), (4, 32, 32), (384, 96, 2080)])
def test_gemm_i32_exact(pkg, oracle, torch_mod, m, n, k):
    torch = torch_mod
    rng = np.random.default_rng(m * 7 + n + k)
    At = rand_planes(rng, 1, m, k)[0]
    Bt = rand_planes(rng, 1, n, k)[0]
    At[0, :] = -128
    Bt[0, :] = -128                # the largest product magnitude
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    Ad, Bd = T(torch, At), T(torch, Bt)
    C = torch.empty((m, n), dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg._lib.check(L.ozk_gemm_i32(ptr(Ad), ptr(Bd), m, n, k, ptr(C), ptr(err), torch.cuda.current_stream().cuda_stream), "gemm_i32")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(C.cpu().numpy(), oracle.gemm_i32(At, Bt))
    # the same product through torch's INT8 GEMM (the reference checks cuBLASLt against torch._int_mm)
    if m > 16 and k <= 65536:
        ref = torch._int_mm(Ad, Bd.t())
        assert torch.equal(C, ref)


@pytest.mark.parametrize("m,n,k,N", [(256, 256, 256, 20), (132, 160, 288, 32), (512, 768, 640, 16), (8, 64, 64, 6),
                                     (640, 1280, 512, 18), (1152, 256, 384, 3)])
def test_gemm_residues_exact(pkg, oracle, torch_mod, m, n, k, N):
    torch = torch_mod
    rng = np.random.default_rng(m + 3 * n + 5 * k + N)
    Ar = rand_planes(rng, N, m, k)
    Br = rand_planes(rng, N, n, k)
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    Ad, Bd = T(torch, Ar), T(torch, Br)
    X = torch.empty((N, m, n), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg._lib.check(L.ozk_gemm_residues(ptr(Ad), ptr(Bd), m, n, k, N, ptr(X), ptr(err), torch.cuda.current_stream().cuda_stream), "gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(X.cpu().numpy(), oracle.gemm_mod(Ar, Br))


@pytest.mark.parametrize("k", [65536 + 4096, 3 * 65536 + 160])
def test_gemm_residues_k_segments(pkg, oracle, torch_mod, k):
    """Contraction longer than one exact INT32 segment (65536): residues of the exact int64 product."""
    torch = torch_mod
    m, n, N = 64, 64, 3
    rng = np.random.default_rng(k)
    Ar = rand_planes(rng, N, m, k)
    Br = rand_planes(rng, N, n, k)
    Ar[:, 0, :] = -128
    Br[:, 0, :] = -128             # the first entry needs more than 31 bits
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    Ad, Bd = T(torch, Ar), T(torch, Br)
    X = torch.empty((N, m, n), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    pkg._lib.check(L.ozk_gemm_residues(ptr(Ad), ptr(Bd), m, n, k, N, ptr(X), ptr(err), torch.cuda.current_stream().cuda_stream), "gemm")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(X.cpu().numpy(), oracle.gemm_mod(Ar, Br))


# ------------------------------------------------------------------------------------------------ reconstruction
@pytest.mark.parametrize("N,n", [(N, 256) for N in range(1, 33)] + [(N, 36) for N in (6, 16, 19, 32)])
def test_reconstruct_random_residues(pkg, oracle, torch_mod, N, n):
    """Uniform random residues: every CRT value in [0, M) occurs, including |X| close to M/2; every plane count, and
    rows that are not a multiple of the 4-element vectors' 32-byte sectors (n = 36)."""
    torch = torch_mod
    m = 64
    rng = np.random.default_rng(N)
    X = np.stack([rng.integers(0, pkg.MODS[t], size=(m, n)) for t in range(N)]).astype(np.uint8)
    r = rng.integers(-40, 40, size=m).astype(np.int32)
    c = rng.integers(-40, 40, size=n).astype(np.int32)
    for p in (1, 60, 200):
        L = pkg._lib.lib()
        ptr = pkg._lib.ptr
        Xd, rd, cd = T(torch, X), T(torch, r), T(torch, c)
        pd = torch.tensor([p], dtype=torch.int32, device="cuda")
        C = torch.empty((m, n), dtype=torch.float64, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        pkg._lib.check(L.ozk_reconstruct(ptr(Xd), ptr(rd), ptr(cd), ptr(pd), m, n, N, ptr(C), ptr(err),
                                         torch.cuda.current_stream().cuda_stream), "recon")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        want = oracle.recon(X, r, c, p)
        np.testing.assert_array_equal(C.cpu().numpy().view(np.uint64), want.view(np.uint64))


def test_reconstruct_extreme_exponents(pkg, oracle, torch_mod):
    torch = torch_mod
    m, n, N = 8, 64, 16
    rng = np.random.default_rng(9)
    X = np.stack([rng.integers(0, pkg.MODS[t], size=(m, n)) for t in range(N)]).astype(np.uint8)
    X[:, 0, :] = 0                                   # zero
    X[:, 1, :5] = 1                                  # +1 in every modulus
    for t in range(N):
        X[t, 2, :5] = pkg.MODS[t] - 1                # -1
    for r0, c0, p in ((-1000, -60, 30), (900, 200, 10), (-600, -500, 0)):   # subnormal, overflow, deep underflow
        r = np.full(m, r0, np.int32)
        c = np.full(n, c0, np.int32)
        L = pkg._lib.lib()
        ptr = pkg._lib.ptr
        Xd, rd, cd = T(torch, X), T(torch, r), T(torch, c)
        pd = torch.tensor([p], dtype=torch.int32, device="cuda")
        C = torch.empty((m, n), dtype=torch.float64, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        pkg._lib.check(L.ozk_reconstruct(ptr(Xd), ptr(rd), ptr(cd), ptr(pd), m, n, N, ptr(C), ptr(err),
                                         torch.cuda.current_stream().cuda_stream), "recon")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        np.testing.assert_array_equal(C.cpu().numpy().view(np.uint64), oracle.recon(X, r, c, p).view(np.uint64))


# ------------------------------------------------------------------------------------------------ end to end
@pytest.mark.parametrize("ci", range(6))
def test_core_matches_reference_expected_core(pkg, engine, torch_mod, ci):
    """The reference's selftest (ozaki_engine.py:1682-1738): stats on the device, (N, p) forced, core -> C must equal
    the Python big-integer expected_core bit for bit (48 cases)."""
    torch = torch_mod
    (m, k, n), kind, A, B = selftest_inputs()[ci]
    Ad, Bd = T(torch, A), T(torch, B)
    b = engine.buffers(m, n, k, 32)
    engine.stats(Ad, Bd, b, True)
    full = np.load(os.path.join(HERE, "selftest_golden.npz"))
    for c in SELF["cases"][ci]["cores"]:
        b["pdev"].fill_(c["p"])
        C = torch.empty((m, n), dtype=torch.float64, device="cuda")
        engine.core(Ad, Bd, b, c["N"], C)
        torch.cuda.synchronize()
        got = C.cpu().numpy()
        key = f"C_{ci}_N{c['N']}_p{c['p']}"
        if key in full:
            np.testing.assert_array_equal(got.view(np.uint64), full[key].view(np.uint64))
        assert sha(got) == c["sha"], (kind, c["N"], c["p"])
    engine.check_errors()


@pytest.mark.parametrize("shape,phi,seed", [((128, 256, 128), 0.5, 0), ((96, 512, 160), 2.0, 1), ((256, 1024, 256), 1.0, 2),
                                            ((64, 96, 32), 2.0, 3)])
def test_run_matches_oracle(pkg, oracle, engine, torch_mod, shape, phi, seed):
    torch = torch_mod
    m, k, n = shape
    A, B = pkg.make_inputs(m, k, n, phi, seed)
    Ad, Bd = T(torch, A), T(torch, B)
    C, info = engine.run(Ad, Bd)
    Cref, iref = oracle.run(A, B)
    assert (info["N"], info["p"], info["p_req"], info["probe"]) == (iref["N"], iref["p"], iref["p_req"], iref["probe"])
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint64), Cref.view(np.uint64))
    # graph path: same plane count and bit-identical C
    Cg = torch.empty_like(C)
    engine.run(Ad, Bd, C=Cg, graph=True)
    _, ig = engine.run(Ad, Bd, C=Cg, graph=True)
    torch.cuda.synchronize()
    assert (ig["N"], ig["p"]) == (info["N"], info["p"])
    assert torch.equal(C, Cg)
    engine.check_errors()


def test_run_inside_off_and_forced(pkg, oracle, engine, torch_mod):
    torch = torch_mod
    A, B = pkg.make_inputs(128, 384, 96, 2.0, seed=5)
    Ad, Bd = T(torch, A), T(torch, B)
    C, info = engine.run(Ad, Bd, inside=False)
    Cref, iref = oracle.run(A, B, inside=False)
    assert (info["N"], info["p"]) == (iref["N"], iref["p"])
    np.testing.assert_array_equal(C.cpu().numpy(), Cref)
    C, info = engine.run(Ad, Bd, force_N=24)
    Cref, iref = oracle.run(A, B, force_N=24)
    assert (info["N"], info["p"]) == (24, iref["p"])
    np.testing.assert_array_equal(C.cpu().numpy(), Cref)
    # a configuration from the data-independent table
    tab = pkg.make_config_table()
    cfg = pkg.pick_config(tab, 384, 2.0 ** -50)
    C, info = engine.run(Ad, Bd, config=cfg)
    assert not info.get("fallback") and info["N"] == cfg["N"] and info["p"] == cfg["p"]
    Cref, _ = oracle.run(A, B, force_N=cfg["N"], force_p=cfg["p"])
    np.testing.assert_array_equal(C.cpu().numpy(), Cref)
    # an unsafe forced p is rejected with a native fallback
    C, info = engine.run(Ad, Bd, force_N=8, force_p=200)
    assert info.get("fallback") and info.get("config_rejected")
    np.testing.assert_allclose(C.cpu().numpy(), A @ B, rtol=1e-12, atol=1e-300)


def test_nonfinite_falls_back(pkg, engine, torch_mod):
    torch = torch_mod
    A, B = pkg.make_inputs(64, 64, 64, 1.0, seed=8)
    A[3, 3] = np.nan
    Ad, Bd = T(torch, A), T(torch, B)
    C, info = engine.run(Ad, Bd)
    assert info["fallback"] and info["nonfinite"]
    Cg, ig = engine.run(Ad, Bd, C=torch.empty_like(C), graph=True)
    assert ig["fallback"]


def test_integer_inputs_are_exact(pkg, engine, torch_mod):
    """Size-independent property: small-integer matrices have an exactly representable product, which the engine
    must return exactly."""
    torch = torch_mod
    rng = np.random.default_rng(17)
    m, k, n = 512, 2048, 384
    A = rng.integers(-1000, 1000, size=(m, k)).astype(np.float64)
    B = rng.integers(-1000, 1000, size=(k, n)).astype(np.float64)
    C, info = engine.run(T(torch, A), T(torch, B))
    exact = (A.astype(np.int64) @ B.astype(np.int64)).astype(np.float64)
    assert np.array_equal(C.cpu().numpy(), exact)


def test_accuracy_lemma_L1_and_native(pkg, engine, torch_mod):
    """n = 2048, phi = 2: sampled errors against the correctly rounded product; no Lemma L1 violation and no worse
    than native FP64 DGEMM."""
    torch = torch_mod
    A, B = pkg.make_inputs(2048, 2048, 2048, 2.0, seed=0)
    Ad, Bd = T(torch, A), T(torch, B)
    Cn = Ad @ Bd
    S = pkg.Sample(Ad, Bd, Cn)
    C, info = engine.run(Ad, Bd)
    e, en = S.errors(C), S.errors(Cn)
    assert e["E1"] <= en["E1"] and e["E2"] <= en["E2"], (e, en)
    assert e["E2"] <= 2.0 ** -52
    h, p = info["stats"], info["p"]
    Eb = pkg.bound_matrix(h["r"], h["c"], h["sA"], h["sB"], 2048, p, S.ri, S.ci)
    Cs = C[S.tri][:, S.tci].cpu().numpy()
    err = np.abs(Cs - S.ref)
    lim = Eb * (1 + 1e-9) + 2.0 ** -53 * (np.abs(Cs) + np.abs(S.ref)) * (1 + 1e-9)
    assert int((err > lim).sum()) == 0


# the hard-row / hard-column selection of the rule (top 32 of 2^r k / s, stable: larger first, then lower index),
# read back from the rule workspace (RuleCtl: done, nI, nJ, pad, pv[33], nuA, nuB, I[96] at byte 168, J[96] at 552)
@pytest.mark.parametrize("m,n,ties", [(1000, 64, True), (4096, 2048, False), (20, 40, True), (33000, 96, True)])
def test_rule_hard_selection(pkg, oracle, torch_mod, m, n, ties):
    torch = torch_mod
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    rng = np.random.default_rng(m)
    k = 512
    if ties:   # few distinct values: long runs of equal hard values
        r = rng.integers(-3, 3, m).astype(np.int32)
        sA = rng.choice([1.0, 2.0, 4.0], m)
        c = rng.integers(-3, 3, n).astype(np.int32)
        sB = rng.choice([1.0, 2.0], n)
    else:
        r = rng.integers(-40, 40, m).astype(np.int32)
        sA = rng.uniform(0.5, 600.0, m)
        c = rng.integers(-40, 40, n).astype(np.int32)
        sB = rng.uniform(0.5, 600.0, n)
    sA[::7] = 0.0                                           # hard value 0
    dv = {x: torch.from_numpy(np.ascontiguousarray(v)).cuda() for x, v in
          (("r", r), ("c", c), ("sA", sA), ("sB", sB), ("nA", np.ones(m)), ("nB", np.ones(n)),
           ("flag", np.zeros(1, np.int32)))}
    ws = torch.zeros(L.ozk_rule_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    ctl = torch.zeros(8, dtype=torch.int32, device="cuda")
    aux = torch.zeros(8, dtype=torch.float64, device="cuda")
    pkg._lib.check(L.ozk_rule_prepare(ptr(dv["r"]), ptr(dv["c"]), ptr(dv["sA"]), ptr(dv["nA"]), ptr(dv["sB"]),
                                      ptr(dv["nB"]), ptr(dv["flag"]), m, n, k, None, 0, None, 0, 0, -1,
                                      ptr(ctl[0:4]), ptr(ctl[5:6]), ptr(aux), ptr(ws), ws.numel(),
                                      torch.cuda.current_stream().cuda_stream), "ozk_rule_prepare")
    torch.cuda.synchronize()
    raw = ws.cpu().numpy()
    I = raw[168:168 + 96 * 4].view(np.int32)[:min(32, m)]
    J = raw[552:552 + 96 * 4].view(np.int32)[:min(32, n)]
    assert np.array_equal(I, oracle.hard_top(r, sA, k)) and np.array_equal(J, oracle.hard_top(c, sB, k))


@pytest.mark.parametrize("shape,phi,seed", [((256, 1024, 192), 1.0, 21), ((384, 640, 96), 2.0, 22)])
def test_ozk_core_c_abi_equals_engine_core(pkg, oracle, engine, torch_mod, shape, phi, seed):
    """``ozk_core``, the one-call replacement of the reference's core() (ozaki_engine.py:1310-1350) that an
    integrator binds directly, called through ctypes with its own plane buffers: C bit for bit equal to
    ``engine.core`` and to the oracle, with skip_a reusing the A planes of the first call."""
    torch = torch_mod
    L, ptr = pkg._lib.lib(), pkg._lib.ptr
    m, k, n = shape
    A, B = pkg.make_inputs(m, k, n, phi, seed)
    Ad, Bd = T(torch, A), T(torch, B)
    C_ref, info = engine.run(Ad, Bd)
    N, p = info["N"], info["p"]
    b = engine.buffers(m, n, k, N)
    engine.stats(Ad, Bd, b, True)
    b["pdev"].fill_(p)
    Ares = torch.empty(N * m * k, dtype=torch.int8, device="cuda")
    Bres = torch.empty(N * n * k, dtype=torch.int8, device="cuda")
    X = torch.empty(N * m * n, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for skip_a in (0, 1):
        C = torch.full((m, n), float("nan"), dtype=torch.float64, device="cuda")
        pkg._lib.check(L.ozk_core(ptr(Ad), ptr(Bd), ptr(b["gam"]), ptr(b["r"]), ptr(b["c"]), ptr(b["pdev"]), m, n, k,
                                  N, skip_a, ptr(Ares), ptr(Bres), ptr(X), ptr(C), ptr(err), st), "ozk_core")
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(C, C_ref), skip_a
    st_o = oracle.stats(A, B, True)
    np.testing.assert_array_equal(C.cpu().numpy().view(np.uint64), oracle.core(A, B, st_o, N, p).view(np.uint64))


def test_host_paths_raise_on_device_error_word(pkg, torch_mod):
    """A device error word set by a bounded wait that ran out (split, products or reconstruction) makes the
    host-buffer entry points raise instead of returning C: here the word is set by hand between calls."""
    torch = torch_mod
    A, B = pkg.make_inputs(128, 128, 128, 0.5, seed=3)
    E = pkg.OzakiCRT()
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    C, _ = E.run_host(Ah, Bh)
    Cd, _ = E.run(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
    assert torch.equal(C, Cd.cpu())
    for ws in E.bufs.values():
        ws.error_word.fill_(16)                                  # OZK_DEVERR_TIMEOUT_SPLIT
    with pytest.raises(pkg._lib.OzkError):
        E.run_host(Ah, Bh)
    with pytest.raises(pkg._lib.OzkError):
        E.run_host_many([(Ah, Bh, None), (Ah, Bh, None)])
    with pytest.raises(pkg._lib.OzkError):
        E.check_errors()


_GENERAL_SPLIT_CHILD = r"""
import os, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, os.path.join(sys.argv[1], "oracle"))
import __graft_entry__
import oracle
pkg = __graft_entry__.load_package()
oracle.build()
L, ptr = pkg._lib.lib(), pkg._lib.ptr
for (m, k, n, N, p) in [(96, 160, 64, 18, 67), (40, 96, 32, 13, 104), (64, 256, 96, 20, 58)]:
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=m + N)
    Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    st = {x: torch.empty(m if x in ("r", "sA", "nA") else (n if x in ("c", "sB", "nB") else (k if x == "gam" else 1)),
                         dtype=torch.float64 if x[0] in "sn" else torch.int32, device="cuda")
          for x in ("gam", "r", "c", "sA", "nA", "sB", "nB", "flag")}
    ws = torch.empty(L.ozk_stats_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    pkg._lib.check(L.ozk_stats(ptr(Ad), ptr(Bd), m, n, k, 1, *(ptr(st[x]) for x in ("gam", "r", "c", "sA", "nA", "sB", "nB", "flag")),
                               ptr(ws), ws.numel(), s), "stats")
    pd = torch.tensor([p], dtype=torch.int32, device="cuda"); err = torch.zeros(1, dtype=torch.int32, device="cuda")
    Ar = torch.empty((N, m, k), dtype=torch.int8, device="cuda"); Br = torch.empty((N, n, k), dtype=torch.int8, device="cuda")
    pkg._lib.check(L.ozk_split_a(ptr(Ad), ptr(st["r"]), ptr(st["gam"]), ptr(pd), m, k, N, ptr(Ar), ptr(err), s), "a")
    pkg._lib.check(L.ozk_split_b(ptr(Bd), ptr(st["c"]), ptr(st["gam"]), ptr(pd), k, n, N, ptr(Br), ptr(err), s), "b")
    torch.cuda.synchronize()
    sto = oracle.stats(A, B, True)
    assert np.array_equal(Ar.cpu().numpy(), oracle.split_A(A, sto["r"], sto["gam"], p, N)), (m, k, n, N, p)
    assert np.array_equal(Br.cpu().numpy(), oracle.split_B(B, sto["c"], sto["gam"], p, N)), (m, k, n, N, p)
    assert int(err.item()) == 0
print("general split ok")
"""


def test_general_split_kernel_for_small_p(oracle, torch_mod):
    """OZK_SPLIT_TC=0 (read once per process, hence a child process) keeps split.cu's kernel for p <= 119 too: it
    stays bit-exact against the oracle, as the tensor-core kernel is."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, OZK_SPLIT_TC="0")
    r = subprocess.run([sys.executable, "-c", _GENERAL_SPLIT_CHILD, root], env=env, cwd=root, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "general split ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
