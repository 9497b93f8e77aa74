"""The GEMM's bounded waits on a B200 (matrix-numbers_b200/csrc/gemm_tc.cu: mbar_wait_bounded, raise_abort).

ozk_wait_selftest runs the GEMM's roles on one CTA over mbarriers that nothing arrives on.  The timed role waits
out its limit, reports its OZK_DEVERR_TIMEOUT_* flag and raises the CTA's abort flag.  The other role has the
GEMM's own 4 s limit and must leave through that flag, well before 4 s.  The TMEM that the CTA holds is freed.
The context stays usable: a GEMM launched on the same stream afterwards is exact.  Every wait ends by its own
wall-time limit.  No fault, trap or endless loop is involved.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLAGS = {0: 1, 1: 4}          # OZK_DEVERR_TIMEOUT_PRODUCER, OZK_DEVERR_TIMEOUT_EPILOGUE
LIMIT_NS = 20_000_000         # 20 ms: the timed role's limit
SLACK_NS = 200_000_000        # the wait checks its clock every 256 polls, so it ends within microseconds of the limit


@pytest.mark.parametrize("role", [0, 1])
def test_wait_runs_out_and_reports(pkg, oracle, engine, role):
    import torch
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    s = torch.cuda.current_stream().cuda_stream
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    pkg._lib.check(L.ozk_wait_selftest(role, LIMIT_NS, ptr(err), ptr(waited), s), "ozk_wait_selftest")
    torch.cuda.synchronize()
    assert int(err.item()) == FLAGS[role]            # only the timed role reports; the other left by the abort flag
    w = waited.cpu().numpy()
    assert LIMIT_NS <= w[role] < LIMIT_NS + SLACK_NS
    assert 0 <= w[1 - role] < LIMIT_NS + SLACK_NS    # far below its own 4 s limit

    # the context is intact: the tensor-core GEMM (which allocates all 512 TMEM columns) runs next and is exact
    rng = np.random.default_rng(11 + role)
    m, n, k = 256, 512, 1024
    At = rng.integers(-128, 128, size=(m, k), dtype=np.int8)
    Bt = rng.integers(-128, 128, size=(n, k), dtype=np.int8)
    Ad, Bd = torch.from_numpy(At).cuda(), torch.from_numpy(Bt).cuda()
    C = torch.empty((m, n), dtype=torch.int32, device="cuda")
    err.zero_()
    pkg._lib.check(L.ozk_gemm_i32(ptr(Ad), ptr(Bd), m, n, k, ptr(C), ptr(err), s), "gemm_i32")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert np.array_equal(C.cpu().numpy(), oracle.gemm_i32(At, Bt))
