"""ozk_stats_noalloc: the statistics entry point for callers that cannot allocate device memory.

Such callers (a plugin that only receives device pointers from its host runtime, or code that may not call cudaMalloc
while it runs or records a CUDA graph) get the scratch from a static array inside the library instead of a workspace
argument.  This file is collected last on purpose: it checks that the static scratch gives the same outputs as the
workspace entry point, on two calls in a row (the second call must not see stale contents of the first), both in a
fresh process and after every other test has used the library."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _outputs(torch, m, n, k):
    d = "cuda"
    return {"gam": torch.empty(k, dtype=torch.int32, device=d), "r": torch.empty(m, dtype=torch.int32, device=d),
            "c": torch.empty(n, dtype=torch.int32, device=d), "sA": torch.empty(m, dtype=torch.float64, device=d),
            "nA": torch.empty(m, dtype=torch.float64, device=d), "sB": torch.empty(n, dtype=torch.float64, device=d),
            "nB": torch.empty(n, dtype=torch.float64, device=d), "flag": torch.empty(1, dtype=torch.int32, device=d)}


ORDER = ("gam", "r", "c", "sA", "nA", "sB", "nB", "flag")


def test_noalloc_stats_equal_workspace_stats_on_two_calls(pkg, oracle):
    import torch
    if not (torch.cuda.is_available() and torch.cuda.get_device_capability()[0] == 10):
        pytest.skip("no B200 GPU")
    L = pkg._lib.lib()
    ptr = pkg._lib.ptr
    st = torch.cuda.current_stream().cuda_stream
    # two different problems, the second smaller in k and with a zero row, so stale scratch would show
    for (m, k, n, phi, seed) in ((256, 2048, 384, 2.0, 41), (128, 512, 96, 0.5, 42)):
        A, B = pkg.make_inputs(m, k, n, phi, seed)
        A[5, :] = 0.0
        Ad, Bd = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
        ref = _outputs(torch, m, n, k)
        ws = torch.empty(L.ozk_stats_workspace_bytes(m, n, k), dtype=torch.uint8, device="cuda")
        pkg._lib.check(L.ozk_stats(ptr(Ad), ptr(Bd), m, n, k, 1, *(ptr(ref[x]) for x in ORDER), ptr(ws), ws.numel(), st),
                       "ozk_stats")
        got = _outputs(torch, m, n, k)
        for x in ORDER:
            got[x].fill_(-7)                      # outputs start as garbage
        pkg._lib.check(L.ozk_stats_noalloc(ptr(Ad), ptr(Bd), m, n, k, 1, *(ptr(got[x]) for x in ORDER), st),
                       "ozk_stats_noalloc")
        torch.cuda.synchronize()
        # the same kernels in the same fixed summation order: every output equal bit for bit
        for x in ORDER:
            assert torch.equal(got[x], ref[x]), x
        # and against the CPU restatement of the reference's statistics (sums within rtol 1e-13: the oracle adds in
        # another order)
        want = oracle.stats(A, B, True)
        for x in ("gam", "r", "c"):
            assert np.array_equal(got[x].cpu().numpy(), want[x]), x
        assert int(got["flag"].item()) == int(want["flag"])
        for x in ("sA", "nA", "sB", "nB"):
            np.testing.assert_allclose(got[x].cpu().numpy(), want[x], rtol=1e-13, atol=0, err_msg=x)


def test_noalloc_rejects_problems_beyond_its_scratch(pkg):
    L = pkg._lib.lib()
    # 2 column-chunk partial arrays of n doubles per 512 rows of B: k = n = 65536 needs 64 MiB > 16 MiB
    assert L.ozk_stats_workspace_bytes(64, 65536, 65536) > (16 << 20)
    rc = L.ozk_stats_noalloc(None, None, 64, 65536, 65536, 1, *([None] * 8), None)
    assert rc == -6
    assert "16 MiB" in pkg._lib.error_string(rc)
