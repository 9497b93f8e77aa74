"""``run_host``: host buffers in and out, the core in row blocks with each finished block of C copied back while the
next one computes.  Bit-exact against the device-resident ``run``; the fallback path fills the host C too."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,k,n,blocks", [(1000, 512, 256, 4), (256, 1024, 512, 1), (1536, 256, 128, 3)])
def test_run_host_equals_run(pkg, engine, m, k, n, blocks):
    import torch
    A, B = pkg.make_inputs(m, k, n, 2.0, seed=m + n)
    Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
    for _ in range(2):
        Ch, info = engine.run_host(Ah, Bh, blocks=blocks)
        assert not Ch.is_cuda and not info.get("fallback")
        C, ir = engine.run(Ah.cuda(), Bh.cuda())
        assert (info["N"], info["p"]) == (ir["N"], ir["p"])
        assert np.array_equal(Ch.numpy(), C.cpu().numpy())


def test_run_host_fallback(pkg, engine):
    import torch
    A, B = pkg.make_inputs(256, 256, 128, 1.0, seed=1)
    B[7, 9] = np.inf
    Ch, info = engine.run_host(torch.from_numpy(A), torch.from_numpy(B))
    assert info.get("fallback")
    assert np.array_equal(np.isinf(Ch.numpy()), np.isinf(A @ B))


def test_run_host_many_equals_run_host(pkg, engine):
    """A stream of jobs through the double-buffered host path (next job's H2D overlapped with this job's products):
    every result equals run_host's bit for bit, including a non-finite job in the middle (native fallback) and
    results written into caller-supplied pinned buffers."""
    import torch
    m, k, n = 260, 192, 320
    jobs, want = [], []
    for seed in range(5):
        A, B = pkg.make_inputs(m, k, n, 1.0 + 0.5 * seed, seed=seed)
        if seed == 2:
            A[3, 5] = np.nan
        Ah, Bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(B).pin_memory()
        Ch = torch.full((m, n), -1.0, dtype=torch.float64).pin_memory() if seed % 2 else None
        jobs.append((Ah, Bh, Ch))
        want.append(engine.run_host(Ah, Bh, None, blocks=3))
    got = engine.run_host_many(jobs, blocks=3)
    assert len(got) == len(jobs)
    for (C, info), (Cw, iw), (_, _, Ch) in zip(got, want, jobs):
        if Ch is not None:
            assert C is Ch
        if iw.get("fallback"):
            assert info.get("fallback")
            np.testing.assert_array_equal(np.isnan(C.numpy()), np.isnan(Cw.numpy()))
        else:
            assert (info["N"], info["p"]) == (iw["N"], iw["p"])
            np.testing.assert_array_equal(C.numpy().view(np.uint64), Cw.numpy().view(np.uint64))
    assert engine.run_host_many([]) == []
