"""Failure detection without a GPU fault: a wait inside the assignment kernel
that runs out.  A test hook makes the kernel's TMA producer leave one
centroid-plane stage unloaded, so the MMA issuer's bounded wait on it expires
(the limit is shortened to 50 ms); the kernel records MPK_DEV_TIMEOUT in the
engine's status word, every role winds down (in-flight loads drained, MMAs
completed, TMEM freed) and the kernel returns.  The host reads the status,
and the same engine and context then assign correctly."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu

MPK_DEV_TIMEOUT = 1


def test_assign_wait_timeout_is_reported_and_recoverable(cuda):
    rng = np.random.default_rng(21)
    n, d, k = 4096, 64, 300
    P = rng.standard_normal((n, d)).astype(np.float32)
    C = P[rng.choice(n, size=k, replace=False)].copy()
    dP, dC = torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda()
    lab = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    with M.Engine(dP, k, C0=dC) as e:
        e.set_wait_limit(50_000_000)
        e.inject_stall(3)                      # each CTA's fourth centroid-plane stage never arrives
        e.assign(dC, lab, refine=True)
        torch.cuda.synchronize()               # the kernel returned: no hang, no fault
        assert e.counters()["status"] & MPK_DEV_TIMEOUT
        e.inject_stall(-1)
        e.clear_status()
        e.set_wait_limit(0)
        e.assign(dC, lab, refine=True)
        torch.cuda.synchronize()
        assert e.counters()["status"] == 0
    assert np.array_equal(lab.cpu().numpy(), O.assign_fp32(P, C))
    assert float(torch.ones(4, device="cuda").sum()) == 4.0     # the context is still usable
