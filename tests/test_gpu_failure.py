"""Failure detection without a GPU fault.  (1) A wait inside the assignment
kernel that runs out.  A test hook makes the kernel's TMA producer leave one
centroid-plane stage unloaded, so the MMA issuer's bounded wait on it expires
(the limit is shortened to 50 ms); the kernel records MPK_DEV_TIMEOUT in the
engine's status word, every role winds down (in-flight loads drained, MMAs
completed, TMEM freed) and the kernel returns.  The host reads the status,
and the same engine and context then assign correctly.  (2) Failures made on
the host: an allocation that fails, and an asynchronous NCCL error seen by the
multi-GPU driver's non-blocking wait."""
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


@pytest.mark.parametrize("d", [128, 512])         # resident point tile; streaming point chunks
def test_pair_kernel_wait_timeout_winds_down(cuda, d):
    """The CTA-pair assignment kernel with every wait limited to 2 us: waits run
    out in both CTAs of every pair, which then let their loads in flight land,
    meet at the cluster barrier and return.  The timeout is reported, the
    context stays usable, and the next assignment is exact."""
    rng = np.random.default_rng(22)
    n, k = 6000, 520
    P = rng.standard_normal((n, d)).astype(np.float32)
    C = P[rng.choice(n, size=k, replace=False)].copy()
    dP, dC = torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda()
    lab = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    with M.Engine(dP, k, C0=dC) as e:
        e.assign_pair(1)
        e.set_wait_limit(2_000)
        e.assign(dC, lab, refine=True)
        torch.cuda.synchronize()               # the kernel returned: no hang, no fault
        assert e.counters()["status"] & MPK_DEV_TIMEOUT
        e.clear_status()
        e.set_wait_limit(0)
        e.assign(dC, lab, refine=True)
        torch.cuda.synchronize()
        assert e.counters()["status"] == 0
    assert np.array_equal(lab.cpu().numpy(), O.assign_fp32(P, C))
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def test_allocation_failures_unwind(cuda):
    """Host-side injection: the n-th device allocation of a fit fails, for
    every n the fit makes.  Each call returns MPK_ERR_ALLOC with nothing left
    allocated, and the next fit is unaffected."""
    import ctypes
    rng = np.random.default_rng(5)
    n, d, k = 6000, 48, 300                      # k > 256: the wide scratch is allocated too
    P = rng.standard_normal((n, d)).astype(np.float32)
    C = P[rng.choice(n, size=k, replace=False)].copy()
    dP = torch.from_numpy(P).cuda()
    dC = torch.from_numpy(C).cuda()
    lab = torch.empty(n, dtype=torch.int32, device="cuda")
    L = M.lib()
    par = M.params_init(max_iter=3)
    # warm everything (pools, module loads) before the memory baseline
    assert L.mpkMeansMixed(None, dP.data_ptr(), n, d, k, dC.data_ptr(), lab.data_ptr(), ctypes.byref(par), None) == M.MPK_OK
    want_lab, want_C = lab.clone(), dC.clone()
    torch.cuda.synchronize()
    L.mpkTrimMemoryPool(0)
    free0 = torch.cuda.mem_get_info()[0]
    failed = 0
    for nth in range(1, 64):
        dC.copy_(torch.from_numpy(C))
        L.mpkDebugFailAlloc(nth)
        rc = L.mpkMeansMixed(None, dP.data_ptr(), n, d, k, dC.data_ptr(), lab.data_ptr(), ctypes.byref(par), None)
        if rc == M.MPK_OK:                       # the fit makes fewer than nth allocations
            break
        assert rc == M.MPK_ERR_ALLOC, (nth, rc)
        failed += 1
    L.mpkDebugFailAlloc(0)
    assert failed >= 10, failed                  # engine scratch, wide scratch and driver buffers
    torch.cuda.synchronize()
    L.mpkTrimMemoryPool(0)
    assert abs(torch.cuda.mem_get_info()[0] - free0) < (8 << 20)
    dC.copy_(torch.from_numpy(C))
    assert L.mpkMeansMixed(None, dP.data_ptr(), n, d, k, dC.data_ptr(), lab.data_ptr(), ctypes.byref(par), None) == M.MPK_OK
    assert torch.equal(lab, want_lab) and torch.equal(dC, want_C)


def test_mg_async_error_aborts_and_recovers(cuda):
    """mpkMeansMixedMG never blocks on a device: a (host-injected)
    asynchronous NCCL error found at its next wait on the devices (the one
    after the communicators' first, warm-up allreduce) aborts the communicators
    and returns MPK_ERR_CUDA; the next call builds new ones and matches the
    single-GPU driver."""
    import ctypes
    rng = np.random.default_rng(6)
    n, d, k = 8000, 32, 64
    P = rng.standard_normal((n, d)).astype(np.float32)
    C = P[:k].copy()
    dP = torch.from_numpy(P).cuda()
    L = M.lib()

    def mg(inject):
        dC = torch.from_numpy(C).cuda()
        lab = torch.empty(n, dtype=torch.int32, device="cuda")
        devs = (ctypes.c_int * 1)(0)
        Ps = (ctypes.c_void_p * 1)(dP.data_ptr())
        ns = (ctypes.c_int * 1)(n)
        Cs = (ctypes.c_void_p * 1)(dC.data_ptr())
        As = (ctypes.c_void_p * 1)(lab.data_ptr())
        st = M.mpkStats()
        par = M.params_init(max_iter=4)
        if inject:
            L.mpkDebugMGFailNextWait()
        rc = L.mpkMeansMixedMG(1, devs, Ps, ns, d, k, Cs, As, ctypes.byref(par), ctypes.byref(st))
        torch.cuda.synchronize()
        return rc, dC, lab

    rc, _, _ = mg(True)
    if rc == M.MPK_ERR_INVALID:
        pytest.skip("NCCL not loadable here")
    assert rc == M.MPK_ERR_CUDA
    rc, dC, lab = mg(False)
    assert rc == M.MPK_OK
    dC1 = torch.from_numpy(C).cuda()
    lab1 = torch.empty(n, dtype=torch.int32, device="cuda")
    M.means_mixed(dP, dC1, lab1, M.params_init(max_iter=4))
    assert torch.equal(lab, lab1) and torch.equal(dC, dC1)
