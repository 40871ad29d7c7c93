"""mpkUpdateNoAlloc, the update for callers that cannot allocate device memory
(a device owned by a pool or custom allocator, an allocator that may not be
re-entered, a fixed footprint): it must give exactly what mpkUpdate gives,
through the C ABI, on two calls in a row -- the second call finds the first
call's values still in the shared fixed scratch array and must not be
affected by them.  Collected last so that a failure here cannot hide any
other test's result."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu


def _problem(n, d, k, seed):
    rng = np.random.default_rng(seed)
    P = rng.standard_normal((n, d)).astype(np.float32) * 3.0
    C = P[rng.choice(n, size=k, replace=False)].copy()
    lab = rng.integers(0, k, size=n).astype(np.int32)
    lab[lab == k - 1] = 0                      # one empty cluster: keeps its centroid
    return torch.from_numpy(P).cuda(), torch.from_numpy(C).cuda(), torch.from_numpy(lab).cuda()


def _update_both(P, C, lab):
    n, d = P.shape
    k = C.shape[0]
    lib = M.lib()
    C_ref = C.clone()
    m_ref = torch.empty(k, dtype=torch.float32, device="cuda")
    assert lib.mpkUpdate(None, P.data_ptr(), n, d, k, lab.data_ptr(), C_ref.data_ptr(), m_ref.data_ptr()) == M.MPK_OK
    C_na = C.clone()
    m_na = torch.empty(k, dtype=torch.float32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.mpkUpdateNoAlloc(stream, P.data_ptr(), n, d, k, lab.data_ptr(), C_na.data_ptr(),
                                m_na.data_ptr()) == M.MPK_OK
    torch.cuda.synchronize()
    return C_ref, m_ref, C_na, m_na


def test_no_alloc_update_matches_update_twice(cuda):
    # the first call is larger than the second, so the second finds stale
    # sums, counts and row indices past its own sizes in the fixed array
    for (n, d, k, seed) in [(300_000, 128, 1024, 1), (40_000, 32, 64, 2)]:
        P, C, lab = _problem(n, d, k, seed)
        C_ref, m_ref, C_na, m_na = _update_both(P, C, lab)
        assert torch.equal(C_na, C_ref)          # same arithmetic: bit for bit
        assert torch.equal(m_na, m_ref)
        assert torch.equal(C_na[k - 1], C[k - 1])


def test_no_alloc_update_allocates_nothing(cuda):
    """After a first call (which may place the library's fixed array on the device),
    further calls leave the device's free memory exactly where it was."""
    n, d, k = 200_000, 64, 256
    P, C, lab = _problem(n, d, k, 3)
    lib = M.lib()
    stream = torch.cuda.current_stream().cuda_stream
    moved = torch.empty(k, dtype=torch.float32, device="cuda")

    def call():
        assert lib.mpkUpdateNoAlloc(stream, P.data_ptr(), n, d, k, lab.data_ptr(), C.data_ptr(),
                                    moved.data_ptr()) == M.MPK_OK

    call()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_no_alloc_update_rejects_what_does_not_fit(cuda):
    lib = M.lib()
    P = torch.zeros((16, 8), dtype=torch.float32, device="cuda")
    C = torch.zeros((4, 8), dtype=torch.float32, device="cuda")
    lab = torch.zeros(16, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # k*d int64 sums alone exceed the 32 MiB array: refused before any device work
    assert lib.mpkUpdateNoAlloc(stream, P.data_ptr(), 16, 8, 600_000, lab.data_ptr(), C.data_ptr(),
                                None) == M.MPK_ERR_INVALID
    bad = torch.full((16,), 9, dtype=torch.int32, device="cuda")
    assert lib.mpkUpdateNoAlloc(stream, P.data_ptr(), 16, 8, 4, bad.data_ptr(), C.data_ptr(),
                                None) == M.MPK_ERR_INVALID
