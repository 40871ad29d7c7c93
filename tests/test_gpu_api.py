"""The rest of the k-means C ABI on a B200, each entry point against the
reference's own implementation (oracle/_ref, compiled from its sources) on the
same device inputs: preprocessing helpers, random-point seeding, the multiword
driver, and the optional back ends this build does not have."""
import ctypes

import numpy as np
import pytest

import oracle as O
import parity

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu

VP = ctypes.c_void_p


@pytest.fixture(scope="module")
def ref():
    if not O.REF_LIB_PATH.exists():
        pytest.skip("oracle/_ref/libmpkref.so not built")
    r = ctypes.CDLL(str(O.REF_LIB_PATH))
    r.mpkShiftNonNegative.argtypes = [VP, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
    r.mpkShiftCentroids.argtypes = [VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    r.mpkStandardize.argtypes = [VP, ctypes.c_int, ctypes.c_int]
    r.mpkInitRandomPoints.argtypes = [VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint, VP]
    r.mpkParamsInit.argtypes = [ctypes.POINTER(M.mpkParams)]
    r.mpkMeansMultiword.argtypes = [VP, VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, VP, VP,
                                    ctypes.POINTER(M.mpkParams), ctypes.POINTER(M.mpkStats)]
    return r


def data(n, d, seed, scale=3.0):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, d)) * scale + rng.uniform(-2, 2, d)).astype(np.float32)


def test_shift_helpers_equal_reference(cuda, ref):
    P = data(50_000, 24, 1)
    a, b = torch.from_numpy(P).cuda(), torch.from_numpy(P).cuda()
    sa, sb = ctypes.c_float(), ctypes.c_float()
    assert M.lib().mpkShiftNonNegative(a.data_ptr(), 50_000, 24, ctypes.byref(sa)) == M.MPK_OK
    assert ref.mpkShiftNonNegative(b.data_ptr(), 50_000, 24, ctypes.byref(sb)) == M.MPK_OK
    torch.cuda.synchronize()
    assert sa.value == sb.value == float(np.abs(P).max())
    assert torch.equal(a, b) and float(a.min()) >= 0.0
    C = torch.from_numpy(P[:100].copy()).cuda()
    C2 = C.clone()
    assert M.lib().mpkShiftCentroids(C.data_ptr(), 100, 24, ctypes.c_float(-1.25)) == M.MPK_OK
    assert ref.mpkShiftCentroids(C2.data_ptr(), 100, 24, ctypes.c_float(-1.25)) == M.MPK_OK
    torch.cuda.synchronize()
    assert torch.equal(C, C2)


def test_standardize_close_to_reference(cuda, ref):
    P = data(30_001, 17, 2)
    P[:, 5] = 4.0                                   # a constant feature (sd 0: divided by 1)
    a, b = torch.from_numpy(P).cuda(), torch.from_numpy(P).cuda()
    assert M.lib().mpkStandardize(a.data_ptr(), 30_001, 17) == M.MPK_OK
    assert ref.mpkStandardize(b.data_ptr(), 30_001, 17) == M.MPK_OK
    torch.cuda.synchronize()
    x, y = a.cpu().numpy(), b.cpu().numpy()
    assert np.abs(x - y).max() <= 4e-6 * max(1.0, float(np.abs(y).max())), np.abs(x - y).max()
    assert np.abs(x.mean(axis=0)).max() < 1e-5 and np.abs(x[:, 5]).max() == 0.0


def test_init_random_points_equal_reference(cuda, ref):
    P = data(20_000, 12, 3)
    dP = torch.from_numpy(P).cuda()
    for k, seed in ((64, 7), (1000, 8), (20_000, 9)):
        a = torch.zeros((k, 12), device="cuda")
        b = torch.zeros((k, 12), device="cuda")
        assert M.lib().mpkInitRandomPoints(dP.data_ptr(), 20_000, 12, k, seed, a.data_ptr()) == M.MPK_OK
        assert ref.mpkInitRandomPoints(dP.data_ptr(), 20_000, 12, k, seed, b.data_ptr()) == M.MPK_OK
        torch.cuda.synchronize()
        assert torch.equal(a, b)
        assert np.array_equal(a.cpu().numpy(), P[np.sort(O.init_random_idx(20_000, k, seed))])


def test_multiword_driver_against_reference(cuda, ref):
    """The reference's double-fp16 driver needs non-negative data (it shifts
    first) and at least one exclusion condition; one iteration from the same
    start gives the same labels up to FP32 near-ties and centroids within 1e-6;
    ten iterations the same inertia within 1e-5."""
    P = O.make_config1(60_000, 32, seed=4)
    dP = torch.from_numpy(P).cuda()
    sh = ctypes.c_float()
    assert M.lib().mpkShiftNonNegative(dP.data_ptr(), 60_000, 32, ctypes.byref(sh)) == M.MPK_OK
    Ps = dP.cpu().numpy()
    C0 = Ps[np.sort(O.init_random_idx(60_000, 64, 4))].copy()
    blas = torch.cuda.current_blas_handle()
    out = {}
    for name, lib in (("ours", M.lib()), ("ref", ref)):
        for iters in (1, 10):
            p = M.mpkParams()
            ref.mpkParamsInit(ctypes.byref(p))
            p.max_iter = iters
            st = M.mpkStats()
            dC = torch.from_numpy(C0).cuda()
            lab = torch.empty(60_000, dtype=torch.int32, device="cuda")
            assert lib.mpkMeansMultiword(blas, dP.data_ptr(), 60_000, 32, 64, dC.data_ptr(), lab.data_ptr(),
                                         ctypes.byref(p), ctypes.byref(st)) == M.MPK_OK, name
            torch.cuda.synchronize()
            out[(name, iters)] = (lab.cpu().numpy(), dC.cpu().numpy(), st.inertia, st.iters)
    lo, Co, _, _ = out[("ours", 1)]
    lr, Cr, _, _ = out[("ref", 1)]
    s = parity.summary(Ps, C0, lo, lr)
    assert s["agree"] >= 0.9999 and s["max_gap32"] < 1e-5, s
    rel = np.linalg.norm(Co - Cr, axis=1) / np.maximum(np.linalg.norm(Cr, axis=1), 1e-30)
    assert rel.max() < 1e-6, rel.max()
    io, ir = out[("ours", 10)][2], out[("ref", 10)][2]
    assert out[("ours", 10)][3] == out[("ref", 10)][3] == 10
    assert abs(io - ir) <= 1e-5 * ir, (io, ir)
    p = M.mpkParams()
    ref.mpkParamsInit(ctypes.byref(p))
    p.use_cond3 = p.use_cond6 = 0
    for lib in (M.lib(), ref):
        assert lib.mpkMeansMultiword(blas, dP.data_ptr(), 60_000, 32, 64, dC.data_ptr(), lab.data_ptr(),
                                     ctypes.byref(p), ctypes.byref(M.mpkStats())) == M.MPK_ERR_INVALID


def test_absent_backends_report_invalid(cuda):
    L = M.lib()
    assert L.mpkHaveCuvs() == 0
    z = torch.zeros(64, device="cuda")
    lab = torch.zeros(16, dtype=torch.int32, device="cuda")
    for fn in (L.mpkMeansBaselineRT, L.mpkMeansCuvs):
        assert fn(None, z.data_ptr(), 16, 4, 2, z.data_ptr(), lab.data_ptr(), None, None) == M.MPK_ERR_INVALID


def test_trim_memory_pool(cuda):
    """After a fit the engine's pool keeps its blocks; trimming hands them back."""
    P = torch.randn((200_000, 64), device="cuda")
    C = P[:256].clone()
    lab = torch.empty(200_000, dtype=torch.int32, device="cuda")
    M.means_mixed(P, C, lab, M.params_init(max_iter=2))
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert M.lib().mpkTrimMemoryPool(-1) == M.MPK_OK
    free1, _ = torch.cuda.mem_get_info()
    assert free1 >= free0 + 50 * 2**20          # at least the 51 MB of split planes came back
    assert M.lib().mpkTrimMemoryPool(999) == M.MPK_ERR_INVALID
