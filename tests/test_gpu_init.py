"""k-means++ seeding on the device (mpkInitKMeansPP) against the oracle's
restatement of the same definition (oracle.kmeanspp_int): the picked rows
must be identical -- FP64 warp-order distances and exact integer sampling
leave nothing to the launch shape."""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu


def gpu_kpp(P, k, seed):
    dP = torch.from_numpy(np.ascontiguousarray(P)).cuda()
    C = M.kmeanspp(dP, k, seed)
    torch.cuda.synchronize()
    return C.cpu().numpy()


@pytest.mark.parametrize("n,d,k,seed", [(100_000, 32, 64, 1), (4096, 8, 100, 2), (4097, 3, 17, 3),
                                        (20_000, 300, 128, 4), (777, 1, 5, 5), (50, 16, 50, 6),
                                        (300_000, 128, 256, 7)])
def test_kmeanspp_equals_oracle(cuda, n, d, k, seed):
    rng = np.random.default_rng(seed)
    P = (rng.standard_normal((n, d)) * rng.uniform(0.5, 3.0, (n, 1))).astype(np.float32)
    got = gpu_kpp(P, k, seed)
    want, idx = O.kmeanspp_int(P, k, seed)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    if k < n:
        assert len(set(idx.tolist())) == k          # D^2 weighting never re-picks a chosen row


def test_kmeanspp_duplicates_and_degenerate(cuda):
    # many repeated rows: once every distinct row is chosen all weights are zero
    base = np.random.default_rng(9).standard_normal((6, 4)).astype(np.float32)
    P = np.repeat(base, 50, axis=0)
    got = gpu_kpp(P, 10, 11)
    want, _ = O.kmeanspp_int(P, 10, 11)
    assert np.array_equal(got, want)
    assert len({tuple(r) for r in got[:6]}) == 6      # the six distinct rows come first
    Z = np.zeros((1000, 8), np.float32)              # all identical: W = 0 from the start
    assert np.array_equal(gpu_kpp(Z, 7, 3), O.kmeanspp_int(Z, 7, 3)[0])


def test_kmeanspp_rejects_invalid(cuda):
    lib = M.lib()
    P = torch.zeros((10, 4), device="cuda")
    C = torch.zeros((11, 4), device="cuda")
    assert lib.mpkInitKMeansPP(P.data_ptr(), 10, 4, 11, 1, C.data_ptr()) == M.MPK_ERR_INVALID
    assert lib.mpkInitKMeansPP(P.data_ptr(), 10, 4, 0, 1, C.data_ptr()) == M.MPK_ERR_INVALID
    assert lib.mpkInitKMeansPP(None, 10, 4, 3, 1, C.data_ptr()) == M.MPK_ERR_INVALID


def test_config1_gpu_seeding_then_lloyd_bit_exact(cuda):
    """Configuration 1 end to end on the device: k-means++ from the seed, then
    20 Lloyd iterations -- centroids and labels equal to the oracle's."""
    P = O.make_config1(100_000, 32, seed=1)
    dP = torch.from_numpy(P).cuda()
    dC = M.kmeanspp(dP, 64, 1)
    lab = torch.empty(100_000, dtype=torch.int32, device="cuda")
    st = M.means_mixed(dP, dC, lab, M.params_init(max_iter=20))
    C0, _ = O.kmeanspp_int(P, 64, 1)
    frac = O.fixed_frac(float(np.abs(P).max()), len(P))
    olab, oC, _, it = O.lloyd(P, C0, 20, update_mode=1, frac=frac)
    assert st.iters == 20 and it == 20
    assert np.array_equal(lab.cpu().numpy(), olab)
    assert np.array_equal(dC.cpu().numpy().view(np.uint32), oC.view(np.uint32))
