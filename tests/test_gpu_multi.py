"""Multi-GPU entry point: mpkMeansMixedMG over two B200s equals the one-GPU
mpkMeansMixed bit for bit (exact int64 sums, one global operand scale)."""
import ctypes

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d,k", [(64, 128), (256, 1024)])     # d = 256: the CTA-pair assignment
def test_mg_two_gpus_equals_one(cuda, d, k):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    P = O.make_gmm(200_000, d, k, 9, 5.0, 0.5, 2.0, True)
    C0 = P[np.sort(O.init_random_idx(200_000, k, 9))].copy()
    lab1 = torch.empty(200_000, dtype=torch.int32, device="cuda:0")
    dC1 = torch.from_numpy(C0).to("cuda:0")
    M.means_mixed(torch.from_numpy(P).to("cuda:0"), dC1, lab1, M.params_init(max_iter=6))
    halves = [(0, 123_457), (123_457, 200_000)]
    dPs = [torch.from_numpy(P[a:b]).to(f"cuda:{g}") for g, (a, b) in enumerate(halves)]
    dCs = [torch.from_numpy(C0).to(f"cuda:{g}") for g in range(2)]
    dAs = [torch.empty(b - a, dtype=torch.int32, device=f"cuda:{g}") for g, (a, b) in enumerate(halves)]
    arr = lambda t, xs: (t * 2)(*xs)
    st = M.mpkStats()
    p = M.params_init(max_iter=6)
    rc = M.lib().mpkMeansMixedMG(2, arr(ctypes.c_int, [0, 1]), arr(ctypes.c_void_p, [x.data_ptr() for x in dPs]),
                                 arr(ctypes.c_int, [b - a for a, b in halves]), d, k,
                                 arr(ctypes.c_void_p, [x.data_ptr() for x in dCs]),
                                 arr(ctypes.c_void_p, [x.data_ptr() for x in dAs]), ctypes.byref(p), ctypes.byref(st))
    assert rc == M.MPK_OK
    assert st.iters == 6
    labs = torch.cat([dAs[0].cpu(), dAs[1].cpu()])
    assert torch.equal(labs, lab1.cpu())
    for g in range(2):
        assert torch.equal(dCs[g].cpu(), dC1.cpu())


def test_mg_two_gpus_wide_refinement_equals_one(cuda):
    """Config-5 geometry (k = 4096, offset 1e3) takes the wide refinement on
    each GPU; the sharded run still equals the one-GPU run bit for bit."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    rng = np.random.default_rng(12)
    n, d, k = 60_000, 64, 4096
    o = rng.standard_normal(d)
    o = o / np.linalg.norm(o) * 1e3
    means = o + 2.0 * rng.standard_normal((k, d))
    P = (means[rng.integers(0, k, n)] + rng.standard_normal((n, d))).astype(np.float32)
    C0 = P[np.sort(rng.choice(n, size=k, replace=False))].copy()
    lab1 = torch.empty(n, dtype=torch.int32, device="cuda:0")
    dC1 = torch.from_numpy(C0).to("cuda:0")
    M.means_mixed(torch.from_numpy(P).to("cuda:0"), dC1, lab1, M.params_init(max_iter=3))
    halves = [(0, 31_111), (31_111, n)]
    dPs = [torch.from_numpy(P[a:b]).to(f"cuda:{g}") for g, (a, b) in enumerate(halves)]
    dCs = [torch.from_numpy(C0).to(f"cuda:{g}") for g in range(2)]
    dAs = [torch.empty(b - a, dtype=torch.int32, device=f"cuda:{g}") for g, (a, b) in enumerate(halves)]
    arr = lambda t, xs: (t * 2)(*xs)
    st = M.mpkStats()
    p = M.params_init(max_iter=3)
    rc = M.lib().mpkMeansMixedMG(2, arr(ctypes.c_int, [0, 1]), arr(ctypes.c_void_p, [x.data_ptr() for x in dPs]),
                                 arr(ctypes.c_int, [b - a for a, b in halves]), d, k,
                                 arr(ctypes.c_void_p, [x.data_ptr() for x in dCs]),
                                 arr(ctypes.c_void_p, [x.data_ptr() for x in dAs]), ctypes.byref(p), ctypes.byref(st))
    assert rc == M.MPK_OK and st.iters == 3
    assert torch.equal(torch.cat([dAs[0].cpu(), dAs[1].cpu()]), lab1.cpu())
    for g in range(2):
        assert torch.equal(dCs[g].cpu(), dC1.cpu())
