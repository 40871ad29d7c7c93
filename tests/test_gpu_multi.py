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


@pytest.mark.parametrize("d,k", [(64, 300), (256, 1024)])
def test_peer_combine_two_gpus_equals_allreduce_and_finalize(cuda, d, k):
    """mpkPeerCombine (each GPU finalises its half of the clusters from both GPUs'
    int64 sums read over NVLink, then copies the other half) equals adding the
    two sums and finalising, bit for bit, centroids and moved^2, for six
    iterations driven by mpkEngineStep; and the fit equals the one-GPU
    mpkMeansMixed.  k = 300 splits the clusters 150 / 150, k = 1024 512 / 512."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n = 120_000
    P = O.make_gmm(n, d, k, 17, 5.0, 0.5, 2.0, True)
    C0 = P[np.sort(O.init_random_idx(n, k, 17))].copy()
    lab1 = torch.empty(n, dtype=torch.int32, device="cuda:0")
    dC1 = torch.from_numpy(C0).to("cuda:0")
    M.means_mixed(torch.from_numpy(P).to("cuda:0"), dC1, lab1, M.params_init(max_iter=6))
    pmax = float(max(np.abs(P).max(), np.abs(C0).max()))
    halves = [(0, 70_001), (70_001, n)]
    devs = [torch.device("cuda", g) for g in range(2)]
    streams = [torch.cuda.Stream(dv) for dv in devs]
    dPs = [torch.from_numpy(P[a:b]).to(dv) for (a, b), dv in zip(halves, devs)]
    eng, grp, labs, Cs, Cr, sums_r, mv, mv_r = [], [], [], [], [], [], [], []
    for g, dv in enumerate(devs):
        with torch.cuda.device(dv):
            eng.append(M.Engine(dPs[g], k, pmax_global=pmax, n_global=n, stream=streams[g].cuda_stream))
            grp.append(M.PeerGroup(g, 2, k, d))
            labs.append(torch.empty(halves[g][1] - halves[g][0], dtype=torch.int32, device=dv))
            Cs.append(torch.from_numpy(C0).to(dv))
            Cr.append(torch.from_numpy(C0).to(dv))
            sums_r.append(torch.empty(eng[g].sums_length, dtype=torch.int64, device=dv))
            mv.append(torch.empty(k, dtype=torch.float32, device=dv))
            mv_r.append(torch.empty(k, dtype=torch.float32, device=dv))
    try:
        bases = [grp[0].base(), grp[1].base()]
        for g in range(2):
            with torch.cuda.device(devs[g]):
                grp[g].connect_local(bases, [0, 1])
        lab_r = [torch.empty_like(x) for x in labs]
        for _ in range(6):
            # the reference path: the same steps into plain buffers, sums added on the host side, finalised
            for g in range(2):
                with torch.cuda.device(devs[g]):
                    eng[g].step(Cr[g], lab_r[g], sums_r[g])
            for g in range(2):
                streams[g].synchronize()
            tot = sums_r[0].cpu() + sums_r[1].cpu()
            for g in range(2):
                with torch.cuda.device(devs[g]), torch.cuda.stream(streams[g]):
                    sums_r[g].copy_(tot)           # on the engine's stream, before its finalisation
                    eng[g].finalize(sums_r[g], Cr[g], mv_r[g])
            # the fused path
            for g in range(2):
                with torch.cuda.device(devs[g]):
                    eng[g].step(Cs[g], labs[g], grp[g].sums)
            for g in range(2):
                with torch.cuda.device(devs[g]):
                    grp[g].combine(eng[g], Cs[g], mv[g])
            for g in range(2):
                streams[g].synchronize()
                with torch.cuda.device(devs[g]):
                    assert eng[g].counters()["status"] == 0
                assert torch.equal(Cs[g].cpu(), Cr[g].cpu())
                assert torch.equal(mv[g].cpu(), mv_r[g].cpu())
                assert torch.equal(labs[g].cpu(), lab_r[g].cpu())
        assert torch.equal(torch.cat([labs[0].cpu(), labs[1].cpu()]), lab1.cpu())
        assert torch.equal(Cs[0].cpu(), dC1.cpu()) and torch.equal(Cs[1].cpu(), dC1.cpu())
    finally:
        for g in range(2):
            with torch.cuda.device(devs[g]):
                streams[g].synchronize()
                eng[g].close()
                grp[g].close()
