"""The CPU oracle, pinned against the reference: its host code (run here from
the reference's own compiled library), its known-answer tests, and the golden
outputs of its GPU code (tests/golden/*.npz, made by make_golden.py)."""
import ctypes

import numpy as np
import pytest

import oracle as O
import parity
from conftest import golden


def adjudicate(P, C, la, lb):
    """Label mismatches between two assignments against the same C, with the
    FP64 direct-formula relative gap |D(a) - D(b)| / max(D(a), D(b))."""
    idx = np.nonzero(la != lb)[0]
    if len(idx) == 0:
        return 0, 0.0
    da = O.dist64_pairs(P, C, idx, la[idx])
    db = O.dist64_pairs(P, C, idx, lb[idx])
    rel = np.abs(da - db) / np.maximum(np.maximum(da, db), 1e-300)
    return len(idx), float(rel.max())


def ref_lib():
    if not O.REF_LIB_PATH.exists():
        pytest.skip("oracle/_ref/libmpkref.so not built (needs the reference sources)")
    return ctypes.CDLL(str(O.REF_LIB_PATH))


# ------------------------------------------------ reference host code -------

def test_blobs_bit_exact_vs_reference_host_code():
    ref = ref_lib()
    for (n, d, k, std, box, seed) in [(1000, 8, 4, 1.0, 10.0, 7), (333, 17, 5, 0.5, 3.0, 123)]:
        P, L = O.make_blobs_ref(n, d, k, std, box, seed)
        Pr = np.empty((n, d), np.float32)
        Lr = np.empty(n, np.int32)
        ref.mpkMakeBlobs(n, d, k, ctypes.c_float(std), ctypes.c_float(box), ctypes.c_uint(seed),
                         Pr.ctypes.data_as(ctypes.c_void_p), Lr.ctypes.data_as(ctypes.c_void_p))
        assert np.array_equal(P.view(np.uint32), Pr.view(np.uint32))
        assert np.array_equal(L, Lr)


def test_epsilon_matches_reference_host_code():
    ref = ref_lib()
    ref.mpkEpsilon.restype = ctypes.c_double
    for d in (1, 32, 128, 768, 4096, 100000):
        for acc in (0, 1):
            assert O.mpk_epsilon(d, acc) == ref.mpkEpsilon(d, acc)


def test_library_host_formulas_match_reference_host_code():
    """The library's own mpkEpsilon / mpkMultiwordEpsilon (host functions of the
    product, callable without a GPU) against the reference's, and the
    optional-backend probe."""
    import mpkmeans_b200 as M
    ref = ref_lib()
    ref.mpkEpsilon.restype = ctypes.c_double
    ref.mpkMultiwordEpsilon.restype = ctypes.c_double
    L = M.lib()
    L.mpkMultiwordEpsilon.restype = ctypes.c_double
    L.mpkMultiwordEpsilon.argtypes = [ctypes.c_int, ctypes.c_int]
    for d in (1, 32, 128, 768, 4096, 100000):
        for acc in (0, 1):
            assert L.mpkEpsilon(d, acc) == ref.mpkEpsilon(d, acc)
        for macs in (1, 2, 3, 6):
            assert L.mpkMultiwordEpsilon(d, macs) == ref.mpkMultiwordEpsilon(d, macs), (d, macs)
    assert L.mpkHaveCuvs() == 0


def test_term_schedule_known_answer():
    # gemm-emulation/bench/test_split.cu:135-145
    want = [(0, 0), (0, 1), (1, 0), (0, 2), (1, 1), (2, 0), (1, 2), (2, 1), (2, 2)]
    assert O.term_schedule(3, 16) == want
    for cap in (1, 3, 6, 9):
        assert len(O.term_schedule(3, cap)) == cap
    assert O.term_schedule(0, 4) == [] and O.term_schedule(17, 4) == []
    assert len(O.term_schedule(16, 1000)) == 256


# ------------------------------------------------------------- splits -------

@pytest.mark.parametrize("rows,cols,lda,emax", [(1024, 64, 1024, 0), (1023, 77, 1023, 0), (100, 33, 101, 0),
                                                 (1, 1, 1, 0), (7, 3, 9, 0), (512, 64, 512, 30)])
def test_bf16_three_split_exact(rows, cols, lda, emax):
    # gemm-emulation/bench/test_split.cu:113-126: 3 words reconstruct bit-exactly
    A = O.make_uniform((cols, lda), 99, emax=0)
    if emax:
        w = O.make_uniform((cols, lda), 98)
        A = (A * np.exp2(w.astype(np.float64) * emax)).astype(np.float32)
    S, lds, stride = O.split_bf16(A, rows, cols, lda, 3)
    planes = [O.bf16_to_f32(S[s * stride:(s + 1) * stride]).reshape(cols, lds)[:, :rows] for s in range(3)]
    rec = (planes[0] + planes[1]) + planes[2]
    assert np.array_equal(rec, A[:, :rows])


def test_fp16_split_normwise_bounds():
    # gemm-emulation/bench/test_split_fp16.cu:131-140: [0.25, 0.5], scaled
    rows = cols = 256
    u = O.make_uniform((cols, rows), 5)
    A = (0.375 + 0.125 * u).astype(np.float32)
    sc = O.autoscale_fp16(A, rows, cols, rows)
    for p, bound in ((1, 1e-3), (2, 1e-6), (3, 1e-8)):
        S, lds, stride = O.split_fp16(A, rows, cols, rows, p, sc)
        rec = sum(O.fp16_to_f32(S[s * stride:(s + 1) * stride]).astype(np.float64) for s in range(p))
        rec = rec.reshape(cols, lds)[:, :rows] / sc
        err = np.linalg.norm(rec - A) / np.linalg.norm(A)
        assert err <= bound, (p, err)


def test_autoscale_rule():
    A = np.full((4, 4), 3.0, np.float32)
    assert O.autoscale_fp16(A, 4, 4, 4) == 1024.0     # 4096/3 ~ 1365 -> 2^10
    assert O.autoscale_fp16(np.zeros((2, 2), np.float32), 2, 2, 2) == 1.0


# ------------------------------------------------------------ k-means -------

def test_warp_dot_order_and_norm_tree():
    rng = np.random.default_rng(0)
    for d in (1, 31, 32, 33, 128, 300):
        p = rng.standard_normal(d).astype(np.float32)
        c = rng.standard_normal(d).astype(np.float32)
        ref64 = float(np.dot(p.astype(np.float64), c.astype(np.float64)))
        got = O.lib().orc_dot_warp(p, c, d)
        assert abs(got - ref64) <= d * 2.0 ** -24 * float(np.abs(p) @ np.abs(c)) + 1e-30
        nt = O.lib().orc_norm2_tree(c, d)
        assert abs(nt - float(c.astype(np.float64) @ c)) <= d * 2.0 ** -24 * float(c @ c)


def test_fixed_point_update_matches_fp64_update():
    P = O.make_config1(20_000, 32, seed=2)
    C0 = O.kmeanspp(P, 64, seed=2)
    lab = O.assign_fp32(P, C0)
    frac = O.fixed_frac(float(np.abs(P).max()), len(P))
    Cf, _, cf, S = O.update_fixed(P, lab, C0, frac)
    Cd, _, cd = O.update_fp64(P, lab, C0)
    assert np.array_equal(cf, cd)
    ulp = np.abs(Cf.view(np.int32).astype(np.int64) - Cd.view(np.int32).astype(np.int64))
    assert ulp.max() <= 1
    assert (S.sum(axis=0) == np.round(P.astype(np.float64) * 2.0 ** frac).astype(np.int64).sum(axis=0)).all()


def test_lloyd_runs_max_iter_and_tol():
    P = O.make_config1(5000, 8, seed=4)
    C0 = O.kmeanspp(P, 10, seed=4)
    _, _, _, it = O.lloyd(P, C0, 7)
    assert it == 7
    _, _, _, it = O.lloyd(P, C0, 500, tol=1e-3)
    assert 1 <= it < 500


# ---------------------------------------------------- golden pins -----------

def test_golden_blobs_trajectory():
    g = golden("ref_blobs.npz")
    n, d, k, seed = int(g["n"]), int(g["d"]), int(g["k"]), int(g["seed"])
    P, _ = O.make_blobs_ref(n, d, k, 1.0, 10.0, seed)
    idx = np.sort(O.init_random_idx(n, k, seed))
    assert np.array_equal(P[idx], g["C0"]), "mpkInitRandomPoints selection"
    C = g["C0"].copy()
    for t in range(g["traj_labels"].shape[0]):
        lab = O.assign_fp32(P, C)
        nm, rel = adjudicate(P, C, lab, g["traj_labels"][t].astype(np.int32))
        assert nm == 0 or rel < 1e-5, (t, nm, rel)
        Cn, _, _ = O.update_fp64(P, g["traj_labels"][t].astype(np.int32), C)
        assert np.allclose(Cn, g["traj_C"][t], rtol=1e-6, atol=1e-6)
        C = g["traj_C"][t]
    lab, Cf, ine, _ = O.lloyd(P, g["C0"], 10)
    agree = (lab == g["labels"].astype(np.int32)).mean()
    assert agree >= 0.9999
    assert abs(ine - float(g["inertia"])) / float(g["inertia"]) < 1e-5


def test_golden_config1():
    """BASELINE config 1.  Per iteration on the reference's own centroids the
    oracle's labels differ only on FP32 near-ties; the 20-iteration run is not
    converged, so one near-tie decided the other way moves later iterations a
    little: end-of-run agreement and inertia are bounded, not exact."""
    g = golden("ref_config1.npz")
    P = O.make_config1(int(g["n"]), int(g["d"]), seed=int(g["seed"]))
    C0 = O.kmeanspp(P, int(g["k"]), seed=int(g["seed"]))
    assert np.array_equal(C0, g["C0"])
    lab0 = O.assign_fp32(P, C0)
    s = parity.summary(P, C0, lab0, g["labels_it0"].astype(np.int32))
    assert s["max_gap32"] < 1e-5 and s["max_gap64"] < 1e-5, s
    if "traj_labels" in g.files:
        C = C0
        for t in range(g["traj_labels"].shape[0]):
            lab = O.assign_fp32(P, C)
            s = parity.summary(P, C, lab, g["traj_labels"][t].astype(np.int32))
            assert s["max_gap32"] < 1e-5 and s["agree"] >= 0.9999, (t, s)
            Cn, _, _ = O.update_fp64(P, g["traj_labels"][t].astype(np.int32), C)
            assert np.allclose(Cn, g["traj_C"][t], rtol=1e-6, atol=1e-6), t
            C = g["traj_C"][t]
    lab, C, ine, _ = O.lloyd(P, C0, 20)
    assert (lab == g["labels"].astype(np.int32)).mean() >= 0.999
    assert abs(ine - float(g["inertia"])) / float(g["inertia"]) < 1e-5


def _floor_runs(f, prefix, variants):
    base = (f[f"{prefix}_base_labels"].astype(np.int32), f[f"{prefix}_base_C"], float(f[f"{prefix}_base_inertia"]))
    runs = {v: (f[f"{prefix}_{v}_labels"].astype(np.int32), f[f"{prefix}_{v}_C"], float(f[f"{prefix}_{v}_inertia"]))
            for v in variants}
    return base, runs


@pytest.mark.parametrize("iters", [20, 100])
def test_reference_noise_floor_config1(iters):
    """The reference against itself (tests/golden/ref_floor.npz, made by its own
    mpkMeansFP32 on a B200): a repeated call and a row-permuted copy end bit-identical,
    but permuting the coordinates -- the same points, only every FP32 dot summed in
    another order -- moves the end of a 20- or 100-iteration run: labels agree on
    99.7-99.98 %, centroids differ by 3e-4 to 2e-3 (relative Frobenius).  The oracle's
    run (the engine's arithmetic: its labels and centroids are bit-exact to it on the
    GPU) lies inside that spread: the north-star end-of-run bar (99.99 %, 1e-5) is
    below the reference's own noise floor here."""
    f = golden("ref_floor.npz")
    P = O.make_config1(100_000, 32, seed=1)
    C0 = f["c1_C0"]
    assert np.array_equal(C0, O.kmeanspp(P, 64, seed=1))
    base, runs = _floor_runs(f, f"c1_{iters}", ("rerun", "rowperm", "colperm0", "colperm1", "colperm2"))
    for v in ("rerun", "rowperm"):
        e = parity.end_of_run(P, base, runs[v])
        assert e["agree"] == 1.0 and e["C_rel"] == 0.0, (v, e)
    floors = [parity.end_of_run(P, base, runs[v]) for v in ("colperm0", "colperm1", "colperm2")]
    assert min(fl["agree"] for fl in floors) < 0.9999       # the reference misses the bar against itself
    lab, C, ine, _ = O.lloyd(P, C0, iters, update_mode=1, frac=O.fixed_frac(float(np.abs(P).max()), len(P)))
    ours = parity.end_of_run(P, base, (lab, C, ine))
    ok, bar = parity.within_floor(ours, floors)
    assert ok, (ours, bar, floors)


def test_reference_noise_floor_config3_sample():
    """Config-3 shape (n = 2e5, d = 128, k = 1024), 3 iterations: the reference with
    permuted coordinates agrees with itself on 99.965-99.976 % of labels; the oracle
    (the engine's arithmetic) agrees with the reference inside that spread."""
    f = golden("ref_floor.npz")
    P = O.make_gmm(200_000, 128, 1024, 3, 5.0, 0.5, 2.0, True)
    C0 = P[np.sort(O.init_random_idx(200_000, 1024, 3))].copy()
    base, runs = _floor_runs(f, "c3s", ("colperm0", "colperm1"))
    floors = [parity.end_of_run(P, base, runs[v]) for v in runs]
    lab, C, ine, _ = O.lloyd(P, C0, 3, update_mode=1, frac=O.fixed_frac(float(np.abs(P).max()), len(P)))
    ours = parity.end_of_run(P, base, (lab, C, ine))
    ok, bar = parity.within_floor(ours, floors)
    assert ok, (ours, bar, floors)


@pytest.mark.parametrize("tag,maker,k,seed", [
    ("c4s", lambda: O.make_sphere(30_000, 768, 4096, 41), 4096, 41),
    ("c5s", lambda: O.make_offset(40_000, 256, 16384, 51, 1e3), 16384, 51)])
def test_reference_noise_floor_iteration0_configs4_5(tag, maker, k, seed):
    """One assignment from the random start on the config-4 and config-5 row samples.
    Unit-sphere rows: the reference agrees with itself under permuted coordinates on every
    row, and so does the oracle (the bar holds).  Offset-1e3 rows (cancellation stress):
    the reference agrees with itself on 99.815 % only, every mismatch an FP32 near-tie
    (gap32 < 1e-5); the oracle agrees with it on 99.855 %, every mismatch a near-tie too."""
    f = golden("ref_floor.npz")
    P = maker()
    C0 = P[np.sort(O.init_random_idx(P.shape[0], k, seed))].copy()
    base = f[f"{tag}_base_labels"].astype(np.int32)
    floor_agree = []
    for v in ("colperm0", "colperm1"):
        s = parity.summary(P, C0, f[f"{tag}_{v}_labels"].astype(np.int32), base)
        assert s["max_gap32"] < 1e-5, (v, s)
        floor_agree.append(s["agree"])
    s = parity.summary(P, C0, O.assign_fp32(P, C0), base)
    assert s["max_gap32"] < 1e-5, s
    assert 1.0 - s["agree"] <= max(1e-4, 1.25 * (1.0 - min(floor_agree))), (s, floor_agree)


@pytest.mark.parametrize("name", ["ref_config3_sample.npz", "ref_offset.npz", "ref_sphere.npz"])
def test_golden_assignment_on_identical_centroids(name):
    g = golden(name)
    n, d, k, seed = int(g["n"]), int(g["d"]), int(g["k"]), int(g["seed"])
    if name == "ref_config3_sample.npz":
        P = O.make_gmm(n, d, k, seed, 5.0, 0.5, 2.0, True)
        rows = np.arange(0, n, 10)   # a 10% sample keeps the CPU time small
    elif name == "ref_offset.npz":
        P = O.make_offset(n, d, k, seed, 1e3)
        rows = np.arange(n)
    else:
        P = O.make_sphere(n, d, k, seed)
        rows = np.arange(n)
    C0 = g["C0"]
    lab = O.assign_fp32(P[rows], C0)
    s = parity.summary(P[rows], C0, lab, g["labels_it0"].astype(np.int32)[rows])
    assert s["agree"] >= 0.995 and s["max_gap32"] < 1e-5, s
    if name != "ref_offset.npz":
        assert s["agree"] >= 0.9999 and s["max_gap64"] < 1e-5, s
    Cn, _, _ = O.update_fp64(P, g["labels_it0"].astype(np.int32), C0)
    assert np.allclose(Cn, g["C_it1"], rtol=2e-6, atol=1e-5)


def test_golden_mpemu_splits_bit_exact():
    g = golden("ref_mpemu.npz")
    rows, cols, lda = (int(x) for x in g["shape"])
    A = g["A"]
    for ns in (1, 2, 3, 4):
        S, _, _ = O.split_bf16(A, rows, cols, lda, ns)
        assert np.array_equal(S, g[f"bf16_split_{ns}"]), ns
    sc = O.autoscale_fp16(A, rows, cols, lda)
    assert np.float32(sc) == g["fp16_scale"]
    for ns in (1, 2, 3):
        S, _, _ = O.split_fp16(A, rows, cols, lda, ns, sc)
        assert np.array_equal(S, g[f"fp16_split_{ns}"]), ns
    assert [tuple(x) for x in g["schedule_3"].reshape(-1, 2)] == O.term_schedule(3, 16)
    assert list(g["multiword_macs"]) == [0, 1, 3, 6, 10]


def test_golden_mpemu_gemm_error_model():
    """The reference's emulated GEMM sits within its error model of the exact
    FP64 product of the same split words (cuBLAS order: tolerance pin)."""
    g = golden("ref_mpemu.npz")
    m, n, k = (int(x) for x in g["gemm_shape"])
    for opa in (0, 1):
        for opb in (0, 1):
            A, B = g[f"gemm_A_{opa}{opb}"], g[f"gemm_B_{opa}{opb}"]
            ra = m if opa == 0 else k
            rb = k if opb == 0 else n
            D = O.gemm_f64(opa, opb, m, n, k, A, ra, B, rb)        # n x m (column major)
            absAB = O.gemm_f64(opa, opb, m, n, k, np.abs(A), ra, np.abs(B), rb)
            for macs, tol in ((1, 2 ** -7), (3, 2 ** -14), (6, 2 ** -20), (9, 2 ** -20)):
                got = g[f"gemm_bf16_{opa}{opb}_{macs}"].reshape(n, m)
                assert np.all(np.abs(got - D) <= tol * absAB + 1e-30), (opa, opb, macs)
            for macs, tol in ((1, 2 ** -9), (3, 2 ** -19)):
                got = g[f"gemm_fp16_{opa}{opb}_{macs}"].reshape(n, m)
                assert np.all(np.abs(got - D) <= tol * absAB + 1e-30), (opa, opb, macs)


def test_kmeanspp_int_definition():
    """The integer-sampled k-means++ (the device seeding's definition): first
    pick floor(u * n / 2^53), no re-picks while weight remains, deterministic,
    and D^2-proportional: far rows are picked far more often than near ones."""
    rng = np.random.default_rng(3)
    P = rng.standard_normal((5000, 16)).astype(np.float32)
    C, idx = O.kmeanspp_int(P, 40, 123)
    C2, idx2 = O.kmeanspp_int(P, 40, 123)
    assert np.array_equal(idx, idx2) and np.array_equal(C, P[idx])
    assert len(set(idx.tolist())) == 40
    # two tight groups plus one far point: the far point is always the second pick
    Q = np.zeros((2001, 4), np.float32)
    Q[1000:2000] += 0.01
    Q[2000] = 100.0
    hits = sum(int(O.kmeanspp_int(Q, 2, s)[1][1] == 2000) for s in range(20))
    first_far = sum(int(O.kmeanspp_int(Q, 1, s)[1][0] == 2000) for s in range(20))
    assert hits >= 19 - first_far


# ------------------------------------------------- update invariants -----

def test_fixed_point_update_is_order_and_shard_independent():
    """The properties the GPU update and the multi-GPU sum rely on, stated on
    the oracle: integer sums do not depend on the order of the rows, and the
    sums of two row shards add up to the sums of the whole, bit for bit."""
    rng = np.random.default_rng(12)
    n, d, k = 5000, 24, 37
    P = (rng.standard_normal((n, d)) * rng.uniform(0.1, 50.0, d)).astype(np.float32)
    C = P[:k].copy()
    lab = rng.integers(0, k, n).astype(np.int32)
    lab[lab == 5] = 6                                       # an empty cluster
    frac = O.fixed_frac(float(np.abs(P).max()), n)
    Cw, m2w, cw, sw = O.update_fixed(P, lab, C, frac)
    perm = rng.permutation(n)
    Cp, m2p, cp, sp = O.update_fixed(P[perm], lab[perm], C, frac)
    assert np.array_equal(sw, sp) and np.array_equal(cw, cp)
    assert np.array_equal(Cw.view(np.uint32), Cp.view(np.uint32))
    assert np.array_equal(m2w.view(np.uint32), m2p.view(np.uint32))
    _, _, c1, s1 = O.update_fixed(P[:1234], lab[:1234], C, frac)
    _, _, c2, s2 = O.update_fixed(P[1234:], lab[1234:], C, frac)
    assert np.array_equal(s1 + s2, sw) and np.array_equal(c1 + c2, cw)
    assert np.array_equal(Cw[5], C[5])                      # the empty cluster keeps its centroid


def test_fp32_assignment_ties_go_to_the_smaller_index():
    """kernels.cu:19-23: on equal FP32 distances the smaller centroid index
    wins, however the duplicates are placed."""
    rng = np.random.default_rng(13)
    P = rng.standard_normal((400, 16)).astype(np.float32)
    base = rng.standard_normal((10, 16)).astype(np.float32)
    C = np.concatenate([base, base[::-1], base])           # every centroid three times
    lab = O.assign_fp32(P, C)
    first = {tuple(r): i for i, r in reversed(list(enumerate(map(tuple, C))))}
    assert all(lab[i] == first[tuple(C[lab[i]])] for i in range(len(P)))
    assert lab.max() < 10
