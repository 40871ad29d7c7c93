"""Generate golden fixtures from the reference implementation itself.

Runs ``oracle/_ref/libmpkref.so`` -- CornellHPC/mpkmeans' own k-means and
split-GEMM sources compiled by ``oracle/build_ref.sh`` -- on a GPU, on seeded
inputs that the CPU oracle regenerates bit for bit, and writes the outputs to
``tests/golden/*.npz``.  The CPU test suite then pins the oracle against these
files (tolerance pins where the reference's arithmetic is cuBLAS's, exact pins
where it is its own code).

Usage (GPU machine, from the repository root):
    python tests/golden/make_golden.py [outdir] [--only kmeans|mpemu|large|floor]

The ``large`` cases (configs 4 and 5 shapes on row samples) also run this
repository's engine (mpkmeans_b200) for two Lloyd iterations and then let the
reference assign against those centroids -- the reference's own per-iteration
check, fed the engine's centroids.
"""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle as O  # noqa: E402
from mpkmeans_b200 import mpkParams, mpkStats  # noqa: E402  (struct layouts only)

_args = [a for a in sys.argv[1:] if not a.startswith("--")]
ONLY = sys.argv[sys.argv.index("--only") + 1] if "--only" in sys.argv else None
if ONLY in _args:
    _args.remove(ONLY)
OUT = Path(_args[0]) if _args else Path(__file__).resolve().parent

ref = ctypes.CDLL(str(O.REF_LIB_PATH))
VP = ctypes.c_void_p
I64 = ctypes.c_int64
for name in ("mpkMeansFP32", "mpkMeansMixed"):
    getattr(ref, name).argtypes = [VP, VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, VP, VP,
                                   ctypes.POINTER(mpkParams), ctypes.POINTER(mpkStats)]
    getattr(ref, name).restype = ctypes.c_int
ref.mpkParamsInit.argtypes = [ctypes.POINTER(mpkParams)]
ref.mpkInitRandomPoints.argtypes = [VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_uint, VP]
ref.mpkShiftNonNegative.argtypes = [VP, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]
ref.mpemuSplitBF16.argtypes = [VP, I64, I64, I64, ctypes.c_int, VP, I64, I64, VP]
ref.mpemuSplitFP16.argtypes = [VP, I64, I64, I64, ctypes.c_int, ctypes.c_float, VP, I64, I64, VP]
ref.mpemuAutoScaleFP16.argtypes = [VP, I64, I64, I64, ctypes.POINTER(ctypes.c_float), VP]
ref.mpemuGemmEmulated.argtypes = [VP, ctypes.c_int, ctypes.c_int, I64, I64, I64, ctypes.c_float, VP, I64, I64,
                                  VP, I64, I64, ctypes.c_int, ctypes.c_int, ctypes.c_float, VP, I64]
ref.mpemuGemmMultiword.argtypes = [VP, ctypes.c_int, ctypes.c_int, I64, I64, I64, ctypes.c_float, VP, I64, I64,
                                   ctypes.c_float, VP, I64, I64, ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, VP, I64]
ref.mpemuTermSchedule.argtypes = [ctypes.c_int, ctypes.c_int, VP]
ref.mpemuMultiwordMacs.argtypes = [ctypes.c_int]

dev = torch.device("cuda:0")
blas = torch.cuda.current_blas_handle()


def params(**kw):
    p = mpkParams()
    ref.mpkParamsInit(ctypes.byref(p))
    for k_, v in kw.items():
        setattr(p, k_, v)
    return p


def run(fn, P, C0, max_iter, **kw):
    n, d = P.shape
    k = C0.shape[0]
    dP = torch.from_numpy(P).to(dev)
    dC = torch.from_numpy(C0).to(dev)
    dA = torch.empty(n, dtype=torch.int32, device=dev)
    st = mpkStats()
    rc = getattr(ref, fn)(blas, dP.data_ptr(), n, d, k, dC.data_ptr(), dA.data_ptr(),
                          ctypes.byref(params(max_iter=max_iter, **kw)), ctypes.byref(st))
    torch.cuda.synchronize()
    assert rc == 0, (fn, rc)
    return dA.cpu().numpy(), dC.cpu().numpy(), st


def trajectory(P, C0, iters):
    """Chain max_iter=1 calls: labels_t = assign(C_t), C_{t+1} = update."""
    labs, cents = [], []
    C = C0.copy()
    for _ in range(iters):
        lab, C, _ = run("mpkMeansFP32", P, C, 1)
        labs.append(lab)
        cents.append(C)
    return np.stack(labs), np.stack(cents)


def lab_dtype(k):
    return np.int8 if k <= 127 else np.int16


def kmeans_cases():
    # (a) mpkMakeBlobs data (reference generator) + mpkInitRandomPoints (reference init)
    n, d, k, seed = 4096, 32, 16, 5
    P, _ = O.make_blobs_ref(n, d, k, 1.0, 10.0, seed)
    dP = torch.from_numpy(P).to(dev)
    dC = torch.empty((k, d), dtype=torch.float32, device=dev)
    assert ref.mpkInitRandomPoints(dP.data_ptr(), n, d, k, seed, dC.data_ptr()) == 0
    C0 = dC.cpu().numpy()
    lab, C, st = run("mpkMeansFP32", P, C0, 10)
    tl, tc = trajectory(P, C0, 4)
    # the mixed driver on the reference's shifted frame, verify on (MPK_STATS build)
    Ps = P.copy()
    dPs = torch.from_numpy(Ps).to(dev)
    shift = ctypes.c_float()
    assert ref.mpkShiftNonNegative(dPs.data_ptr(), n, d, ctypes.byref(shift)) == 0
    Ps = dPs.cpu().numpy()
    C0s = C0 + np.float32(shift.value)
    mlab, mC, mst = run("mpkMeansMixed", Ps, C0s, 10, verify=1)
    np.savez_compressed(OUT / "ref_blobs.npz", n=n, d=d, k=k, seed=seed, C0=C0,
                        labels=lab.astype(lab_dtype(k)), C=C, inertia=st.inertia, iters=st.iters,
                        traj_labels=tl.astype(lab_dtype(k)), traj_C=tc,
                        shift=shift.value, mixed_labels=mlab.astype(lab_dtype(k)), mixed_C=mC,
                        mixed_inertia=mst.inertia, mixed_verify_excluded_best=mst.verify_excluded_best,
                        mixed_hp_update=mst.hp_update)
    print("ref_blobs", st.inertia, mst.inertia, mst.verify_excluded_best)

    # (b) BASELINE config 1: n=1e5, d=32, k=64, k-means++ from the same seed, 20 iterations
    P = O.make_config1(100_000, 32, seed=1)
    C0 = O.kmeanspp(P, 64, seed=1)
    lab, C, st = run("mpkMeansFP32", P, C0, 20)
    lab1, C1, _ = run("mpkMeansFP32", P, C0, 1)
    tl, tc = trajectory(P, C0, 20)
    np.savez_compressed(OUT / "ref_config1.npz", n=100_000, d=32, k=64, seed=1, C0=C0,
                        labels=lab.astype(np.int8), C=C, inertia=st.inertia,
                        labels_it0=lab1.astype(np.int8), C_it1=C1,
                        traj_labels=tl.astype(np.int8), traj_C=tc)
    print("ref_config1", st.inertia)

    # (c) config-3 shape sample: n=200k, d=128, k=1024, one assignment + update and 3 iterations
    P = O.make_gmm(200_000, 128, 1024, 3, 5.0, 0.5, 2.0, True)
    idx = O.init_random_idx(200_000, 1024, 3)
    C0 = P[np.sort(idx)].copy()
    lab1, C1, _ = run("mpkMeansFP32", P, C0, 1)
    lab3, C3, st3 = run("mpkMeansFP32", P, C0, 3)
    np.savez_compressed(OUT / "ref_config3_sample.npz", n=200_000, d=128, k=1024, seed=3, C0=C0,
                        labels_it0=lab1.astype(np.int16), C_it1=C1, labels_it2=lab3.astype(np.int16), C_it3=C3,
                        inertia_it3=st3.inertia)
    print("ref_config3_sample", st3.inertia)

    # (d) cancellation and unit-sphere shapes, small
    P = O.make_offset(20_000, 64, 64, 5, 1e3)
    C0 = P[np.sort(O.init_random_idx(20_000, 64, 5))].copy()
    lab, C, st = run("mpkMeansFP32", P, C0, 5)
    lab1, C1, _ = run("mpkMeansFP32", P, C0, 1)
    np.savez_compressed(OUT / "ref_offset.npz", n=20_000, d=64, k=64, seed=5, C0=C0, labels=lab.astype(np.int8),
                        C=C, inertia=st.inertia, labels_it0=lab1.astype(np.int8), C_it1=C1)
    P = O.make_sphere(20_000, 96, 128, 4)
    C0 = P[np.sort(O.init_random_idx(20_000, 128, 4))].copy()
    lab, C, st = run("mpkMeansFP32", P, C0, 5)
    lab1, C1, _ = run("mpkMeansFP32", P, C0, 1)
    np.savez_compressed(OUT / "ref_sphere.npz", n=20_000, d=96, k=128, seed=4, C0=C0, labels=lab.astype(np.int16),
                        C=C, inertia=st.inertia, labels_it0=lab1.astype(np.int16), C_it1=C1)
    print("ref_offset/sphere done")


def mpemu_cases():
    out = {}
    # splits of a 96 x 80 column-major matrix (lda 101), seed 9, values u*2^e, e in [-8, 8]
    rows, cols, lda = 96, 80, 101
    A = O.make_uniform((cols, lda), 9, emax=8)          # column-major storage: cols x lda
    dA = torch.from_numpy(A).to(dev)
    lds = (rows + 7) // 8 * 8
    stride = lds * cols
    for ns in (1, 2, 3, 4):
        dS = torch.zeros(stride * ns, dtype=torch.int16, device=dev)
        assert ref.mpemuSplitBF16(dA.data_ptr(), lda, rows, cols, ns, dS.data_ptr(), lds, stride, None) == 0
        torch.cuda.synchronize()
        out[f"bf16_split_{ns}"] = dS.cpu().numpy().view(np.uint16)
    sc = ctypes.c_float()
    assert ref.mpemuAutoScaleFP16(dA.data_ptr(), lda, rows, cols, ctypes.byref(sc), None) == 0
    out["fp16_scale"] = np.float32(sc.value)
    for ns in (1, 2, 3):
        dS = torch.zeros(stride * ns, dtype=torch.int16, device=dev)
        assert ref.mpemuSplitFP16(dA.data_ptr(), lda, rows, cols, ns, sc, dS.data_ptr(), lds, stride, None) == 0
        torch.cuda.synchronize()
        out[f"fp16_split_{ns}"] = dS.cpu().numpy().view(np.uint16)
    out["A"] = A
    out["shape"] = np.array([rows, cols, lda])
    t = np.zeros(32, np.int32)
    out["schedule_3"] = t[:2 * ref.mpemuTermSchedule(3, 16, t.ctypes.data_as(VP))].copy()
    out["multiword_macs"] = np.array([ref.mpemuMultiwordMacs(p) for p in range(0, 5)], np.int32)

    # emulated GEMM, m=96, n=72, k=80, every op combination, a few MAC counts
    m, n, kk = 96, 72, 80
    for opa in (0, 1):
        for opb in (0, 1):
            ra, ca = (m, kk) if opa == 0 else (kk, m)
            rb, cb = (kk, n) if opb == 0 else (n, kk)
            Am = O.make_uniform((ca, ra), 100 + 2 * opa + opb)
            Bm = O.make_uniform((cb, rb), 200 + 2 * opa + opb)
            out[f"gemm_A_{opa}{opb}"] = Am
            out[f"gemm_B_{opa}{opb}"] = Bm
            dAm = torch.from_numpy(Am).to(dev)
            dBm = torch.from_numpy(Bm).to(dev)
            la, lb = (ra + 7) // 8 * 8, (rb + 7) // 8 * 8
            sa, sb = la * ca, lb * cb
            dSA = torch.zeros(sa * 3, dtype=torch.int16, device=dev)
            dSB = torch.zeros(sb * 3, dtype=torch.int16, device=dev)
            assert ref.mpemuSplitBF16(dAm.data_ptr(), ra, ra, ca, 3, dSA.data_ptr(), la, sa, None) == 0
            assert ref.mpemuSplitBF16(dBm.data_ptr(), rb, rb, cb, 3, dSB.data_ptr(), lb, sb, None) == 0
            for macs in (1, 3, 6, 9):
                dC = torch.zeros(n * m, dtype=torch.float32, device=dev)
                assert ref.mpemuGemmEmulated(blas, opa, opb, m, n, kk, 1.0, dSA.data_ptr(), la, sa, dSB.data_ptr(),
                                             lb, sb, 3, macs, 0.0, dC.data_ptr(), m) == 0
                torch.cuda.synchronize()
                out[f"gemm_bf16_{opa}{opb}_{macs}"] = dC.cpu().numpy()
            sA, sB = ctypes.c_float(), ctypes.c_float()
            assert ref.mpemuAutoScaleFP16(dAm.data_ptr(), ra, ra, ca, ctypes.byref(sA), None) == 0
            assert ref.mpemuAutoScaleFP16(dBm.data_ptr(), rb, rb, cb, ctypes.byref(sB), None) == 0
            assert ref.mpemuSplitFP16(dAm.data_ptr(), ra, ra, ca, 2, sA, dSA.data_ptr(), la, sa, None) == 0
            assert ref.mpemuSplitFP16(dBm.data_ptr(), rb, rb, cb, 2, sB, dSB.data_ptr(), lb, sb, None) == 0
            for macs in (1, 3):
                dC = torch.zeros(n * m, dtype=torch.float32, device=dev)
                assert ref.mpemuGemmMultiword(blas, opa, opb, m, n, kk, 1.0, dSA.data_ptr(), la, sa, sA,
                                              dSB.data_ptr(), lb, sb, sB, 2, macs, 0.0, dC.data_ptr(), m) == 0
                torch.cuda.synchronize()
                out[f"gemm_fp16_{opa}{opb}_{macs}"] = dC.cpu().numpy()
    out["gemm_shape"] = np.array([m, n, kk])
    np.savez_compressed(OUT / "ref_mpemu.npz", **out)
    print("ref_mpemu done")


def large_cases():
    """Configs 4 and 5 geometries on row samples: the reference's FP32 assignment (a) against random
    start centroids and (b) against the centroids after two iterations of this engine."""
    import hashlib
    import mpkmeans_b200 as M
    for name, P, k, seed in (
            ("ref_config4_sample", O.make_sphere(30_000, 768, 4096, 41), 4096, 41),
            ("ref_config5_sample", O.make_offset(40_000, 256, 16384, 51, 1e3), 16384, 51)):
        n, d = P.shape
        idx = np.sort(O.init_random_idx(n, k, seed))
        C0 = P[idx].copy()
        lab0, _, _ = run("mpkMeansFP32", P, C0, 1)
        dP = torch.from_numpy(P).to(dev)
        dC = torch.from_numpy(C0).to(dev)
        lab = torch.empty(n, dtype=torch.int32, device=dev)
        M.means_mixed(dP, dC, lab, M.params_init(max_iter=2))
        C2 = dC.cpu().numpy()
        lab2, _, _ = run("mpkMeansFP32", P, C2, 1)
        np.savez_compressed(OUT / f"{name}.npz", n=n, d=d, k=k, seed=seed, labels_it0=lab0.astype(np.int16),
                            labels_c2=lab2.astype(np.int16),
                            c2_sha256=np.frombuffer(hashlib.sha256(C2.tobytes()).digest(), np.uint8))
        print(name, "done")


def _colperm_run(P, C0, iters, q):
    """The reference on P and C0 with their coordinates permuted by q (the same points and
    centroids; only the order of every FP32 dot product changes), mapped back."""
    lab, C, st = run("mpkMeansFP32", np.ascontiguousarray(P[:, q]), np.ascontiguousarray(C0[:, q]), iters)
    return lab, np.ascontiguousarray(C[:, np.argsort(q)]), st.inertia


def floor_cases():
    """The reference against itself: how far two of its own FP32 runs on the same
    problem drift apart.  Each variant changes nothing a k-means answer depends on:
    `rerun` repeats the call (its FP64-atomic update sums in arrival order), `rowperm`
    permutes the rows (labels mapped back), `colperm*` permutes the coordinates of the
    points and start centroids alike (every FP32 dot is summed in another order; the
    centroids are mapped back).  The agreement between these runs is the noise floor
    that end-of-run label and centroid agreement with any other FP32 implementation
    is read against."""
    rng = np.random.default_rng(2024)
    out = {}

    def store(prefix, lab, C, ine, dt):
        out[f"{prefix}_labels"] = lab.astype(dt)
        if C is not None:
            out[f"{prefix}_C"] = C
        if ine is not None:
            out[f"{prefix}_inertia"] = np.float64(ine)

    # n = 1e5, d = 32, k = 64, k-means++ from seed 1, 20 iterations (and 100)
    P = O.make_config1(100_000, 32, seed=1)
    C0 = O.kmeanspp(P, 64, seed=1)
    n, d = P.shape
    out["c1_C0"] = C0
    for iters in (20, 100):
        lab, C, st = run("mpkMeansFP32", P, C0, iters)
        store(f"c1_{iters}_base", lab, C, st.inertia, np.int8)
        lab, C, st = run("mpkMeansFP32", P, C0, iters)
        store(f"c1_{iters}_rerun", lab, C, st.inertia, np.int8)
        perm = rng.permutation(n)
        inv = np.empty(n, np.int64)
        inv[perm] = np.arange(n)
        lab, C, st = run("mpkMeansFP32", np.ascontiguousarray(P[perm]), C0, iters)
        store(f"c1_{iters}_rowperm", lab[inv], C, st.inertia, np.int8)
        for s in range(3):
            lab, C, ine = _colperm_run(P, C0, iters, rng.permutation(d))
            store(f"c1_{iters}_colperm{s}", lab, C, ine, np.int8)
        print("floor config1", iters, "done")

    # config-3 shape sample (n = 2e5, d = 128, k = 1024), 3 iterations
    P = O.make_gmm(200_000, 128, 1024, 3, 5.0, 0.5, 2.0, True)
    C0 = P[np.sort(O.init_random_idx(200_000, 1024, 3))].copy()
    lab, C, st = run("mpkMeansFP32", P, C0, 3)
    store("c3s_base", lab, C, st.inertia, np.int16)
    for s in range(2):
        lab, C, ine = _colperm_run(P, C0, 3, rng.permutation(128))
        store(f"c3s_colperm{s}", lab, C, ine, np.int16)

    # configs 4 and 5 geometries on the row samples of large_cases: iteration 0 (one assignment)
    for tag, P, k, seed in (("c4s", O.make_sphere(30_000, 768, 4096, 41), 4096, 41),
                            ("c5s", O.make_offset(40_000, 256, 16384, 51, 1e3), 16384, 51)):
        n, d = P.shape
        C0 = P[np.sort(O.init_random_idx(n, k, seed))].copy()
        lab, _, _ = run("mpkMeansFP32", P, C0, 1)
        store(f"{tag}_base", lab, None, None, np.int16)
        for s in range(2):
            lab, _, _ = _colperm_run(P, C0, 1, rng.permutation(d))
            store(f"{tag}_colperm{s}", lab, None, None, np.int16)
        print("floor", tag, "done")
    np.savez_compressed(OUT / "ref_floor.npz", **out)
    print("ref_floor done")


if __name__ == "__main__":
    OUT.mkdir(parents=True, exist_ok=True)
    if ONLY in (None, "kmeans"):
        kmeans_cases()
    if ONLY in (None, "mpemu"):
        mpemu_cases()
    if ONLY in (None, "large"):
        large_cases()
    if ONLY in (None, "floor"):
        floor_cases()
