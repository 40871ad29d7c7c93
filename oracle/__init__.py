"""CPU oracle for the mpkmeans hot path -- TEST INFRASTRUCTURE ONLY.

numpy wrappers over ``oracle/liboracle.so`` (built from ``mpk_oracle.cpp`` by
``oracle/Makefile``).  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU legs use this module, as the checker or as the timed CPU
port; the product library never does.

Reference behaviour restated here is cited file:line in ``mpk_oracle.cpp``.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libmpkref.so"

_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_LL = ctypes.c_longlong
_I = ctypes.c_int
_U64 = ctypes.c_uint64
_D = ctypes.c_double
_F = ctypes.c_float
_VP = ctypes.c_void_p


def build() -> Path:
    """Compile liboracle.so if it is missing or older than its source."""
    src = HERE / "mpk_oracle.cpp"
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        h = ctypes.CDLL(str(LIB_PATH))
        sig = {
            "orc_num_threads": (_I, []),
            "orc_set_threads": (None, [_I]),
            "orc_make_gmm": (None, [_LL, _I, _I, _U64, _D, _D, _D, _I, _VP, _VP, _VP]),
            "orc_make_sphere": (None, [_LL, _I, _I, _U64, _VP, _VP]),
            "orc_make_offset": (None, [_LL, _I, _I, _U64, _D, _VP, _VP]),
            "orc_make_uniform": (None, [_LL, _U64, _I, _f32p]),
            "orc_kmeanspp": (None, [_f32p, _LL, _I, _I, _U64, _f32p]),
            "orc_kmeanspp_int": (None, [_f32p, _LL, _I, _I, _U64, _f32p, _VP]),
            "orc_make_blobs_ref": (None, [_I, _I, _I, _F, _F, ctypes.c_uint, _VP, _VP]),
            "orc_init_random_idx": (None, [_I, _I, ctypes.c_uint, _i32p]),
            "orc_norm2_tree": (_F, [_f32p, _I]),
            "orc_row_norms": (None, [_f32p, _I, _I, _f32p]),
            "orc_dot_warp": (_F, [_f32p, _f32p, _I]),
            "orc_assign_fp32": (None, [_f32p, _LL, _I, _f32p, _I, _i32p, _VP]),
            "orc_dist_fp32": (None, [_f32p, _LL, _I, _f32p, _I, _f32p]),
            "orc_dist64_pairs": (None, [_f32p, _I, _f32p, _i64p, _i32p, _LL, _f64p]),
            "orc_update_fp64": (None, [_f32p, _LL, _I, _i32p, _I, _f32p, _VP, _VP]),
            "orc_update_fixed": (None, [_f32p, _LL, _I, _i32p, _I, _I, _f32p, _VP, _VP, _VP]),
            "orc_inertia": (_D, [_f32p, _LL, _I, _f32p, _i32p]),
            "orc_lloyd": (_I, [_f32p, _LL, _I, _I, _f32p, _i32p, _I, _F, _I, _I, ctypes.POINTER(_D)]),
            "orc_mpk_epsilon": (_D, [_I, _I]),
            "orc_bf16_round": (_F, [_F]),
            "orc_fp16_round": (_F, [_F]),
            "orc_split_bf16": (None, [_f32p, _LL, _LL, _LL, _I, _u16p, _LL, _LL]),
            "orc_split_fp16": (None, [_f32p, _LL, _LL, _LL, _I, _F, _u16p, _LL, _LL]),
            "orc_autoscale_fp16": (_F, [_f32p, _LL, _LL, _LL]),
            "orc_term_schedule": (_I, [_I, _I, _i32p]),
            "orc_gemm_f64": (None, [_I, _I, _LL, _LL, _LL, _f32p, _LL, _f32p, _LL, _f64p, _LL]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def _vp(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------ generators ----

def make_gmm(n, d, ncomp, seed, box, sig_lo, sig_hi, dirichlet, with_truth=False):
    P = np.empty((n, d), np.float32)
    truth = np.empty(n, np.int32) if with_truth else None
    lib().orc_make_gmm(n, d, ncomp, seed, box, sig_lo, sig_hi, int(dirichlet), _vp(P), _vp(truth), None)
    return (P, truth) if with_truth else P


def make_config1(n=100_000, d=32, seed=1):
    """64-component isotropic mixture, means U[-10,10]^d, sigma 1, equal weights."""
    return make_gmm(n, d, 64, seed, 10.0, 1.0, 1.0, False)


def make_config3(n=10_000_000, d=128, seed=3):
    """BASELINE config 3 shape: 1024 components, means U[-5,5]^d, sigma U[0.5,2], Dirichlet(1) weights."""
    return make_gmm(n, d, 1024, seed, 5.0, 0.5, 2.0, True)


def make_sphere(n, d, ncomp, seed):
    P = np.empty((n, d), np.float32)
    lib().orc_make_sphere(n, d, ncomp, seed, _vp(P), None)
    return P


def make_offset(n, d, ncomp, seed, onorm=1e3):
    P = np.empty((n, d), np.float32)
    lib().orc_make_offset(n, d, ncomp, seed, onorm, _vp(P), None)
    return P


def make_uniform(shape, seed, emax=0):
    A = np.empty(shape, np.float32)
    lib().orc_make_uniform(A.size, seed, emax, A.reshape(-1))
    return A


def kmeanspp(P, k, seed):
    n, d = P.shape
    C = np.empty((k, d), np.float32)
    lib().orc_kmeanspp(np.ascontiguousarray(P), n, d, k, seed, C)
    return C


def kmeanspp_int(P, k, seed):
    """k-means++ with exact integer sampling (the GPU's mpkInitKMeansPP definition).
    Returns (C, picked row indices)."""
    n, d = P.shape
    C = np.empty((k, d), np.float32)
    idx = np.empty(k, np.int64)
    lib().orc_kmeanspp_int(np.ascontiguousarray(P, np.float32), n, d, k, seed, C, _vp(idx))
    return C, idx


def make_blobs_ref(n, d, k, std, box, seed):
    P = np.empty((n, d), np.float32)
    L = np.empty(n, np.int32)
    lib().orc_make_blobs_ref(n, d, k, std, box, seed, _vp(P), _vp(L))
    return P, L


def init_random_idx(n, k, seed):
    idx = np.empty(k, np.int32)
    lib().orc_init_random_idx(n, k, seed, idx)
    return idx


# ------------------------------------------------------------ k-means -------

def row_norms(C):
    k, d = C.shape
    out = np.empty(k, np.float32)
    lib().orc_row_norms(np.ascontiguousarray(C), k, d, out)
    return out


def assign_fp32(P, C, with_dist=False):
    n, d = P.shape
    k = C.shape[0]
    lab = np.empty(n, np.int32)
    db = np.empty(n, np.float32) if with_dist else None
    lib().orc_assign_fp32(np.ascontiguousarray(P), n, d, np.ascontiguousarray(C), k, lab, _vp(db))
    return (lab, db) if with_dist else lab


def dist_fp32(P, C):
    n, d = P.shape
    k = C.shape[0]
    D = np.empty((n, k), np.float32)
    lib().orc_dist_fp32(np.ascontiguousarray(P), n, d, np.ascontiguousarray(C), k, D)
    return D


def dist64_pairs(P, C, rows, cols):
    rows = np.ascontiguousarray(rows, np.int64)
    cols = np.ascontiguousarray(cols, np.int32)
    out = np.empty(len(rows), np.float64)
    lib().orc_dist64_pairs(np.ascontiguousarray(P), P.shape[1], np.ascontiguousarray(C), rows, cols, len(rows), out)
    return out


def update_fp64(P, labels, C):
    """Reference FP64 update; returns (C_new, moved2, counts)."""
    n, d = P.shape
    k = C.shape[0]
    Cn = np.array(C, np.float32, copy=True)
    m2 = np.empty(k, np.float32)
    cnt = np.empty(k, np.int64)
    lib().orc_update_fp64(np.ascontiguousarray(P), n, d, np.ascontiguousarray(labels, np.int32), k, Cn,
                          _vp(m2), _vp(cnt))
    return Cn, m2, cnt


def update_fixed(P, labels, C, frac):
    """The library's fixed-point update; returns (C_new, moved2, counts, sums int64)."""
    n, d = P.shape
    k = C.shape[0]
    Cn = np.array(C, np.float32, copy=True)
    m2 = np.empty(k, np.float32)
    cnt = np.empty(k, np.int64)
    S = np.empty((k, d), np.int64)
    lib().orc_update_fixed(np.ascontiguousarray(P), n, d, np.ascontiguousarray(labels, np.int32), k, frac, Cn,
                           _vp(m2), _vp(cnt), _vp(S))
    return Cn, m2, cnt, S


def inertia(P, C, labels):
    n, d = P.shape
    return lib().orc_inertia(np.ascontiguousarray(P), n, d, np.ascontiguousarray(C),
                             np.ascontiguousarray(labels, np.int32))


def lloyd(P, C0, max_iter, tol=0.0, update_mode=0, frac=0):
    """mpkMeansFP32 on the CPU.  update_mode 0: reference FP64; 1: fixed point."""
    n, d = P.shape
    k = C0.shape[0]
    C = np.array(C0, np.float32, copy=True)
    lab = np.empty(n, np.int32)
    ine = ctypes.c_double()
    it = lib().orc_lloyd(np.ascontiguousarray(P), n, d, k, C, lab, max_iter, tol, update_mode, frac, ctypes.byref(ine))
    return lab, C, ine.value, it


def fixed_frac(pmax: float, n_total: int) -> int:
    """Fractional bits of the fixed-point update (the library's k_set_scale rule)."""
    if pmax > 0 and np.isfinite(pmax):
        _, E = np.frexp(np.float32(pmax))
        E = int(E)
    else:
        E = 0
    lg = 0
    while (1 << lg) < n_total and lg < 62:
        lg += 1
    return min(62 - E - lg, 100)


def mpk_epsilon(d, accum_fp16=0):
    return lib().orc_mpk_epsilon(d, accum_fp16)


# ------------------------------------------------------ split GEMM ----------

def split_lds(rows):
    return (rows + 7) // 8 * 8


def split_bf16(A_colmajor, rows, cols, lda, nsplits):
    lds = split_lds(rows)
    stride = lds * cols
    S = np.zeros(stride * nsplits, np.uint16)
    lib().orc_split_bf16(np.ascontiguousarray(A_colmajor, np.float32).reshape(-1), lda, rows, cols, nsplits, S, lds,
                         stride)
    return S, lds, stride


def split_fp16(A_colmajor, rows, cols, lda, nsplits, scale):
    lds = split_lds(rows)
    stride = lds * cols
    S = np.zeros(stride * nsplits, np.uint16)
    lib().orc_split_fp16(np.ascontiguousarray(A_colmajor, np.float32).reshape(-1), lda, rows, cols, nsplits, scale, S,
                         lds, stride)
    return S, lds, stride


def autoscale_fp16(A_colmajor, rows, cols, lda):
    return lib().orc_autoscale_fp16(np.ascontiguousarray(A_colmajor, np.float32).reshape(-1), lda, rows, cols)


def term_schedule(nsplits, max_terms):
    ij = np.zeros(2 * max(1, max_terms), np.int32)
    n = lib().orc_term_schedule(nsplits, max_terms, ij)
    return [(int(ij[2 * t]), int(ij[2 * t + 1])) for t in range(n)]


def gemm_f64(transA, transB, m, n, k, A, lda, B, ldb):
    D = np.zeros((n, m), np.float64)  # column major m x n stored as n rows of m
    lib().orc_gemm_f64(int(transA), int(transB), m, n, k, np.ascontiguousarray(A, np.float32).reshape(-1), lda,
                       np.ascontiguousarray(B, np.float32).reshape(-1), ldb, D.reshape(-1), m)
    return D


def bf16_to_f32(u16):
    return (np.asarray(u16, np.uint32) << 16).view(np.float32)


def fp16_to_f32(u16):
    return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)
