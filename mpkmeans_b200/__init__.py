"""mpkmeans_b200 -- B200-native mixed-precision k-means.

The product is the C-ABI library ``libmpkmeans_b200.so`` (declared in
``include/mpkmeans.h``).  This module is its host-side mirror: ctypes
structures with the exact layout of the reference's ``mpkParams`` /
``mpkStats`` (``kmeans/include/mpkmeans/mpkmeans.h:54-181``), the same
function names, argument meaning and status codes, plus an ``Engine`` class
for callers that drive the iteration themselves (one process per GPU with a
collective between steps).

Device memory is passed as integer addresses; the helpers accept CUDA torch
tensors and use their ``data_ptr()``.  There is no fallback: if the compiled
library is missing, importing the bindings raises ``MpkLibraryError``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libmpkmeans_b200.so"

MPK_OK, MPK_ERR_CUDA, MPK_ERR_CUBLAS, MPK_ERR_CUSPARSE, MPK_ERR_INVALID, MPK_ERR_ALLOC = range(6)
MPK_ACCUM_FP32, MPK_ACCUM_FP16 = 0, 1
MPK_MAX_HIST = 256
STATUS_NAMES = {0: "MPK_OK", 1: "MPK_ERR_CUDA", 2: "MPK_ERR_CUBLAS", 3: "MPK_ERR_CUSPARSE",
                4: "MPK_ERR_INVALID", 5: "MPK_ERR_ALLOC"}


class MpkLibraryError(ImportError):
    """The compiled library is absent or does not load."""


class MpkError(RuntimeError):
    """A library call returned a status other than MPK_OK."""

    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} returned {STATUS_NAMES.get(status, status)}")
        self.status = status


class mpemuBatchWorkspace(ctypes.Structure):
    """mpemuBatchWorkspace_t (include/mpemu.h)."""
    _fields_ = [("tmp", ctypes.c_void_p), ("ldt", ctypes.c_int64), ("strideT", ctypes.c_int64),
                ("aptr", ctypes.c_void_p), ("bptr", ctypes.c_void_p), ("cptr", ctypes.c_void_p),
                ("bins", ctypes.c_void_p), ("capacity", ctypes.c_int), ("planned", ctypes.c_int),
                ("elemBytes", ctypes.c_int)]


class mpemuWorkspace(ctypes.Structure):
    """mpemuBf16Workspace_t / mpemuFp16Workspace_t (same layout)."""
    _fields_ = [("sA", ctypes.c_void_p), ("ldA", ctypes.c_int64), ("strideA", ctypes.c_int64),
                ("sB", ctypes.c_void_p), ("ldB", ctypes.c_int64), ("strideB", ctypes.c_int64),
                ("nsplits", ctypes.c_int)]


class mpkParams(ctypes.Structure):
    _fields_ = [("max_iter", ctypes.c_int), ("tol", ctypes.c_float), ("use_cond3", ctypes.c_int),
                ("use_cond6", ctypes.c_int), ("cascade", ctypes.c_int), ("accum", ctypes.c_int),
                ("mw_macs", ctypes.c_int), ("mw_gather_frac", ctypes.c_float), ("cuvs_batch", ctypes.c_int),
                ("rt_theta", ctypes.c_float), ("verify", ctypes.c_int), ("verbose", ctypes.c_int)]


class mpkStats(ctypes.Structure):
    _fields_ = [("iters", ctypes.c_int), ("inertia", ctypes.c_double),
                ("hp_baseline", ctypes.c_longlong), ("hp_reference", ctypes.c_longlong),
                ("hp_update", ctypes.c_longlong), ("mw_products", ctypes.c_longlong),
                ("mw_refine_rows", ctypes.c_longlong), ("tested", ctypes.c_longlong),
                ("excl_cond3", ctypes.c_longlong), ("excl_cond6", ctypes.c_longlong),
                ("excl_both", ctypes.c_longlong), ("n_hist", ctypes.c_int),
                ("hist_survivors", ctypes.c_longlong * MPK_MAX_HIST),
                ("verify_excluded_best", ctypes.c_longlong), ("verify_label_diff", ctypes.c_longlong),
                ("verify_excess", ctypes.c_double), ("stats_built", ctypes.c_int),
                ("t_total_ms", ctypes.c_double), ("t_dist_ms", ctypes.c_double), ("t_prep_ms", ctypes.c_double),
                ("t_gemm_lo_ms", ctypes.c_double), ("t_argmin_ms", ctypes.c_double),
                ("t_hp_update_ms", ctypes.c_double), ("t_assign_ms", ctypes.c_double),
                ("t_update_ms", ctypes.c_double)]


_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_F = ctypes.c_float
_D = ctypes.c_double
_I64 = ctypes.c_int64
_PARAMS = ctypes.POINTER(mpkParams)
_STATS = ctypes.POINTER(mpkStats)

# name -> (restype, argtypes).  Every symbol include/mpkmeans.h and
# include/mpemu.h declare is listed here; tests check the library exports all.
SIGNATURES = {
    "mpkParamsInit": (None, [_PARAMS]),
    "mpkEpsilon": (_D, [_I, _I]),
    "mpkMultiwordEpsilon": (_D, [_I, _I]),
    "mpkShiftNonNegative": (_I, [_P, _I, _I, ctypes.POINTER(_F)]),
    "mpkStandardize": (_I, [_P, _I, _I]),
    "mpkShiftCentroids": (_I, [_P, _I, _I, _F]),
    "mpkMeansMixed": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkMeansFP32": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkMeansMultiword": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkMeansBaselineRT": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkHaveCuvs": (_I, []),
    "mpkMeansCuvs": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkLoadBin": (_I, [ctypes.c_char_p, _I, _LL, ctypes.POINTER(_I), ctypes.POINTER(ctypes.POINTER(_F))]),
    "mpkLoadLibsvm": (_I, [ctypes.c_char_p, ctypes.POINTER(_I), ctypes.POINTER(_I),
                           ctypes.POINTER(ctypes.POINTER(_F)), ctypes.POINTER(ctypes.POINTER(_I)),
                           ctypes.POINTER(_I)]),
    "mpkMakeBlobs": (None, [_I, _I, _I, _F, _F, ctypes.c_uint, _P, _P]),
    "mpkInitRandomPoints": (_I, [_P, _I, _I, _I, ctypes.c_uint, _P]),
    "mpkInitKMeansPP": (_I, [_P, _I, _I, _I, ctypes.c_ulonglong, _P]),
    "mpkTrimMemoryPool": (_I, [_I]),
    "mpkAssign": (_I, [_P, _P, _I, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkUpdate": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "mpkMeansMixedMG": (_I, [_I, _P, _P, _P, _I, _I, _P, _P, _PARAMS, _STATS]),
    "mpkUpdateNoAlloc": (_I, [_P, _P, _I, _I, _I, _P, _P, _P]),
    "mpkEngineCreate": (_I, [ctypes.POINTER(_P), _P, _LL, _I, _I, _P, _F, _LL, _P]),
    "mpkEngineDestroy": (_I, [_P]),
    "mpkEngineAssign": (_I, [_P, _P, _P, _I]),
    "mpkEngineAccumulate": (_I, [_P, _P, _P]),
    "mpkEngineFinalize": (_I, [_P, _P, _P, _P]),
    "mpkEngineIterate": (_I, [_P, _P, _P, _P, _I, _I]),
    "mpkEngineStep": (_I, [_P, _P, _P, _P, _I]),
    "mpkPeerCreate": (_I, [ctypes.POINTER(_P), _I, _I, _I, _I]),
    "mpkPeerExportHandle": (_I, [_P, _P]),
    "mpkPeerLocalBase": (_I, [_P, ctypes.POINTER(_P)]),
    "mpkPeerConnect": (_I, [_P, _P, _P, _P]),
    "mpkPeerSums": (_P, [_P]),
    "mpkPeerCombine": (_I, [_P, _P, _P, _P]),
    "mpkPeerDestroy": (_I, [_P]),
    "mpkDebugFailAlloc": (_I, [_I]),
    "mpkDebugMGFailNextWait": (_I, []),
    "mpkEngineInertia": (_I, [_P, _P, _P, ctypes.POINTER(_D)]),
    "mpkEngineFracBits": (_I, [_P]),
    "mpkEngineCounters": (_I, [_P, ctypes.POINTER(_LL), ctypes.POINTER(_LL), ctypes.POINTER(_LL),
                               ctypes.POINTER(_I)]),
    "mpkEngineSumsLength": (_LL, [_P]),
    "mpkDebugSetAssignTrace": (_I, [_P, _P]),
    # include/mpemu.h
    "mpemuStatusString": (ctypes.c_char_p, [_I]),
    "mpemuSplitLd": (ctypes.c_int64, [ctypes.c_int64]),
    "mpemuSplitStride": (ctypes.c_int64, [ctypes.c_int64, ctypes.c_int64]),
    "mpemuSplitBytes": (ctypes.c_size_t, [ctypes.c_int64, ctypes.c_int64, _I]),
    "mpemuSplitBF16": (_I, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I, _P, ctypes.c_int64,
                            ctypes.c_int64, _P]),
    "mpemuGemmBF16": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P, ctypes.c_int64, _P,
                           ctypes.c_int64, _F, _P, ctypes.c_int64]),
    "mpemuTermCount": (_I, [_I]),
    "mpemuTermSchedule": (_I, [_I, _I, _P]),
    "mpemuGemmEmulatedRange": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P,
                                    ctypes.c_int64, ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int64, _I, _I, _I,
                                    _F, _P, ctypes.c_int64]),
    "mpemuGemmEmulated": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P, ctypes.c_int64,
                               ctypes.c_int64, _P, ctypes.c_int64, ctypes.c_int64, _I, _I, _F, _P, ctypes.c_int64]),
    "mpemuMultiwordMacs": (_I, [_I]),
    "mpemuSplitFP16": (_I, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I, _F, _P, ctypes.c_int64,
                            ctypes.c_int64, _P]),
    "mpemuAutoScaleFP16": (_I, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(_F), _P]),
    "mpemuCheckSplitFP16": (_I, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I, _F, _P, ctypes.c_int64,
                                 ctypes.c_int64, _P, _P]),
    "mpemuGemmFP16": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P, ctypes.c_int64, _P,
                           ctypes.c_int64, _F, _P, ctypes.c_int64]),
    "mpemuGemmMultiwordRange": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P,
                                     ctypes.c_int64, ctypes.c_int64, _F, _P, ctypes.c_int64, ctypes.c_int64, _F, _I,
                                     _I, _I, _F, _P, ctypes.c_int64]),
    "mpemuGemmMultiword": (_I, [_P, _I, _I, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _F, _P, ctypes.c_int64,
                                ctypes.c_int64, _F, _P, ctypes.c_int64, ctypes.c_int64, _F, _I, _I, _F, _P,
                                ctypes.c_int64]),
    "mpemuContextCreate": (_I, [ctypes.POINTER(_P)]),
    "mpemuContextDestroy": (_I, [_P]),
    "mpemuContextReserve": (_I, [_P, ctypes.c_size_t]),
    "mpemuContextCapacity": (ctypes.c_size_t, [_P]),
    "mpemuContextBase": (_P, [_P]),
    "mpemuContextAllocCount": (_I, [_P]),
    "mpemuBf16WorkspaceBytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I]),
    "mpemuFp16WorkspaceBytes": (ctypes.c_size_t, [_I64, _I64, _I64, _I]),
    "mpemuBf16WorkspaceInit": (_I, [_P, _I64, _I64, _I64, _I, _P]),
    "mpemuFp16WorkspaceInit": (_I, [_P, _I64, _I64, _I64, _I, _P]),
    "mpemuBatchWorkspaceBytes": (ctypes.c_size_t, [_I64, _I64, _I, _I]),
    "mpemuBatchWorkspaceInit": (_I, [_P, _I64, _I64, _I, _I, ctypes.c_size_t, _P]),
    "mpemuBatchPlan": (_I, [_P, _P, _I64, _P, _I64, _I, _I, _I, _I, _P]),
    "mpemuGemmEmulatedBatched": (_I, [_P, _I, _I, _I64, _I64, _I64, _F, _I, _I, _F, _P, _I64, _P, _P]),
    "mpemuGemmMultiwordBatched": (_I, [_P, _I, _I, _I64, _I64, _I64, _F, _F, _F, _I, _I, _F, _P, _I64, _P, _P]),
    "mpemuStackedLd": (_I64, [_I64, _I]),
    "mpemuStackedBytes": (ctypes.c_size_t, [_I64, _I64, _I, _I]),
    "mpemuSplitBF16Stacked": (_I, [_P, _I64, _I64, _I64, _I, _P, _I64, _P]),
    "mpemuSplitFP16Stacked": (_I, [_P, _I64, _I64, _I64, _I, _F, _P, _I64, _P]),
    "mpemuGemmEmulatedConcat": (_I, [_P, _I64, _I64, _I64, _F, _P, _I64, _P, _I64, _I, _I, _F, _P, _I64]),
    "mpemuGemmMultiwordConcat": (_I, [_P, _I64, _I64, _I64, _F, _F, _F, _P, _I64, _P, _I64, _I, _I, _F, _P, _I64]),
    "mpkDebugEngineInfo": (_I, [_P, ctypes.POINTER(_F), ctypes.POINTER(_F), ctypes.POINTER(_I),
                                ctypes.POINTER(_F), ctypes.POINTER(_F)]),
    "mpkDebugProfile": (_I, [_P, _I]),
    "mpkDebugProfileRead": (_I, [_P, ctypes.POINTER(_D), ctypes.POINTER(_LL), ctypes.POINTER(_D),
                                 ctypes.POINTER(_LL), ctypes.POINTER(_D), ctypes.POINTER(_LL)]),
    "mpkDebugWideCounters": (_I, [_P, ctypes.POINTER(_LL), ctypes.POINTER(_LL), ctypes.POINTER(_LL)]),
    "mpkDebugWideRoundRows": (_I, [_P, _LL]),
    "mpkDebugGemmStatus": (_I, [_I]),
    "mpkDebugEngineLaunches": (_LL, [_P]),
    "mpkDebugSetWaitLimit": (_I, [_P, ctypes.c_ulonglong]),
    "mpkDebugInjectStall": (_I, [_P, _I]),
    "mpkDebugAssignPair": (_I, [_P, _I]),
    "mpkDebugOverlapRefine": (_I, [_P, _I]),
    "mpkDebugClearStatus": (_I, [_P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load the compiled library (once).  Raises MpkLibraryError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise MpkLibraryError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "or python mpkmeans_b200/build.py")
    try:
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | ctypes.RTLD_GLOBAL)
    except OSError as exc:  # pragma: no cover - depends on the host
        raise MpkLibraryError(f"cannot load {LIB_PATH}: {exc}") from exc
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


def check(fn: str, status: int) -> None:
    if status != MPK_OK:
        raise MpkError(fn, status)


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if not x.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not x.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return x.data_ptr()


def params_init(**kw) -> mpkParams:
    p = mpkParams()
    lib().mpkParamsInit(ctypes.byref(p))
    for k_, v in kw.items():
        setattr(p, k_, v)
    return p


def epsilon(d: int, accum: int = MPK_ACCUM_FP32) -> float:
    return lib().mpkEpsilon(d, accum)


def _lloyd(fn_name: str, P, C, labels, params: mpkParams | None, blas: int | None) -> mpkStats:
    n, d = P.shape
    k = C.shape[0]
    st = mpkStats()
    fn = getattr(lib(), fn_name)
    rc = fn(blas, _ptr(P), n, d, k, _ptr(C), _ptr(labels),
            ctypes.byref(params) if params is not None else None, ctypes.byref(st))
    check(fn_name, rc)
    return st


def kmeanspp(P, k: int, seed: int, C=None):
    """k-means++ seeding on the device (mpkInitKMeansPP): k rows of P (n x d,
    row major, device) into C (k x d, device; allocated when None)."""
    import torch
    n, d = P.shape
    if C is None:
        C = torch.empty((k, d), dtype=torch.float32, device=P.device)
    check("mpkInitKMeansPP", lib().mpkInitKMeansPP(_ptr(P), n, d, k, seed, _ptr(C)))
    return C


def means_mixed(P, C, labels, params: mpkParams | None = None, blas: int | None = None) -> mpkStats:
    """mpkMeansMixed on CUDA tensors: P (n x d fp32), C (k x d fp32, in/out), labels (n int32, out)."""
    return _lloyd("mpkMeansMixed", P, C, labels, params, blas)


def means_fp32(P, C, labels, params: mpkParams | None = None, blas: int | None = None) -> mpkStats:
    return _lloyd("mpkMeansFP32", P, C, labels, params, blas)


def assign(P, C, labels, params: mpkParams | None = None, blas: int | None = None) -> mpkStats:
    n, d = P.shape
    k = C.shape[0]
    st = mpkStats()
    rc = lib().mpkAssign(blas, _ptr(P), n, d, k, _ptr(C), _ptr(labels),
                         ctypes.byref(params) if params is not None else None, ctypes.byref(st))
    check("mpkAssign", rc)
    return st


def update(P, labels, C, moved2=None, blas: int | None = None) -> None:
    n, d = P.shape
    k = C.shape[0]
    check("mpkUpdate", lib().mpkUpdate(blas, _ptr(P), n, d, k, _ptr(labels), _ptr(C), _ptr(moved2)))


class PeerGroup:
    """One rank's exchange block for combining the ranks' sums over NVLink peer memory
    (mpkPeer*), created on the current device.  Per iteration: Engine.step into
    ``sums`` (an int device address), then ``combine`` instead of an allreduce and
    Engine.finalize.  Ranks of one process connect by addresses and devices
    (``connect_local``); ranks of different processes by exported IPC handles
    (``handle`` and ``connect_handles``)."""

    def __init__(self, rank: int, world: int, k: int, d: int):
        h = _P()
        check("mpkPeerCreate", lib().mpkPeerCreate(ctypes.byref(h), int(rank), int(world), int(k), int(d)))
        self.h = h
        self.rank, self.world = int(rank), int(world)
        self.sums = int(lib().mpkPeerSums(self.h))

    def handle(self) -> bytes:
        buf = ctypes.create_string_buffer(64)
        check("mpkPeerExportHandle", lib().mpkPeerExportHandle(self.h, buf))
        return buf.raw

    def base(self) -> int:
        b = _P()
        check("mpkPeerLocalBase", lib().mpkPeerLocalBase(self.h, ctypes.byref(b)))
        return int(b.value)

    def connect_handles(self, handles: list) -> None:
        bufs = [ctypes.create_string_buffer(bytes(h), 64) if (i != self.rank and h is not None) else None
                for i, h in enumerate(handles)]
        arr = (_P * self.world)(*[ctypes.cast(b, _P) if b is not None else None for b in bufs])
        check("mpkPeerConnect", lib().mpkPeerConnect(self.h, arr, None, None))
        self._keep = bufs

    def connect_local(self, bases: list, devices: list) -> None:
        arr = (_P * self.world)(*bases)
        dev = (_I * self.world)(*devices)
        check("mpkPeerConnect", lib().mpkPeerConnect(self.h, None, arr, dev))

    def combine(self, engine, C, moved2=None) -> None:
        check("mpkPeerCombine", lib().mpkPeerCombine(self.h, engine.h, _ptr(C), _ptr(moved2)))

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().mpkPeerDestroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:                        # noqa: BLE001 - interpreter shutdown
            pass


class Engine:
    """Handle over ``mpkEngine``: the split points and all scratch stay on the
    device; assign / accumulate / finalize are the three steps of a Lloyd
    iteration, with the caller free to all-reduce the int64 sums between
    accumulate and finalize."""

    def __init__(self, P, k: int, C0=None, pmax_global: float = 0.0, n_global: int = 0, stream: int | None = None):
        n, d = P.shape
        self.n, self.d, self.k = n, d, k
        self._P = P
        h = ctypes.c_void_p()
        rc = lib().mpkEngineCreate(ctypes.byref(h), _ptr(P), n, d, k, _ptr(C0), float(pmax_global),
                                   int(n_global), stream)
        check("mpkEngineCreate", rc)
        self.h = h

    @property
    def sums_length(self) -> int:
        return int(lib().mpkEngineSumsLength(self.h))

    def assign(self, C, labels, refine: bool = True) -> None:
        check("mpkEngineAssign", lib().mpkEngineAssign(self.h, _ptr(C), _ptr(labels), int(bool(refine))))

    def accumulate(self, labels, sums) -> None:
        check("mpkEngineAccumulate", lib().mpkEngineAccumulate(self.h, _ptr(labels), _ptr(sums)))

    def finalize(self, sums, C, moved2=None) -> None:
        check("mpkEngineFinalize", lib().mpkEngineFinalize(self.h, _ptr(sums), _ptr(C), _ptr(moved2)))

    def iterate(self, C, labels, sums, iters: int = 1, refine: bool = True) -> None:
        """``iters`` Lloyd iterations of this shard alone (assign, accumulate,
        finalize), replayed from CUDA graphs after the first call."""
        check("mpkEngineIterate", lib().mpkEngineIterate(self.h, _ptr(C), _ptr(labels), _ptr(sums), int(iters),
                                                         int(bool(refine))))

    def step(self, C, labels, sums, refine: bool = True) -> None:
        """One multi-GPU step of this shard: assign then accumulate into ``sums`` (no
        finalisation; allreduce ``sums`` and call finalize), replayed from CUDA graphs."""
        check("mpkEngineStep", lib().mpkEngineStep(self.h, _ptr(C), _ptr(labels), _ptr(sums), int(bool(refine))))

    def inertia(self, C, labels) -> float:
        out = ctypes.c_double()
        check("mpkEngineInertia", lib().mpkEngineInertia(self.h, _ptr(C), _ptr(labels), ctypes.byref(out)))
        return out.value

    def frac_bits(self) -> int:
        return int(lib().mpkEngineFracBits(self.h))

    def counters(self) -> dict:
        r, c, f = _LL(), _LL(), _LL()
        s = _I()
        check("mpkEngineCounters", lib().mpkEngineCounters(self.h, ctypes.byref(r), ctypes.byref(c),
                                                           ctypes.byref(f), ctypes.byref(s)))
        return {"rows_refined": r.value, "cand_refined": c.value, "rows_full_scan": f.value, "status": s.value}

    def wide_counters(self) -> dict:
        w, f, c = _LL(), _LL(), _LL()
        check("mpkDebugWideCounters", lib().mpkDebugWideCounters(self.h, ctypes.byref(w), ctypes.byref(f),
                                                                 ctypes.byref(c)))
        return {"wide_rows": w.value, "full_scans": f.value, "capacity": c.value}

    def launches(self) -> int:
        return int(lib().mpkDebugEngineLaunches(self.h))

    def set_wait_limit(self, ns: int) -> None:
        check("mpkDebugSetWaitLimit", lib().mpkDebugSetWaitLimit(self.h, ns))

    def inject_stall(self, stage: int) -> None:
        check("mpkDebugInjectStall", lib().mpkDebugInjectStall(self.h, stage))

    def assign_pair(self, mode: int) -> None:
        """CTA-pair assignment kernel where it applies (the default); 0: one CTA per row tile."""
        check("mpkDebugAssignPair", lib().mpkDebugAssignPair(self.h, int(mode)))

    def overlap_refine(self, mode: int) -> None:
        """Refinement beside the update's segmented sum (the default); 0: refine, then update."""
        check("mpkDebugOverlapRefine", lib().mpkDebugOverlapRefine(self.h, int(mode)))

    def clear_status(self) -> None:
        check("mpkDebugClearStatus", lib().mpkDebugClearStatus(self.h))

    def wide_round_rows(self, rows: int) -> None:
        check("mpkDebugWideRoundRows", lib().mpkDebugWideRoundRows(self.h, rows))

    def info(self) -> dict:
        sc, eta, c1, c2 = _F(), _F(), _F(), _F()
        fr = _I()
        check("mpkDebugEngineInfo", lib().mpkDebugEngineInfo(self.h, ctypes.byref(sc), ctypes.byref(eta),
                                                             ctypes.byref(fr), ctypes.byref(c1), ctypes.byref(c2)))
        return {"scale": sc.value, "eta": eta.value, "frac": fr.value, "c1": c1.value, "c2": c2.value}

    def profile(self, enable: bool = True) -> None:
        check("mpkDebugProfile", lib().mpkDebugProfile(self.h, int(bool(enable))))

    def profile_read(self) -> dict:
        a, r, u = _D(), _D(), _D()
        na, nr, nu = _LL(), _LL(), _LL()
        check("mpkDebugProfileRead", lib().mpkDebugProfileRead(self.h, ctypes.byref(a), ctypes.byref(na),
                                                               ctypes.byref(r), ctypes.byref(nr),
                                                               ctypes.byref(u), ctypes.byref(nu)))
        return {"assign_ms": a.value, "assign_launches": na.value, "refine_ms": r.value, "refine_launches": nr.value,
                "accum_ms": u.value, "accum_launches": nu.value}

    def trace(self, out4) -> None:
        check("mpkDebugSetAssignTrace", lib().mpkDebugSetAssignTrace(self.h, _ptr(out4)))

    def close(self) -> None:
        if getattr(self, "h", None):
            lib().mpkEngineDestroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
