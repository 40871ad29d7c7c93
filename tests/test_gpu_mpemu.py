"""The split-precision GEMM ABI (include/mpemu.h) on a B200, through the C ABI.

Pins: splits bit-exact against the oracle and against the reference's own
split outputs (tests/golden/ref_mpemu.npz); AutoScale and the term schedule
exactly; GEMMs within the error model of the exact FP64 sum of the split
words' products and close to the reference's cuBLAS results; bitwise
resumability of ranges (gemm-emulation/bench/test_refine.cu); accuracy
against FP64 within twice that of native FP32 SGEMM.
"""
import ctypes

import numpy as np
import pytest

import oracle as O
from conftest import golden

torch = pytest.importorskip("torch")
import mpkmeans_b200 as M  # noqa: E402

pytestmark = pytest.mark.gpu

OK = 0


def lib():
    return M.lib()


def handle():
    return torch.cuda.current_blas_handle()


def split_gpu(A_cm, rows, cols, lda, nsplits, bf16=True, scale=1.0):
    """A_cm: column-major storage as a (cols, lda) float32 array."""
    lds = int(lib().mpemuSplitLd(rows))
    stride = lds * cols
    dA = torch.from_numpy(np.ascontiguousarray(A_cm, np.float32)).cuda()
    dS = torch.zeros(stride * nsplits, dtype=torch.int16, device="cuda")
    if bf16:
        rc = lib().mpemuSplitBF16(dA.data_ptr(), lda, rows, cols, nsplits, dS.data_ptr(), lds, stride, None)
    else:
        rc = lib().mpemuSplitFP16(dA.data_ptr(), lda, rows, cols, nsplits, scale, dS.data_ptr(), lds, stride, None)
    assert rc == OK
    torch.cuda.synchronize()
    return dS, lds, stride


def autoscale_gpu(A_cm, rows, cols, lda):
    dA = torch.from_numpy(np.ascontiguousarray(A_cm, np.float32)).cuda()
    sc = ctypes.c_float()
    assert lib().mpemuAutoScaleFP16(dA.data_ptr(), lda, rows, cols, ctypes.byref(sc), None) == OK
    return sc.value


def words_f64(S_u16, nsplits, lds, stride, rows, cols, bf16, scale=1.0):
    planes = []
    for s in range(nsplits):
        w = S_u16[s * stride:(s + 1) * stride]
        f = O.bf16_to_f32(w) if bf16 else O.fp16_to_f32(w)
        planes.append(f.reshape(cols, lds)[:, :rows].astype(np.float64) / scale)
    return planes                      # each (cols, rows): column-major storage


def exact_emulated(opa, opb, m, n, k, Ap, Bp, terms):
    """Exact FP64 sum over terms of op(A_i) op(B_j); planes are (cols, rows) column-major arrays."""
    D = np.zeros((m, n))
    for (i, j) in terms:
        A = Ap[i].T if True else None          # stored rows x cols
        B = Bp[j].T
        opA = A if opa == 0 else A.T           # m x k
        opB = B if opb == 0 else B.T           # k x n
        D += opA @ opB
    return D


def gemm_bf16(opa, opb, m, n, k, dSA, lda, sa, dSB, ldb, sb, nsplits, b, e, dC, alpha=1.0, beta=0.0):
    return lib().mpemuGemmEmulatedRange(handle(), opa, opb, m, n, k, alpha, dSA.data_ptr(), lda, sa, dSB.data_ptr(),
                                        ldb, sb, nsplits, b, e, beta, dC.data_ptr(), m)


def gemm_fp16(opa, opb, m, n, k, dSA, lda, sa, scA, dSB, ldb, sb, scB, nsplits, b, e, dC, alpha=1.0, beta=0.0):
    return lib().mpemuGemmMultiwordRange(handle(), opa, opb, m, n, k, alpha, dSA.data_ptr(), lda, sa, scA,
                                         dSB.data_ptr(), ldb, sb, scB, nsplits, b, e, beta, dC.data_ptr(), m)


# ------------------------------------------------------------------ splits --

@pytest.mark.parametrize("rows,cols,lda,emax", [(1024, 64, 1024, 0), (1023, 77, 1023, 0), (100, 33, 101, 0),
                                                 (1, 1, 1, 0), (7, 3, 9, 0), (512, 64, 512, 8)])
def test_splits_bit_exact_vs_oracle(cuda, rows, cols, lda, emax):
    A = O.make_uniform((cols, lda), 7 + rows, emax=emax)
    for ns in (1, 2, 3, 4):
        dS, lds, stride = split_gpu(A, rows, cols, lda, ns, bf16=True)
        want, _, _ = O.split_bf16(A, rows, cols, lda, ns)
        assert np.array_equal(dS.cpu().numpy().view(np.uint16), want)
    sc = autoscale_gpu(A, rows, cols, lda)
    assert sc == O.autoscale_fp16(A, rows, cols, lda)
    for ns in (1, 2, 3):
        dS, lds, stride = split_gpu(A, rows, cols, lda, ns, bf16=False, scale=sc)
        want, _, _ = O.split_fp16(A, rows, cols, lda, ns, sc)
        assert np.array_equal(dS.cpu().numpy().view(np.uint16), want)


def test_splits_equal_reference_outputs(cuda):
    g = golden("ref_mpemu.npz")
    rows, cols, lda = (int(x) for x in g["shape"])
    A = g["A"]
    for ns in (1, 2, 3, 4):
        dS, _, _ = split_gpu(A, rows, cols, lda, ns, bf16=True)
        assert np.array_equal(dS.cpu().numpy().view(np.uint16), g[f"bf16_split_{ns}"])
    sc = autoscale_gpu(A, rows, cols, lda)
    assert np.float32(sc) == g["fp16_scale"]
    for ns in (1, 2, 3):
        dS, _, _ = split_gpu(A, rows, cols, lda, ns, bf16=False, scale=sc)
        assert np.array_equal(dS.cpu().numpy().view(np.uint16), g[f"fp16_split_{ns}"])


def test_schedule_and_macs(cuda):
    t = (ctypes.c_int * 32)()
    nt = lib().mpemuTermSchedule(3, 16, t)
    got = [(t[2 * i], t[2 * i + 1]) for i in range(nt)]
    assert got == [(0, 0), (0, 1), (1, 0), (0, 2), (1, 1), (2, 0), (1, 2), (2, 1), (2, 2)]
    assert [lib().mpemuTermSchedule(3, c, t) for c in (1, 3, 6, 9)] == [1, 3, 6, 9]
    assert [lib().mpemuMultiwordMacs(p) for p in range(5)] == [0, 1, 3, 6, 10]
    assert lib().mpemuTermCount(16) == 256 and lib().mpemuTermCount(17) == 0
    assert lib().mpemuSplitLd(13) == 16 and lib().mpemuSplitBytes(13, 5, 3) == 16 * 5 * 3 * 2


def test_check_split_counts(cuda):
    A = O.make_uniform((64, 64), 5) * np.float32(0.5)
    sc = autoscale_gpu(A, 64, 64, 64)
    dA = torch.from_numpy(A).cuda()
    for scale in (1.0, sc):
        dS, lds, stride = split_gpu(A, 64, 64, 64, 2, bf16=False, scale=scale)
        cnt = torch.zeros(3, dtype=torch.int64, device="cuda")
        assert lib().mpemuCheckSplitFP16(dA.data_ptr(), 64, 64, 64, 2, scale, dS.data_ptr(), lds, stride,
                                         cnt.data_ptr(), None) == OK
        c = cnt.cpu().numpy()
        assert c.sum() == 2 * 64 * 64 and c[0] == 0
        if scale != 1.0:
            assert c[1] < c[2]


# ------------------------------------------------------------------- GEMM ---

def _operands(opa, opb, m, n, k, seed, emax=0):
    ra, ca = (m, k) if opa == 0 else (k, m)
    rb, cb = (k, n) if opb == 0 else (n, k)
    A = O.make_uniform((ca, ra), seed, emax=emax)
    B = O.make_uniform((cb, rb), seed + 1, emax=emax)
    return A, (ra, ca), B, (rb, cb)


@pytest.mark.parametrize("m,n,k", [(96, 72, 80), (300, 200, 150), (128, 256, 64), (1, 1, 1), (513, 257, 129)])
@pytest.mark.parametrize("opa,opb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_error_model(cuda, m, n, k, opa, opb):
    A, (ra, ca), B, (rb, cb) = _operands(opa, opb, m, n, k, 31 + m + 2 * opa + opb)
    dSA, la, sa = split_gpu(A, ra, ca, ra, 3, bf16=True)
    dSB, lb, sb = split_gpu(B, rb, cb, rb, 3, bf16=True)
    Ap = words_f64(dSA.cpu().numpy().view(np.uint16), 3, la, sa, ra, ca, True)
    Bp = words_f64(dSB.cpu().numpy().view(np.uint16), 3, lb, sb, rb, cb, True)
    absA = np.abs(A[:, :ra].T.astype(np.float64))
    absB = np.abs(B[:, :rb].T.astype(np.float64))
    absAB = (absA if opa == 0 else absA.T) @ (absB if opb == 0 else absB.T)
    sched = O.term_schedule(3, 9)
    for macs in (1, 3, 6, 9):
        dC = torch.zeros(n * m, dtype=torch.float32, device="cuda")
        assert gemm_bf16(opa, opb, m, n, k, dSA, la, sa, dSB, lb, sb, 3, 0, macs, dC) == OK
        torch.cuda.synchronize()
        got = dC.cpu().numpy().reshape(n, m).T.astype(np.float64)
        D = exact_emulated(opa, opb, m, n, k, Ap, Bp, sched[:macs])
        bound = (macs * ((k + 15) // 16) + 16) * 2.0 ** -22 * absAB + 1e-30
        assert np.all(np.abs(got - D) <= bound), (macs, float(np.max(np.abs(got - D) / bound)))


def test_gemm_close_to_reference_outputs(cuda):
    g = golden("ref_mpemu.npz")
    m, n, k = (int(x) for x in g["gemm_shape"])
    for opa in (0, 1):
        for opb in (0, 1):
            A, B = g[f"gemm_A_{opa}{opb}"], g[f"gemm_B_{opa}{opb}"]
            ra, ca = (m, k) if opa == 0 else (k, m)
            rb, cb = (k, n) if opb == 0 else (n, k)
            dSA, la, sa = split_gpu(A, ra, ca, ra, 3, True)
            dSB, lb, sb = split_gpu(B, rb, cb, rb, 3, True)
            D = O.gemm_f64(opa, opb, m, n, k, A, ra, B, rb)                    # exact product, (n, m)
            absAB = O.gemm_f64(opa, opb, m, n, k, np.abs(A), ra, np.abs(B), rb)
            for macs, tol in ((1, 2 ** -7), (3, 2 ** -14), (6, 2 ** -19), (9, 2 ** -19)):
                dC = torch.zeros(n * m, dtype=torch.float32, device="cuda")
                assert gemm_bf16(opa, opb, m, n, k, dSA, la, sa, dSB, lb, sb, 3, 0, macs, dC) == OK
                torch.cuda.synchronize()
                got = dC.cpu().numpy().reshape(n, m)
                ref = g[f"gemm_bf16_{opa}{opb}_{macs}"].reshape(n, m)
                assert np.all(np.abs(got - ref) <= 2 * tol * absAB + 1e-30)
                assert np.all(np.abs(got - D) <= tol * absAB + 1e-30)
            sA = autoscale_gpu(A, ra, ca, ra)
            sB = autoscale_gpu(B, rb, cb, rb)
            dSA, la, sa = split_gpu(A, ra, ca, ra, 2, False, sA)
            dSB, lb, sb = split_gpu(B, rb, cb, rb, 2, False, sB)
            for macs, tol in ((1, 2 ** -9), (3, 2 ** -19)):
                dC = torch.zeros(n * m, dtype=torch.float32, device="cuda")
                assert gemm_fp16(opa, opb, m, n, k, dSA, la, sa, sA, dSB, lb, sb, sB, 2, 0, macs, dC) == OK
                torch.cuda.synchronize()
                got = dC.cpu().numpy().reshape(n, m)
                ref = g[f"gemm_fp16_{opa}{opb}_{macs}"].reshape(n, m)
                assert np.all(np.abs(got - ref) <= 2 * tol * absAB + 1e-30)


def test_ranges_resume_bitwise(cuda):
    # gemm-emulation/bench/test_refine.cu: [0,e) == [0,c) + [c,e) for every cut
    N = 256
    A = O.make_uniform((N, N), 11)
    B = O.make_uniform((N, N), 22)
    dSA, l, s = split_gpu(A, N, N, N, 3, True)
    dSB, _, _ = split_gpu(B, N, N, N, 3, True)
    whole = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 0, 9, whole) == OK
    for cut in range(1, 9):
        part = torch.zeros(N * N, dtype=torch.float32, device="cuda")
        assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 0, cut, part) == OK
        assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, cut, 9, part, beta=1.0) == OK
        torch.cuda.synchronize()
        assert torch.equal(part, whole), cut
    # MPEMU_ALL_MACS, the whole-budget driver, and an empty range with beta = 1
    part = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 0, 4, part) == OK
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 4, -1, part, beta=1.0) == OK
    torch.cuda.synchronize()
    assert torch.equal(part, whole)
    six = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert lib().mpemuGemmEmulated(handle(), 0, 0, N, N, N, 1.0, dSA.data_ptr(), l, s, dSB.data_ptr(), l, s, 3, 6,
                                   0.0, six.data_ptr(), N) == OK
    six_r = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 0, 6, six_r) == OK
    keep = six_r.clone()
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 6, 6, six_r, beta=1.0) == OK
    torch.cuda.synchronize()
    assert torch.equal(six, six_r) and torch.equal(six_r, keep)
    # FP16 multiword, autoscaled operands
    sA, sB = autoscale_gpu(A, N, N, N), autoscale_gpu(B, N, N, N)
    dHA, _, _ = split_gpu(A, N, N, N, 3, False, sA)
    dHB, _, _ = split_gpu(B, N, N, N, 3, False, sB)
    whole = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert gemm_fp16(0, 0, N, N, N, dHA, l, s, sA, dHB, l, s, sB, 3, 0, 6, whole) == OK
    for cut in range(1, 6):
        part = torch.zeros(N * N, dtype=torch.float32, device="cuda")
        assert gemm_fp16(0, 0, N, N, N, dHA, l, s, sA, dHB, l, s, sB, 3, 0, cut, part) == OK
        assert gemm_fp16(0, 0, N, N, N, dHA, l, s, sA, dHB, l, s, sB, 3, cut, 6, part, beta=1.0) == OK
        torch.cuda.synchronize()
        assert torch.equal(part, whole), cut


def test_unaligned_layout_fallback(cuda):
    m, n, k = 77, 45, 33
    A = O.make_uniform((k, m + 1), 3)         # lda = m + 1 (odd): not TMA-addressable
    B = O.make_uniform((n, k), 4)
    lda = m + 1
    dA = torch.from_numpy(A).cuda()
    lds = lda                                   # plane leading dimension equal to lda, not a multiple of 8
    dSA = torch.zeros(lds * k * 3, dtype=torch.int16, device="cuda")
    assert lib().mpemuSplitBF16(dA.data_ptr(), lda, m, k, 3, dSA.data_ptr(), lds, lds * k, None) == OK
    dSB, lb, sb = split_gpu(B, k, n, k, 3, True)
    dC = torch.zeros(n * m, dtype=torch.float32, device="cuda")
    assert gemm_bf16(0, 0, m, n, k, dSA, lds, lds * k, dSB, lb, sb, 3, 0, 9, dC) == OK
    torch.cuda.synchronize()
    exact = O.gemm_f64(0, 0, m, n, k, A, lda, B, k).reshape(n, m)
    absAB = O.gemm_f64(0, 0, m, n, k, np.abs(A), lda, np.abs(B), k).reshape(n, m)
    assert np.all(np.abs(dC.cpu().numpy().reshape(n, m) - exact) <= 2 ** -19 * absAB + 1e-30)


def test_invalid_arguments(cuda):
    d = torch.zeros(64, dtype=torch.int16, device="cuda")
    c = torch.zeros(64, dtype=torch.float32, device="cuda")
    L = lib()
    assert L.mpemuGemmEmulatedRange(handle(), 0, 0, 4, 4, 4, 1.0, d.data_ptr(), 8, 32, d.data_ptr(), 8, 32, 5, 0, 1,
                                    0.0, c.data_ptr(), 4) == 1
    assert L.mpemuGemmEmulatedRange(handle(), 0, 0, 4, 4, 4, 1.0, d.data_ptr(), 8, 32, d.data_ptr(), 8, 32, 3, 2, 1,
                                    0.0, c.data_ptr(), 4) == 1
    assert L.mpemuGemmEmulatedRange(None, 0, 0, 4, 4, 4, 1.0, d.data_ptr(), 8, 32, d.data_ptr(), 8, 32, 3, 3, 3,
                                    1.0, c.data_ptr(), 4) == 0      # empty range with beta 1: no-op
    assert L.mpemuGemmEmulatedRange(None, 0, 0, 4, 4, 4, 1.0, d.data_ptr(), 8, 32, d.data_ptr(), 8, 32, 3, 0, 3,
                                    0.0, c.data_ptr(), 4) == 1      # no handle
    assert L.mpemuSplitBF16(c.data_ptr(), 4, 4, 4, 5, d.data_ptr(), 8, 32, None) == 1
    assert L.mpemuSplitFP16(c.data_ptr(), 4, 4, 4, 2, 0.0, d.data_ptr(), 8, 32, None) == 1
    assert L.mpemuStatusString(3) == b"MPEMU_STATUS_CUBLAS_ERROR"


# ----------------------------------------------------- config-2 accuracy ----

@pytest.mark.parametrize("emax", [0, 8])
def test_emulated_error_within_twice_native_sgemm(cuda, emax):
    """BASELINE config 2 criterion at N = 2048: max |C - C64| of the emulated
    GEMMs (BF16x3 with 6 products; FP16x2 scaled with 3) within 2x that of
    native FP32 SGEMM (TF32 off)."""
    N = 2048
    A = O.make_uniform((N, N), 1000 + emax, emax=emax)       # column-major storage
    B = O.make_uniform((N, N), 2000 + emax, emax=emax)
    tA, tB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    # column-major C = A B  <=>  row-major C^T = B^T A^T, i.e. torch: (B_rm @ A_rm) with rm = the stored arrays
    C64 = (tB.double() @ tA.double())
    torch.backends.cuda.matmul.allow_tf32 = False
    C32 = tB @ tA
    native = float((C32.double() - C64).abs().max())
    dSA, l, s = split_gpu(A, N, N, N, 3, True)
    dSB, _, _ = split_gpu(B, N, N, N, 3, True)
    dC = torch.zeros(N * N, dtype=torch.float32, device="cuda")
    assert gemm_bf16(0, 0, N, N, N, dSA, l, s, dSB, l, s, 3, 0, 6, dC) == OK
    bf = float((dC.reshape(N, N).double() - C64).abs().max())
    sA, sB = autoscale_gpu(A, N, N, N), autoscale_gpu(B, N, N, N)
    dHA, _, _ = split_gpu(A, N, N, N, 2, False, sA)
    dHB, _, _ = split_gpu(B, N, N, N, 2, False, sB)
    assert gemm_fp16(0, 0, N, N, N, dHA, l, s, sA, dHB, l, s, sB, 2, 0, 3, dC) == OK
    fp = float((dC.reshape(N, N).double() - C64).abs().max())
    assert bf <= 2 * native, (bf, native)
    assert fp <= 2 * native, (fp, native)


# ------------------------------------ context, concatenated-k, batched ----

def test_context_arena_and_workspace_views(cuda):
    L = lib()
    ctx = ctypes.c_void_p()
    assert L.mpemuContextCreate(ctypes.byref(ctx)) == OK
    ws = M.mpemuWorkspace()
    assert L.mpemuBf16WorkspaceInit(ctx, 100, 60, 40, 3, ctypes.byref(ws)) == 1     # nothing reserved yet
    need = L.mpemuBf16WorkspaceBytes(100, 60, 40, 3)
    al = lambda v: (v + 255) // 256 * 256                                          # noqa: E731
    assert need == al(104 * 40 * 3 * 2) + al(40 * 60 * 3 * 2)
    assert L.mpemuContextReserve(ctx, need) == OK and L.mpemuContextAllocCount(ctx) == 1
    assert L.mpemuContextReserve(ctx, need // 2) == OK and L.mpemuContextAllocCount(ctx) == 1   # fits: no-op
    assert L.mpemuContextCapacity(ctx) == need
    assert L.mpemuBf16WorkspaceInit(ctx, 100, 60, 40, 3, ctypes.byref(ws)) == OK
    assert ws.sA == L.mpemuContextBase(ctx) and (ws.sB - ws.sA) % 256 == 0
    assert (ws.ldA, ws.strideA, ws.ldB, ws.strideB, ws.nsplits) == (104, 104 * 40, 40, 40 * 60, 3)
    assert L.mpemuFp16WorkspaceInit(ctx, 100, 60, 41, 3, ctypes.byref(ws)) == 1     # needs more than reserved
    assert L.mpemuContextDestroy(ctx) == OK


@pytest.mark.parametrize("m,n,k", [(300, 200, 160), (256, 130, 100), (33, 17, 8)])
def test_concat_equals_range(cuda, m, n, k):
    """mpemu.h's concatenated-k drivers (gemm-emulation/bench/test_concat.cu:
    concat == range within 1e-6): stacked words equal the ordinary split's,
    and the sum over bins [0, nbins) matches the range over the same products."""
    L = lib()
    A = O.make_uniform((k, m), 70 + m)        # column-major m x k
    B = O.make_uniform((n, k), 71 + n)        # column-major k x n
    dSA, la, sa = split_gpu(A, m, k, m, 3, True)
    dSB, lb, sb = split_gpu(B, k, n, k, 3, True)
    ldsb = L.mpemuStackedLd(k, 3)
    assert L.mpemuStackedBytes(k, n, 3, 2) == ldsb * n * 2
    dB = torch.from_numpy(B).cuda()
    dST = torch.zeros(ldsb * n, dtype=torch.int16, device="cuda")
    assert L.mpemuSplitBF16Stacked(dB.data_ptr(), k, k, n, 3, dST.data_ptr(), ldsb, None) == OK
    torch.cuda.synchronize()
    st = dST.cpu().numpy().reshape(n, ldsb)
    nrm = dSB.cpu().numpy().reshape(3, n, lb)
    for j in range(3):
        assert np.array_equal(st[:, (2 - j) * k:(3 - j) * k], nrm[j, :, :k])
    exact = np.abs(O.gemm_f64(0, 0, m, n, k, np.abs(A), m, np.abs(B), k)).reshape(n, m)
    # k % 8 != 0: the stacked planes are not 16-byte aligned for TMA, and the
    # SIMT path (plain FP32 fmaf chains) stands in; both are within 2^-19 of exact
    tol = 1e-6 if k % 8 == 0 else 2.0 ** -18
    for nbins in (1, 2, 3):
        want = torch.zeros(n * m, dtype=torch.float32, device="cuda")
        assert gemm_bf16(0, 0, m, n, k, dSA, la, sa, dSB, lb, sb, 3, 0, nbins * (nbins + 1) // 2, want) == OK
        got = torch.zeros(n * m, dtype=torch.float32, device="cuda")
        assert L.mpemuGemmEmulatedConcat(handle(), m, n, k, 1.0, dSA.data_ptr(), la, dST.data_ptr(), ldsb, 3,
                                         nbins, 0.0, got.data_ptr(), m) == OK
        torch.cuda.synchronize()
        g, w = got.cpu().numpy().reshape(n, m), want.cpu().numpy().reshape(n, m)
        assert np.all(np.abs(g - w) <= tol * exact + 1e-30), nbins
        if k % 8 == 0:
            assert np.array_equal(g, w)          # same kernel, same products, same order
    # FP16 multiword concat against its range driver
    sA, sB = autoscale_gpu(A, m, k, m), autoscale_gpu(B, k, n, k)
    dHA, la2, sa2 = split_gpu(A, m, k, m, 2, False, sA)
    dHT = torch.zeros(L.mpemuStackedLd(k, 2) * n, dtype=torch.int16, device="cuda")
    ld2 = L.mpemuStackedLd(k, 2)
    assert L.mpemuSplitFP16Stacked(dB.data_ptr(), k, k, n, 2, sB, dHT.data_ptr(), ld2, None) == OK
    dHB, lb2, sb2 = split_gpu(B, k, n, k, 2, False, sB)
    want = torch.zeros(n * m, dtype=torch.float32, device="cuda")
    assert gemm_fp16(0, 0, m, n, k, dHA, la2, sa2, sA, dHB, lb2, sb2, sB, 2, 0, 3, want) == OK
    got = torch.zeros(n * m, dtype=torch.float32, device="cuda")
    assert L.mpemuGemmMultiwordConcat(handle(), m, n, k, 1.0, sA, sB, dHA.data_ptr(), la2, dHT.data_ptr(), ld2, 2, 2,
                                      0.0, got.data_ptr(), m) == OK
    torch.cuda.synchronize()
    assert np.all(np.abs(got.cpu().numpy() - want.cpu().numpy()).reshape(n, m) <= tol * exact + 1e-30)
    # argument checks in the reference's order
    assert L.mpemuGemmEmulatedConcat(handle(), m, n, k, 1.0, dSA.data_ptr(), la, dST.data_ptr(), ldsb, 3, 4, 0.0,
                                     got.data_ptr(), m) == 1
    assert L.mpemuGemmEmulatedConcat(None, m, n, k, 1.0, dSA.data_ptr(), la, dST.data_ptr(), ldsb, 3, 1, 0.0,
                                     got.data_ptr(), m) == 1
    assert L.mpemuSplitBF16Stacked(dB.data_ptr(), k, k, n, 3, dST.data_ptr(), 3 * k - 1, None) == 1


def test_batched_equals_range(cuda):
    """The batched drivers take their products from mpemuBatchPlan and give
    the range driver's result for the same products, bit for bit."""
    L = lib()
    m, n, k = 200, 96, 120
    A = O.make_uniform((k, m), 81)
    B = O.make_uniform((n, k), 82)
    dSA, la, sa = split_gpu(A, m, k, m, 3, True)
    dSB, lb, sb = split_gpu(B, k, n, k, 3, True)
    ctx = ctypes.c_void_p()
    assert L.mpemuContextCreate(ctypes.byref(ctx)) == OK
    assert L.mpemuContextReserve(ctx, L.mpemuBatchWorkspaceBytes(m, n, 9, 4) + 4096) == OK
    bw = M.mpemuBatchWorkspace()
    assert L.mpemuBatchWorkspaceInit(ctx, m, n, 9, 4, 1000, ctypes.byref(bw)) == OK
    assert bw.ldt == 208 and bw.capacity == 9 and bw.planned == 0
    assert L.mpemuGemmEmulatedBatched(handle(), 0, 0, m, n, k, 1.0, 0, 1, 0.0, dSA.data_ptr(), m,
                                      ctypes.byref(bw), None) == 1                 # nothing planned yet
    assert L.mpemuBatchPlan(ctypes.byref(bw), dSA.data_ptr(), sa, dSB.data_ptr(), sb, 2, 3, 0, 6, None) == OK
    assert bw.planned == 6
    for begin, count in ((0, 6), (2, 3), (5, 1)):
        want = torch.zeros(n * m, dtype=torch.float32, device="cuda")
        assert gemm_bf16(0, 0, m, n, k, dSA, la, sa, dSB, lb, sb, 3, begin, begin + count, want) == OK
        got = torch.full((n * m,), 7.0, dtype=torch.float32, device="cuda")
        assert L.mpemuGemmEmulatedBatched(handle(), 0, 0, m, n, k, 1.0, begin, count, 0.0, got.data_ptr(), m,
                                          ctypes.byref(bw), None) == OK
        torch.cuda.synchronize()
        assert torch.equal(got, want), (begin, count)
    assert L.mpemuGemmEmulatedBatched(handle(), 0, 0, m, n, k, 1.0, 4, 3, 0.0, got.data_ptr(), m,
                                      ctypes.byref(bw), None) == 1                 # beyond the plan
    assert L.mpemuBatchPlan(ctypes.byref(bw), dSA.data_ptr(), sa, dSB.data_ptr(), sb, 2, 3, 0, 10, None) == 1
    # FP16 multiword batched against the multiword range driver
    sA, sB = autoscale_gpu(A, m, k, m), autoscale_gpu(B, k, n, k)
    dHA, _, _ = split_gpu(A, m, k, m, 2, False, sA)
    dHB, _, _ = split_gpu(B, k, n, k, 2, False, sB)
    assert L.mpemuBatchPlan(ctypes.byref(bw), dHA.data_ptr(), sa, dHB.data_ptr(), sb, 2, 2, 0, 3, None) == OK
    want = torch.zeros(n * m, dtype=torch.float32, device="cuda")
    assert gemm_fp16(0, 0, m, n, k, dHA, la, sa, sA, dHB, lb, sb, sB, 2, 0, 3, want) == OK
    got = torch.zeros(n * m, dtype=torch.float32, device="cuda")
    assert L.mpemuGemmMultiwordBatched(handle(), 0, 0, m, n, k, 1.0, sA, sB, 0, 3, 0.0, got.data_ptr(), m,
                                       ctypes.byref(bw), None) == OK
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert L.mpemuContextDestroy(ctx) == OK


def test_zz_gemm_status_word_clean(cuda):
    """After every GEMM of this module no bounded wait inside the kernel ran out."""
    assert lib().mpkDebugGemmStatus(1) == 0
