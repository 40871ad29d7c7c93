"""The data loaders (mpkLoadBin, mpkLoadLibsvm; reference kmeans/src/data.cu:73-211)
are host code: exercised here on CPU, and compared with the reference's own
loaders (oracle/_ref, compiled from its sources) on the same files."""
import ctypes

import numpy as np
import pytest

import mpkmeans_b200 as M
import oracle as O

libc = ctypes.CDLL(None)
libc.free.argtypes = [ctypes.c_void_p]

LIBSVM = """# a comment line
1 1:0.5 3:-2.25 7:1e-3
-1 2:4 qid:17 3:1.5   # trailing comment

+1 7:8.0 1:-1
2,3 4:0.125\r
-1\t5:3\t6:-6
"""


def load_bin(lib, path, d, max_rows):
    n = ctypes.c_int()
    p = ctypes.POINTER(ctypes.c_float)()
    rc = lib.mpkLoadBin(str(path).encode(), d, max_rows, ctypes.byref(n), ctypes.byref(p))
    if rc != 0:
        return rc, None
    out = np.ctypeslib.as_array(p, shape=(n.value * d,)).copy().reshape(n.value, d)
    libc.free(ctypes.cast(p, ctypes.c_void_p))
    return rc, out


def load_libsvm(lib, path):
    n, d, nc = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    p = ctypes.POINTER(ctypes.c_float)()
    lab = ctypes.POINTER(ctypes.c_int)()
    rc = lib.mpkLoadLibsvm(str(path).encode(), ctypes.byref(n), ctypes.byref(d), ctypes.byref(p), ctypes.byref(lab),
                           ctypes.byref(nc))
    if rc != 0:
        return rc, None, None, None
    P = np.ctypeslib.as_array(p, shape=(n.value * d.value,)).copy().reshape(n.value, d.value)
    L = np.ctypeslib.as_array(lab, shape=(n.value,)).copy()
    libc.free(ctypes.cast(p, ctypes.c_void_p))
    libc.free(ctypes.cast(lab, ctypes.c_void_p))
    return rc, P, L, nc.value


def ref_lib():
    if not O.REF_LIB_PATH.exists():
        return None
    r = ctypes.CDLL(str(O.REF_LIB_PATH))
    r.mpkLoadBin.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_longlong, ctypes.POINTER(ctypes.c_int),
                             ctypes.POINTER(ctypes.POINTER(ctypes.c_float))]
    r.mpkLoadLibsvm.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                ctypes.POINTER(ctypes.POINTER(ctypes.c_float)),
                                ctypes.POINTER(ctypes.POINTER(ctypes.c_int)), ctypes.POINTER(ctypes.c_int)]
    return r


def test_load_bin(tmp_path):
    A = np.random.default_rng(1).standard_normal((37, 12)).astype(np.float32)
    f = tmp_path / "x.f32"
    A.tofile(f)
    rc, out = load_bin(M.lib(), f, 12, 0)
    assert rc == 0 and np.array_equal(out, A)
    rc, out = load_bin(M.lib(), f, 12, 5)                 # a prefix of 5 rows
    assert rc == 0 and np.array_equal(out, A[:5])
    assert load_bin(M.lib(), f, 11, 0)[0] == M.MPK_ERR_INVALID     # not a whole number of rows
    assert load_bin(M.lib(), tmp_path / "missing", 12, 0)[0] == M.MPK_ERR_INVALID
    r = ref_lib()
    if r is not None:
        for d, mr in ((12, 0), (12, 5), (4, 7)):
            a, b = load_bin(M.lib(), f, d, mr), load_bin(r, f, d, mr)
            assert a[0] == b[0] and np.array_equal(a[1], b[1])


def test_load_libsvm(tmp_path):
    f = tmp_path / "x.svm"
    f.write_bytes(LIBSVM.encode())
    rc, P, L, nc = load_libsvm(M.lib(), f)
    assert rc == 0 and P.shape == (5, 7)
    want = np.zeros((5, 7), np.float32)
    want[0, [0, 2, 6]] = [0.5, -2.25, 1e-3]
    want[1, [1, 2]] = [4, 1.5]
    want[2, [6, 0]] = [8.0, -1]
    want[3, 3] = 0.125
    want[4, [4, 5]] = [3, -6]
    assert np.array_equal(P, want)
    assert list(L) == [0, 1, 0, 2, 1] and nc == 3        # classes 1, -1, 2 in order of first appearance
    empty = tmp_path / "e.svm"
    empty.write_text("# nothing\n\n")
    assert load_libsvm(M.lib(), empty)[0] == M.MPK_ERR_INVALID
    r = ref_lib()
    if r is not None:
        a, b = load_libsvm(M.lib(), f), load_libsvm(r, f)
        assert a[0] == b[0] and np.array_equal(a[1], b[1]) and np.array_equal(a[2], b[2]) and a[3] == b[3]
