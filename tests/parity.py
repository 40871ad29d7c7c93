"""Label-parity adjudication shared by the test files.

Two FP32 evaluations of the reference's distance ``D(j) = ||c_j||^2 - 2 x.c_j``
(kmeans/include/mpkmeans/mpkmeans.h:13-21: the ||x||^2 term is dropped) with
different summation orders may pick different centroids only where D is tied
to FP32 precision.  Each mismatch between labels ``a`` and ``r`` on the same
centroids is scored two ways:

  gap32  |E(a) - E(r)| / max(|E(a)|, |E(r)|), E(j) = ||c_j||^2 - 2 x.c_j taken
         exactly (FP64) from the FP32 inputs, ||c_j||^2 as the reference forms
         it: the FP32 distance gap the reference's own argmin compares;
  gap64  |D64(a) - D64(r)| / max(D64(a), D64(r)), D64 the direct-formula
         ||x - c||^2 in FP64: the gap in true distance.

gap32 < 1e-5 means both labels are valid FP32 answers.  gap64 is the stricter
reading; it is only meaningful where the expanded formula does not cancel
(it fails by design on the offset/cancellation configuration, where the FP32
reference itself is off by up to ~0.5% in true distance).
"""
import numpy as np

import oracle as O


def gaps(P, C, la, lr):
    idx = np.nonzero(la != lr)[0]
    if len(idx) == 0:
        return idx, np.zeros(0), np.zeros(0)
    d64a = O.dist64_pairs(P, C, idx, la[idx])
    d64r = O.dist64_pairs(P, C, idx, lr[idx])
    cn = O.row_norms(C).astype(np.float64)
    X = P[idx].astype(np.float64)
    ea = cn[la[idx]] - 2.0 * np.einsum("ij,ij->i", X, C[la[idx]].astype(np.float64))
    er = cn[lr[idx]] - 2.0 * np.einsum("ij,ij->i", X, C[lr[idx]].astype(np.float64))
    g32 = np.abs(ea - er) / np.maximum(np.maximum(np.abs(ea), np.abs(er)), 1e-300)
    g64 = np.abs(d64a - d64r) / np.maximum(np.maximum(d64a, d64r), 1e-300)
    return idx, g32, g64


def summary(P, C, la, lr):
    idx, g32, g64 = gaps(P, C, la, lr)
    return {"n": int(len(la)), "mismatches": int(len(idx)), "agree": float(1.0 - len(idx) / max(1, len(la))),
            "max_gap32": float(g32.max()) if len(idx) else 0.0, "max_gap64": float(g64.max()) if len(idx) else 0.0}
