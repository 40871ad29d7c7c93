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


# ------------------------------------------------------------- noise floor --

def end_of_run(P, base, run):
    """Agreement of one end-of-run result `run` = (labels, C, inertia) with the reference's
    `base` run: label agreement, relative Frobenius distance of the centroids and relative
    inertia difference.  (The centroids differ between runs, so a mismatch is not a
    near-tie on one set of centroids; these three numbers are what end-of-run parity
    can be read from.)"""
    lb, Cb, ib = base
    la, Ca, ia = run
    Cb64 = np.asarray(Cb, np.float64)
    return {"agree": float((np.asarray(la) == np.asarray(lb)).mean()),
            "C_rel": float(np.linalg.norm(np.asarray(Ca, np.float64) - Cb64) / np.linalg.norm(Cb64)),
            "inertia_rel": abs(float(ia) - float(ib)) / abs(float(ib))}


def within_floor(ours, floors, slack=1.25):
    """True when `ours` (an end_of_run dict against the reference) meets the north-star bar --
    labels >= 99.99 %, centroids and inertia within 1e-5 relative -- or, where the reference
    does not meet it against itself (`floors`: end_of_run dicts of the reference's own
    variant runs against its base run), is no further from the reference than those runs
    are, up to `slack` times their largest distance.  Returns (ok, bar) with the bar used."""
    worst = {"disagree": max(1.0 - f["agree"] for f in floors),
             "C_rel": max(f["C_rel"] for f in floors),
             "inertia_rel": max(f["inertia_rel"] for f in floors)}
    bar = {"disagree": max(1e-4, slack * worst["disagree"]),
           "C_rel": max(1e-5, slack * worst["C_rel"]),
           "inertia_rel": max(1e-5, slack * worst["inertia_rel"])}
    ok = (1.0 - ours["agree"] <= bar["disagree"] and ours["C_rel"] <= bar["C_rel"]
          and ours["inertia_rel"] <= bar["inertia_rel"])
    return ok, bar
