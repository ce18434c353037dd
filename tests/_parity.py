"""Parity checkers shared by the CPU and GPU tests.

The bar (from the project's north star):

* labels are bit-identical except where the two candidate centroids' exact
  (float64) squared distances differ by less than ``LABEL_TOL[dtype]``
  relative, and such near-tie mismatches stay under 0.1 % of points (at
  least one is allowed, so a case under 1000 points is not failed by a single
  near-tie that the tensor core's summation order legitimately breaks the
  other way);
* for the dot-product (cosine / dot k-means) labels the gap is the exact score
  difference ``|x.c_a - x.c_b|`` relative to ``||x|| max(||c_a||, ||c_b||)``,
  with the same tolerances;
* for 16-bit Euclidean labels a mismatch is also excused as a summation-order
  tie when the float16 / bfloat16 rounding of a cross product x.c sits so close
  to a rounding boundary that a float32 sum in another order (bounded by
  D * 2^-24 * sum|x_i c_i|) rounds it the other way, and with some such
  rounding the reference's distance chain ranks the kernel's centroid no worse
  (the chain quantises distances at the unit of x_sq, which for large x_sq is
  far above the 1e-3 relative bar); these count against the same 0.1 % budget;
* centroids agree within 1e-3 relative per centroid:
  ``||dc_k|| <= 1e-3 * max(||c_k||, 1e-3 * max_j ||c_j||)``.
"""
from __future__ import annotations

import numpy as np

from oracle import kmeans_oracle as ko

LABEL_TOL = {"float16": 1e-3, "bfloat16": 1e-3, "float32": 1e-5}
MAX_EXCUSED_FRAC = 1e-3
CENTROID_RTOL = 1e-3


def _order_ties(xs, ca, cb, dtype, xsq):
    """Boolean per row: a float32 summation order of the cross products exists
    under which the reference's 16-bit chain gives candidate a (the kernel's)
    a distance no larger than candidate b's (see the module docstring)."""
    D = xs.shape[-1]

    def chain_range(c):
        prod = xs * c
        cross = prod.sum(-1)
        eps = D * 2.0 ** -24 * np.abs(prod).sum(-1)
        csq = ko.row_sqnorm(c[None].astype(np.float32), dtype)[0]
        out = []
        with np.errstate(all="ignore"):
            for cr in (cross - eps, cross + eps):
                rc = ko.round_to(cr, dtype)
                two = ko.round_to(2.0 * rc, dtype)
                t = ko.round_to(xsq - two, dtype)
                out.append(ko.round_to(t + csq, dtype))
        return np.minimum(*out), np.maximum(*out)

    a_lo, _ = chain_range(ca)
    _, b_hi = chain_range(cb)
    return a_lo <= b_hi


def label_report(x, centroids, got, want, dtype, metric="euclid", x_sq=None):
    """Compare two labelings of x against centroids; returns a dict.
    ``metric`` is "euclid" (nearest centroid) or "dot" (largest dot product);
    ``x_sq`` (B, N) is the kernel's x_sq in ``dtype`` (default: the oracle's)."""
    got = np.asarray(got).astype(np.int64).reshape(np.asarray(want).shape)
    want = np.asarray(want).astype(np.int64)
    mism = got != want
    n = want.size
    out = dict(n=n, mismatches=int(mism.sum()), excused=0, bad=0, worst_gap=0.0)
    if not mism.any():
        return out
    x = np.asarray(x, np.float64)
    c = np.asarray(centroids, np.float64)
    bi, ni = np.nonzero(mism)
    xs = x[bi, ni]
    ca = c[bi, got[bi, ni]]
    cb = c[bi, want[bi, ni]]
    if metric == "dot":
        sa = (xs * ca).sum(-1)
        sb = (xs * cb).sum(-1)
        scale = np.linalg.norm(xs, axis=-1) * np.maximum(np.linalg.norm(ca, axis=-1),
                                                         np.linalg.norm(cb, axis=-1))
        gap = np.abs(sa - sb) / (scale + 1e-30)
    else:
        da = ((xs - ca) ** 2).sum(-1)
        db = ((xs - cb) ** 2).sum(-1)
        gap = np.abs(da - db) / (np.minimum(np.abs(da), np.abs(db)) + 1e-3)
    tol = LABEL_TOL[dtype]
    near = gap < tol
    order = np.zeros_like(near)
    if metric == "euclid" and dtype in ("float16", "bfloat16") and (~near).any():
        xq = ko.row_sqnorm(np.asarray(x, np.float32), dtype) if x_sq is None else np.asarray(x_sq)
        order = ~near & _order_ties(xs, ca, cb, dtype, np.asarray(xq, np.float64)[bi, ni])
    out["excused"] = int((near | order).sum())
    out["order_ties"] = int(order.sum())
    out["bad"] = int((~(near | order)).sum())
    out["worst_gap"] = float(gap.max())
    return out


def assert_labels(x, centroids, got, want, dtype, what="", metric="euclid", x_sq=None):
    r = label_report(x, centroids, got, want, dtype, metric, x_sq=x_sq)
    assert r["bad"] == 0, f"{what}: {r['bad']} label mismatches beyond near-tie tolerance {r}"
    allowed = max(1, int(np.ceil(MAX_EXCUSED_FRAC * r["n"])))
    assert r["excused"] <= allowed, f"{what}: too many near-tie mismatches {r}"
    return r


def centroid_errors(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    nrm = np.linalg.norm(want, axis=-1)
    floor = 1e-3 * nrm.max(axis=-1, keepdims=True) if nrm.size else nrm
    denom = np.maximum(nrm, floor)
    denom = np.where(denom > 0, denom, 1.0)
    return np.linalg.norm(got - want, axis=-1) / denom


def assert_centroids(got, want, what="", rtol=CENTROID_RTOL, skip=None):
    err = centroid_errors(got, want)
    if skip is not None:
        err = np.where(skip, 0.0, err)
    worst = float(err.max()) if err.size else 0.0
    assert worst <= rtol, f"{what}: centroid rel error {worst:.3e} > {rtol}"
    return worst


def clusters_touched(labels_a, labels_b, K):
    """Boolean (B, K): clusters whose membership differs between labelings."""
    a = np.asarray(labels_a).astype(np.int64)
    b = np.asarray(labels_b).astype(np.int64)
    B = a.shape[0]
    touched = np.zeros((B, K), dtype=bool)
    for i in range(B):
        m = a[i] != b[i]
        touched[i, a[i][m]] = True
        touched[i, b[i][m]] = True
    return touched


__all__ = ["label_report", "assert_labels", "centroid_errors", "assert_centroids",
           "clusters_touched", "LABEL_TOL", "ko"]
