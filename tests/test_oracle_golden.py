"""Pin the numpy oracle against golden vectors made by the reference itself.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py,
which runs the reference's torch_fallback functions on the seeded inputs of
tests/golden/cases.py.  CPU only.
"""
import numpy as np
import pytest

import cases
from _parity import assert_centroids, assert_labels, clusters_touched
from oracle import kmeans_oracle as ko


def _load(name):
    return np.load(cases.path(name))


@pytest.mark.parametrize("spec", cases.ASSIGN_CASES, ids=lambda s: s["name"])
def test_oracle_assign_matches_reference(spec):
    x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
    g = _load(spec["name"])
    assert abs(float(g["checksum"]) - cases.checksum(x, c, xsq)) < 1e-3 * max(1.0, abs(float(g["checksum"])))
    ids = ko.assign(x, c, xsq, spec["dtype"], xsq_dtype=xsq_dtype)
    r = assert_labels(x, c, ids, g["ids"], spec["dtype"], spec["name"])
    # the restatement follows the reference op by op: expect (near-)exact equality
    assert r["mismatches"] <= max(1, r["n"] // 10000), r


def test_oracle_assign_ties_lowest_index():
    spec = next(s for s in cases.ASSIGN_CASES if s.get("dup"))
    x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
    ids = ko.assign(x, c, xsq, spec["dtype"])
    assert ids.max() < spec["K"] // 2, "duplicated centroids must resolve to the first copy"
    np.testing.assert_array_equal(ids, _load(spec["name"])["ids"])


@pytest.mark.parametrize("spec", cases.UPDATE_CASES, ids=lambda s: s["name"])
@pytest.mark.parametrize("exact", [True, False])
def test_oracle_update_matches_reference(spec, exact):
    x, ids, old = cases.update_inputs(spec)
    g = _load(spec["name"])
    new = ko.centroid_update(x, ids, old, spec["dtype"], exact_order=exact)
    assert_centroids(new, g["centroids"], spec["name"])
    if exact:
        # same summation order and rounding chain as index_add_: bit-identical
        np.testing.assert_array_equal(new, g["centroids"])
    # empty clusters keep the old centroid exactly
    cnt = np.stack([np.bincount(ids[b], minlength=spec["K"]) for b in range(spec["B"])])
    np.testing.assert_array_equal(new[cnt == 0], ko.round_to(old, spec["dtype"])[cnt == 0])


@pytest.mark.parametrize("spec", cases.LLOYD_CASES, ids=lambda s: s["name"])
def test_oracle_lloyd_matches_reference(spec):
    x, c0 = cases.lloyd_inputs(spec)
    g = _load(spec["name"])
    dt = spec["dtype"]
    assert abs(float(g["checksum"]) - cases.checksum(x, c0)) < 1e-6 * abs(float(g["checksum"])) + 1e-3
    # teacher-forced per-iteration trace (the reference's own chain)
    xq = ko.round_to(x, dt)
    x_sq = ko.row_sqnorm(xq, dt)
    cent = ko.round_to(c0, dt)
    for t in range(g["trace_ids"].shape[0]):
        new, shift, ids = ko.lloyd_iter(xq, x_sq, cent, dt)
        assert_labels(xq, cent, ids, g["trace_ids"][t], dt, f"{spec['name']} iter {t}")
        assert abs(shift - float(g["trace_shifts"][t])) <= 1e-3 * max(1.0, abs(shift))
        cent = new
    # full driver, free-running
    ids, cent, n_it = ko.batch_kmeans_euclid(x, spec["K"], spec["iters"], spec["tol"],
                                             init_centroids=c0, dtype=dt)
    assert n_it == int(g["n_iters"])
    r = assert_labels(xq, cent, ids, g["ids"], dt, spec["name"])
    touched = clusters_touched(ids, g["ids"], spec["K"])
    assert_centroids(cent, g["centroids"], spec["name"], skip=touched)
    assert r["mismatches"] <= max(2, r["n"] // 2000)


def test_oracle_tol_break_returns_pre_update_centroids():
    spec = next(s for s in cases.LLOYD_CASES if s["tol"] > 0)
    x, c0 = cases.lloyd_inputs(spec)
    hist = []
    ids, cent, n_it = ko.batch_kmeans_euclid(x, spec["K"], spec["iters"], spec["tol"],
                                             init_centroids=c0, dtype=spec["dtype"], history=hist)
    assert n_it < spec["iters"]
    cin, ids_last, _, shift = hist[-1]
    np.testing.assert_array_equal(cent, cin)
    np.testing.assert_array_equal(ids, ids_last)
    assert shift < spec["tol"] * 1.01
