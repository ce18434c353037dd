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


# --------------------------------------------------------------------------
# cosine / dot-product k-means
# --------------------------------------------------------------------------
def _ulps_apart(a, b, dtype):
    """Elementwise distance in units of the dtype's spacing at |b|."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    mant = {"float16": 10, "bfloat16": 7, "float32": 23}[dtype]
    spacing = np.exp2(np.floor(np.log2(np.maximum(np.abs(b), 1e-30))) - mant)
    return np.abs(a - b) / spacing


@pytest.mark.parametrize("spec", cases.NORMALIZE_CASES, ids=lambda s: s["name"])
def test_oracle_normalize_matches_reference(spec):
    x = cases.normalize_inputs(spec)
    g = _load(spec["name"])
    assert abs(float(g["checksum"]) - cases.checksum(x)) < 1e-3 * max(1.0, abs(float(g["checksum"])))
    y = ko.normalize_rows(x, spec["dtype"])
    want = g["y"]
    # the zero row: 0/eps = 0 where eps survives the dtype, 0/0 = NaN in float16
    np.testing.assert_array_equal(np.isnan(y), np.isnan(want))
    if spec["dtype"] == "float16":
        assert np.isnan(want[0, 5]).all()
    else:
        assert (want[0, 5] == 0).all()
    ok = ~np.isnan(want)
    # the norm's float32 summation order may move a quotient by a unit (two in
    # float32, where the norm itself is not rounded to a coarser type)
    u = _ulps_apart(y[ok], want[ok], spec["dtype"])
    assert u.max() <= (2.0 if spec["dtype"] == "float32" else 1.0), u.max()
    assert (u > 0).mean() < (0.3 if spec["dtype"] == "float32" else 0.01)


@pytest.mark.parametrize("spec", cases.SIM_ASSIGN_CASES, ids=lambda s: s["name"])
def test_oracle_assign_dot_matches_reference(spec):
    x, c = cases.sim_assign_inputs(spec)
    g = _load(spec["name"])
    assert abs(float(g["checksum"]) - cases.checksum(x, c)) < 1e-3 * max(1.0, abs(float(g["checksum"])))
    dt = spec["dtype"]
    if spec["cosine"]:
        x, c = ko.normalize_rows(x, dt), ko.normalize_rows(c, dt)
    ids = ko.assign_dot(x, c)
    r = assert_labels(x, c, ids, g["ids"], dt, spec["name"], metric="dot")
    assert r["mismatches"] <= max(1, r["n"] // 10000), r
    if spec.get("neg"):
        # every winning score is negative: the argmax must not start from zero
        assert (ko.scores_f64(x, c).max(-1) < 0).all()


@pytest.mark.parametrize("spec", cases.SIM_UPDATE_CASES, ids=lambda s: s["name"])
@pytest.mark.parametrize("exact", [True, False])
def test_oracle_cosine_update_matches_reference(spec, exact):
    x, ids, old = cases.sim_update_inputs(spec)
    g = _load(spec["name"])
    dt = spec["dtype"]
    xs = ko.normalize_rows(x, dt)
    new = ko.centroid_update_cosine(xs, ids, old, dt, exact_order=exact)
    assert_centroids(new, g["centroids"], spec["name"])
    if dt == "float32":
        # inputs normalised by a float32 norm of another summation order: the
        # means agree to float32 accuracy per row, not per element
        assert_centroids(new, g["centroids"], spec["name"], rtol=1e-5)
    else:
        u = _ulps_apart(new, g["centroids"], dt)
        assert u.max() <= 1.0, u.max()
    # every row is unit length to the dtype's rounding, empty clusters included
    nrm = np.linalg.norm(new.astype(np.float64), axis=-1)
    assert np.abs(nrm - 1).max() < {"float16": 2e-3, "bfloat16": 1e-2, "float32": 1e-6}[dt]


@pytest.mark.parametrize("spec", cases.SIM_LLOYD_CASES, ids=lambda s: s["name"])
def test_oracle_similarity_lloyd_matches_reference(spec):
    x, c0 = cases.sim_lloyd_inputs(spec)
    g = _load(spec["name"])
    dt, cosine = spec["dtype"], spec["cosine"]
    assert abs(float(g["checksum"]) - cases.checksum(x, c0)) < 1e-6 * abs(float(g["checksum"])) + 1e-3
    xs = ko.normalize_rows(x, dt) if cosine else ko.round_to(x, dt)
    cent = ko.normalize_rows(c0, dt) if cosine else ko.round_to(c0, dt)
    u = _ulps_apart(cent, g["init"], dt)
    assert u.max() <= (2.0 if dt == "float32" else 1.0)
    cent = g["init"]
    # teacher-forced trace: each step starts from the reference's centroids
    for t in range(g["trace_ids"].shape[0]):
        ids = ko.assign_dot(xs, cent)
        assert_labels(xs, cent, ids, g["trace_ids"][t], dt, f"{spec['name']} iter {t}", metric="dot")
        new = ko.centroid_update_cosine(xs, g["trace_ids"][t], cent, dt)
        assert_centroids(new, g["trace_centroids"][t], f"{spec['name']} iter {t}")
        shift = ko.center_shift(g["trace_centroids"][t], cent, dt)
        assert abs(shift - float(g["trace_shifts"][t])) <= 1e-3 * max(1.0, abs(shift))
        cent = g["trace_centroids"][t]
    # the driver, free-running, reproduces the chain's labels
    hist = []
    ids, cf, n_it = ko.batch_kmeans_similarity(x, spec["K"], spec["iters"], 0.0, init_centroids=c0,
                                               dtype=dt, cosine=cosine, history=hist)
    assert n_it == spec["iters"]
    r = assert_labels(xs, hist[-1][0], ids, g["trace_ids"][-1], dt, spec["name"], metric="dot")
    assert r["mismatches"] <= max(2, r["n"] // 2000)
    touched = clusters_touched(ids, g["trace_ids"][-1], spec["K"])
    assert_centroids(cf, g["trace_centroids"][-1], spec["name"], skip=touched)
