"""Parity at the BASELINE configurations' own shapes, and the float16 overflow
edge cases of the reference's distance chain.

* config 4's assignment (float32, D=2048, K=1024: split-D, 3xTF32) on a
  16384-point sample, at the float32 label bar (the reference sweeps D up to
  4096, examples/test_assign_dtype_d.py:24);
* config 3 at full shape (N=2^22, K=128, Dirichlet-weighted GMM, float16) and
  config 2 at full shape (B=32, N=75600, K=1000, float16): one Lloyd
  iteration of the engine from given centroids.  Labels are checked against
  the oracle on a fixed sample of rows (the oracle gets the engine's x_sq);
  the centroids against the oracle's update of the engine's own labels over
  every point, so accumulation across all batch and tile boundaries is
  checked where it happens;
* float16 overflow: rows whose x_sq is inf, centroids whose c_sq is inf and
  cross products whose doubling overflows, so distances reach inf and NaN;
  the kernel must give torch.argmin's answer (the first NaN, else the first
  minimum) bit for bit.
"""
import numpy as np
import pytest
import torch

from _parity import assert_centroids, assert_labels
from oracle import kmeans_oracle as ko

pytestmark = pytest.mark.gpu

TD = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _dev(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(TD[dt])


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(scope="module")
def fk():
    import flash_kmeans
    return flash_kmeans


def test_cfg4_assignment_d2048_vs_oracle(fk):
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    rng = np.random.default_rng(404)
    N, K, D = 16384, 1024, 2048
    x = rng.standard_normal((1, N, D), dtype=np.float32)
    c = x[:, rng.integers(0, N, K)]                       # random-point init, as config 4
    xd = _dev(x, "float32")
    xsq = _ops.row_sqnorm(xd)
    got = euclid_assign_triton(xd, _dev(c, "float32"), xsq).cpu().numpy()
    want = ko.assign(x, c, _np(xsq), "float32")
    r = assert_labels(x, c, got, want, "float32", "config 4 D=2048")
    assert r["mismatches"] <= 2, r


def _engine_step(x_dev, c_dev, K):
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    B, N, D = x_dev.shape
    eng = LloydEngine(B, N, K, D, x_dev.dtype, "cuda")
    eng.load(x_dev, c_dev)
    eng.step()
    shift, code = eng.read_stat()
    assert code == 0
    return eng.ids.cpu().numpy(), _np(eng.c_nxt), shift, _np(eng.x_sq)


def _check_iteration(x, c0, ids, new, shift, x_sq, dt, sample_rows, what):
    B, N, D = x.shape
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(N, size=min(sample_rows, N), replace=False))
    xs = np.ascontiguousarray(x[:, rows])
    xq = np.ascontiguousarray(x_sq[:, rows])
    want = ko.assign(xs, c0, xq, dt)
    assert_labels(xs, c0, ids[:, rows], want, dt, what + " labels (row sample)", x_sq=xq)
    upd = ko.centroid_update(x, ids, c0, dt, exact_order=False)
    assert_centroids(new, upd, what + " centroids (oracle update of the engine's labels)")
    o_shift = ko.center_shift(upd, c0, dt)
    assert abs(shift - o_shift) <= 2e-3 * max(abs(o_shift), 1e-3) + 1e-6


def test_cfg3_full_shape_one_iteration(fk):
    """B=1, N=2^22, D=128, K=128 float16, 128-component GMM with Dirichlet(1)
    weights (skewed cluster sizes): narrow tiles, privatised accumulation."""
    rng = np.random.default_rng(303)
    N, K, D = 1 << 22, 128, 128
    x = ko.round_to(ko.gmm_points(rng, 1, N, D, 128, 3.0, dirichlet=True), "float16")
    c0 = ko.init_from_points(rng, x, K, replace=True)
    ids, new, shift, x_sq = _engine_step(_dev(x, "float16"), _dev(c0, "float16"), K)
    _check_iteration(x, c0, ids, new, shift, x_sq, "float16", 65536, "config 3")


def test_cfg2_full_shape_one_iteration(fk):
    """B=32, N=75600, D=128, K=1000 float16: the fused assign+accumulate kernel
    with CTA tile ranges crossing all 32 batch boundaries."""
    rng = np.random.default_rng(202)
    B, N, K, D = 32, 75600, 1000, 128
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), "float16")
    c0 = ko.init_from_points(rng, x, K, replace=True)
    ids, new, shift, x_sq = _engine_step(_dev(x, "float16"), _dev(c0, "float16"), K)
    _check_iteration(x, c0, ids, new, shift, x_sq, "float16", 3000, "config 2")


def _overflow_inputs(seed, B, N, K, D, dt):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, N, D), dtype=np.float32)
    scale = np.ones((B, N, 1), np.float32)
    scale[:, N // 3:2 * N // 3] = 30.0      # x_sq finite, some 2 x.c beyond float16's range
    scale[:, 2 * N // 3:] = 100.0           # x_sq = inf
    x = ko.round_to(x * scale, dt)
    c = rng.standard_normal((B, K, D), dtype=np.float32)
    big = rng.choice(K, size=K // 4, replace=False)
    c[:, big] *= np.float32(100.0)          # c_sq = inf
    return x, ko.round_to(c, dt)


@pytest.mark.parametrize("K", [64, 300, 1000])
def test_float16_overflow_matches_argmin(fk, K):
    """inf and NaN distances: labels equal the oracle's (torch.argmin's rules)
    bit for bit, through the labels-only kernel and fk_assign_accumulate
    (privatised for K=64 and 300, fused for K=1000)."""
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    B, N, D = 2, 3000, 64
    x, c = _overflow_inputs(K, B, N, K, D, "float16")
    xd, cd = _dev(x, "float16"), _dev(c, "float16")
    xsq = _ops.row_sqnorm(xd)
    assert torch.isinf(xsq).any()
    with np.errstate(all="ignore"):
        want = ko.assign(x, c, _np(xsq), "float16")
    got = euclid_assign_triton(xd, cd, xsq).cpu().numpy()
    np.testing.assert_array_equal(got, want)
    counts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
    sums = torch.zeros((B, K, D), dtype=torch.float32, device="cuda")
    out = torch.empty((B, N), dtype=torch.int32, device="cuda")
    _ops.assign_accumulate(xd, cd, xsq, out, counts, sums)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    np.testing.assert_array_equal(counts.cpu().numpy(),
                                  np.stack([np.bincount(want[b], minlength=K) for b in range(B)]))
