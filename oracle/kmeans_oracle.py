"""CPU restatement (numpy) of Flash-KMeans' pure-torch Lloyd path.

TEST INFRASTRUCTURE ONLY.  This module is the parity checker for the CUDA
path of ``flash_kmeans`` (the package under ``flash-kmeans_b200/``).  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` may
import it; the product path never does.

It restates, operation by operation, the reference's torch fallback
(``flash_kmeans/torch_fallback.py``), which is the parity oracle named by the
project's north star, including that path's rounding: every tensor operation
in the reference produces a tensor of the input dtype, so a float16 run rounds
after each elementwise step.  Values are carried as float32 arrays whose
entries are exactly representable in the emulated dtype (float16, bfloat16 or
float32); ``_round`` performs the per-step rounding.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
``torch_fallback`` functions on seeded inputs and stores their outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module against
every stored vector.

Reference citations are ``path:line`` inside the reference project.
"""
from __future__ import annotations

import numpy as np

DTYPES = ("float32", "float16", "bfloat16")


# --------------------------------------------------------------------------
# rounding helpers
# --------------------------------------------------------------------------
def _round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def round_to(a, dtype: str) -> np.ndarray:
    """Round ``a`` to ``dtype`` and return it as float32 values."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == "float32":
        return a
    if dtype == "float16":
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return _round_bf16(a)
    raise ValueError(f"unsupported dtype {dtype!r}")


def promote(a: str, b: str) -> str:
    """torch type promotion between two floating dtypes of equal category."""
    if a == b:
        return a
    return "float32"  # f16 x bf16 or any x f32 promotes to f32


# --------------------------------------------------------------------------
# x_sq / cent_sq
# --------------------------------------------------------------------------
def row_sqnorm(x: np.ndarray, dtype: str) -> np.ndarray:
    """``(x ** 2).sum(dim=-1)`` evaluated in ``dtype``.

    torch_fallback.py:154 (x_sq) and torch_fallback.py:23 (cent_sq); the
    Triton driver does the same in kmeans_triton_impl.py:84-87.  ``x ** 2`` is
    rounded per element to ``dtype``; the sum accumulates in float32 (torch's
    accumulation type for half types) and is rounded once at the end.
    """
    sq = round_to(np.square(np.asarray(x, dtype=np.float32)), dtype)
    return round_to(sq.sum(axis=-1, dtype=np.float32), dtype)


# --------------------------------------------------------------------------
# assignment
# --------------------------------------------------------------------------
def assign(x, centroids, x_sq, dtype: str, xsq_dtype: str | None = None,
           chunk_size_N: int = 32768, chunk_size_K: int = 1024) -> np.ndarray:
    """Nearest centroid per point, restating torch_fallback.py:4-52.

    ``cent_sq`` is computed in the centroid dtype (torch_fallback.py:23).  For
    each (N-chunk, K-chunk) the distance is
    ``x_sq[:, :, None] - 2 * bmm(x, c^T) + cent_sq[:, None, :]``
    (torch_fallback.py:41-45): the bmm result is rounded to ``dtype`` (float32
    accumulation, one rounding), ``2 *`` is a separate op in that dtype (exact
    unless it overflows to inf, e.g. |x.c| > 32752 in float16), the
    subtraction and the addition each round to the promoted dtype.  There is
    no clamp.  The distances land in a float32 buffer (torch_fallback.py:33)
    and ``argmin`` takes the first minimum, or the first NaN if there is one
    (torch_fallback.py:50; numpy's argmin does the same).  Returns int32 (B, N).
    """
    x = np.asarray(x, dtype=np.float32)
    c = np.asarray(centroids, dtype=np.float32)
    xs = np.asarray(x_sq, dtype=np.float32)
    xsq_dtype = xsq_dtype or dtype
    B, N, D = x.shape
    K = c.shape[1]
    assert c.shape == (B, K, D), "centroids shape mismatch"
    assert xs.shape == (B, N), "x_sq shape mismatch"
    cent_sq = row_sqnorm(c, dtype)
    t_dtype = promote(xsq_dtype, dtype)
    out = np.empty((B, N), dtype=np.int32)
    for n0 in range(0, N, chunk_size_N):
        n1 = min(n0 + chunk_size_N, N)
        dists = np.empty((B, n1 - n0, K), dtype=np.float32)
        for k0 in range(0, K, chunk_size_K):
            k1 = min(k0 + chunk_size_K, K)
            cross = np.matmul(x[:, n0:n1, :], np.swapaxes(c[:, k0:k1, :], 1, 2))
            cross = round_to(cross, dtype)
            with np.errstate(over="ignore", invalid="ignore"):
                two = round_to(2.0 * cross, dtype)
                t = round_to(xs[:, n0:n1, None] - two, t_dtype)
                dists[:, :, k0:k1] = round_to(t + cent_sq[:, None, k0:k1], t_dtype)
        out[:, n0:n1] = np.argmin(dists, axis=-1)
    return out


def distances_f64(x, centroids) -> np.ndarray:
    """Exact squared distances in float64, used to classify near-ties."""
    x = np.asarray(x, dtype=np.float64)
    c = np.asarray(centroids, dtype=np.float64)
    return ((x * x).sum(-1)[:, :, None] + (c * c).sum(-1)[:, None, :]
            - 2.0 * np.matmul(x, np.swapaxes(c, 1, 2)))


# --------------------------------------------------------------------------
# centroid update
# --------------------------------------------------------------------------
def centroid_sums(x, ids, K: int, exact_order: bool = True):
    """float32 per-cluster sums and counts (torch_fallback.py:90-97).

    ``index_add_`` on CPU adds rows in index order; ``np.add.at`` does the
    same.  ``exact_order=False`` sums in float64 and rounds once, which is
    faster for large inputs and agrees to float32 rounding.
    """
    x = np.asarray(x, dtype=np.float32)
    ids = np.asarray(ids).astype(np.int64)
    B, N, D = x.shape
    sums = np.zeros((B, K, D), dtype=np.float32)
    cnts = np.zeros((B, K), dtype=np.float32)
    for b in range(B):
        if exact_order:
            np.add.at(sums[b], ids[b], x[b])
        else:
            order = np.argsort(ids[b], kind="stable")
            sid = ids[b][order]
            bounds = np.flatnonzero(np.diff(sid)) + 1
            starts = np.concatenate(([0], bounds))
            if N:
                seg = np.add.reduceat(x[b][order].astype(np.float64), starts, axis=0)
                sums[b][sid[starts]] = seg.astype(np.float32)
        cnts[b] = np.bincount(ids[b], minlength=K)[:K].astype(np.float32)
    return sums, cnts


def finalize(sums, cnts, old_centroids, dtype: str):
    """Mean, keep-old-if-empty and cast (torch_fallback.py:101-108)."""
    cnt = np.asarray(cnts, dtype=np.float32)[..., None]
    empty = cnt == 0
    mean = np.asarray(sums, dtype=np.float32) / np.maximum(cnt, 1.0)
    new = np.where(empty, np.asarray(old_centroids, dtype=np.float32), mean)
    return round_to(new, dtype)


def centroid_update(x, ids, old_centroids, dtype: str, exact_order: bool = True):
    """``_centroid_update_torch_native`` (torch_fallback.py:72-108)."""
    K = np.asarray(old_centroids).shape[1]
    sums, cnts = centroid_sums(x, ids, K, exact_order=exact_order)
    return finalize(sums, cnts, old_centroids, dtype)


def center_shift(new, old, dtype: str) -> float:
    """``(new - old).norm(dim=-1).max()`` in ``dtype`` (torch_fallback.py:133).

    The difference rounds per element; the norm accumulates in float32 and
    rounds once.
    """
    diff = round_to(np.asarray(new, np.float32) - np.asarray(old, np.float32), dtype)
    norm = round_to(np.sqrt((diff.astype(np.float32) ** 2).sum(-1, dtype=np.float32)), dtype)
    return float(norm.max()) if norm.size else 0.0


def shift_below_tol(shift: float, tol: float, dtype: str) -> bool:
    """``center_shift < tol`` with ``tol`` rounded to the shift's dtype, as a
    0-dim tensor compared with a Python float does (kmeans_triton_impl.py:111)."""
    return bool(np.float32(shift) < round_to(np.float32(tol), dtype))


# --------------------------------------------------------------------------
# Lloyd drivers
# --------------------------------------------------------------------------
def lloyd_iter(x, x_sq, centroids, dtype: str, exact_order: bool = True):
    """``_euclid_iter_torch_naive`` (torch_fallback.py:111-135)."""
    ids = assign(x, centroids, x_sq, dtype)
    new = centroid_update(x, ids, centroids, dtype, exact_order=exact_order)
    return new, center_shift(new, centroids, dtype), ids


def batch_kmeans_euclid(x, n_clusters: int, max_iters: int = 100, tol: float = 0.0,
                        init_centroids=None, dtype: str = "float32",
                        exact_order: bool = True, history: list | None = None):
    """``batch_kmeans_Euclid_torch_native`` (torch_fallback.py:137-178).

    Returns ``(cluster_ids int32 (B,N), centroids (B,K,D), n_iters)``.  On a
    tolerance break the centroids returned are the ones the last assignment
    used, i.e. before that iteration's update (torch_fallback.py:172-178).
    ``init_centroids`` is required (random init lives in the caller).
    When ``history`` is a list, the per-iteration ``(centroids_in, ids,
    centroids_new, shift)`` tuples are appended to it.
    """
    x = round_to(x, dtype)
    B, N, D = x.shape
    if init_centroids is None:
        raise ValueError("the oracle needs explicit init_centroids")
    centroids = round_to(np.asarray(init_centroids, np.float32).reshape(B, n_clusters, D), dtype)
    x_sq = row_sqnorm(x, dtype)
    ids = None
    it = 0
    for it in range(max_iters):
        new, shift, ids = lloyd_iter(x, x_sq, centroids, dtype, exact_order=exact_order)
        if history is not None:
            history.append((centroids, ids, new, shift))
        if shift_below_tol(shift, tol, dtype):
            break
        centroids = new
    return ids, centroids, it + 1


def kmeans_large_n(x, n_clusters: int, max_iters: int = 100, tol: float = 0.0,
                   init_centroids=None, dtype: str = "float32", exact_order: bool = False):
    """Semantics of ``kmeans_largeN`` (kmeans_large.py:33-285) on one host.

    Assignment and update are the batched ones on the (1, N, D) view; the
    difference from ``batch_kmeans_euclid`` is the tolerance break, which
    returns the NEW centroids (kmeans_large.py:251-258, :278) together with
    the labels of the last assignment.  Returns ``(ids (N,), centroids (K,D))``.
    """
    x = round_to(np.asarray(x, np.float32)[None], dtype)
    K = n_clusters
    c = round_to(np.asarray(init_centroids, np.float32).reshape(1, K, -1), dtype)
    x_sq = row_sqnorm(x, dtype)
    ids = None
    new = c
    for _ in range(max_iters):
        new, shift, ids = lloyd_iter(x, x_sq, c, dtype, exact_order=exact_order)
        if shift_below_tol(shift, tol, dtype):
            break
        c = new
    return ids[0], new[0]


# --------------------------------------------------------------------------
# cosine / dot-product k-means
# --------------------------------------------------------------------------
def normalize_rows(x, dtype: str) -> np.ndarray:
    """``F.normalize(x, p=2, dim=-1)`` in ``dtype`` (kmeans_triton_impl.py:135,148).

    The norm accumulates in float32 (here float64, then rounded to float32) and
    rounds to the dtype; it is clamped below by eps = 1e-12 taken in the dtype
    (0 for float16); every element is divided in float32 and rounded.
    """
    x = np.asarray(x, np.float32)
    ss = (x.astype(np.float64) ** 2).sum(-1, keepdims=True)
    norm = round_to(np.sqrt(ss).astype(np.float32), dtype)
    eps = round_to(np.float32(1e-12), dtype)
    den = np.maximum(norm, eps)
    with np.errstate(divide="ignore", invalid="ignore"):
        return round_to(x / den, dtype)


def scores_f64(x, centroids) -> np.ndarray:
    """Exact (float64) dot products x . c^T per batch."""
    x = np.asarray(x, np.float64)
    c = np.asarray(centroids, np.float64)
    return np.einsum("bnd,bkd->bnk", x, c)


def assign_dot(x, centroids) -> np.ndarray:
    """Largest dot product, lowest index on ties: the reference's own check of
    ``cosine_assign_triton`` (examples/test_assign_dtype_d.py:101-106, argmax
    of a float32 einsum), and the einsum/argmax stated in _cosine_iter
    (kmeans_triton_impl.py:20-23).  Scores are exact here; the float32 scores
    of a kernel differ only on near-ties, which the parity bar excuses."""
    return scores_f64(x, centroids).argmax(-1).astype(np.int32)


def finalize_normalized(sums, cnts, old_centroids, dtype: str):
    """Mean, keep-old-if-empty, F.normalize in float32, cast: the mode='cosine'
    finalize of ``_centroid_update_torch_native`` (torch_fallback.py:101-109)."""
    cnt = np.asarray(cnts, dtype=np.float32)[..., None]
    empty = cnt == 0
    mean = np.asarray(sums, dtype=np.float32) / np.maximum(cnt, 1.0)
    new = np.where(empty, np.asarray(old_centroids, dtype=np.float32), mean).astype(np.float32)
    norm = np.sqrt((new.astype(np.float64) ** 2).sum(-1, keepdims=True)).astype(np.float32)
    return round_to(new / np.maximum(norm, np.float32(1e-12)), dtype)


def centroid_update_cosine(x, ids, old_centroids, dtype: str, exact_order: bool = True):
    """``_centroid_update_torch_native(..., mode='cosine')`` (torch_fallback.py:72-109)."""
    K = np.asarray(old_centroids).shape[1]
    sums, cnts = centroid_sums(x, ids, K, exact_order=exact_order)
    return finalize_normalized(sums, cnts, old_centroids, dtype)


def batch_kmeans_similarity(x, n_clusters: int, max_iters: int = 100, tol: float = 0.0,
                            init_centroids=None, dtype: str = "float32", cosine: bool = True,
                            exact_order: bool = True, history: list | None = None):
    """``batch_kmeans_Cosine`` (cosine=True, kmeans_triton_impl.py:118-158) and
    ``batch_kmeans_Dot`` (cosine=False, :161-188): x (and the initial
    centroids) normalised for cosine; each iteration assigns by the largest dot
    product and takes the normalised cluster means (both use the cosine
    update); the tolerance break returns the centroids of the last assignment.
    ``init_centroids`` (B, K, D) is required; ``history`` as in
    ``batch_kmeans_euclid``."""
    x = round_to(x, dtype)
    B, N, D = x.shape
    if init_centroids is None:
        raise ValueError("the oracle needs explicit init_centroids")
    xs = normalize_rows(x, dtype) if cosine else x
    c = round_to(np.asarray(init_centroids, np.float32).reshape(B, n_clusters, D), dtype)
    if cosine:
        c = normalize_rows(c, dtype)
    ids = None
    it = 0
    for it in range(max_iters):
        ids = assign_dot(xs, c)
        new = centroid_update_cosine(xs, ids, c, dtype, exact_order=exact_order)
        shift = center_shift(new, c, dtype)
        if history is not None:
            history.append((c, ids, new, shift))
        if shift_below_tol(shift, tol, dtype):
            break
        c = new
    return ids, c, it + 1


# --------------------------------------------------------------------------
# synthetic inputs (seeded; numpy PCG64 streams are stable across versions)
# --------------------------------------------------------------------------
def gmm_points(rng: np.random.Generator, B: int, N: int, D: int, n_comp: int,
               mean_std: float, sigma: float = 1.0, dirichlet: bool = False) -> np.ndarray:
    """Isotropic Gaussian mixture points, float32 (B, N, D)."""
    means = rng.standard_normal((B, n_comp, D), dtype=np.float32) * np.float32(mean_std)
    out = np.empty((B, N, D), dtype=np.float32)
    for b in range(B):
        if dirichlet:
            w = rng.dirichlet(np.ones(n_comp))
            comp = rng.choice(n_comp, size=N, p=w)
        else:
            comp = rng.integers(0, n_comp, size=N)
        out[b] = means[b, comp] + rng.standard_normal((N, D), dtype=np.float32) * np.float32(sigma)
    return out


def init_from_points(rng: np.random.Generator, x: np.ndarray, K: int,
                     replace: bool = False) -> np.ndarray:
    """K points of each batch as initial centroids (with or without replacement)."""
    B, N, D = x.shape
    out = np.empty((B, K, D), dtype=np.float32)
    for b in range(B):
        idx = rng.integers(0, N, size=K) if replace else rng.permutation(N)[:K]
        out[b] = x[b, idx]
    return out
