"""Seeded input specs for the golden vectors under ``tests/golden/``.

Inputs are regenerated from these specs with numpy's PCG64 generator (stable
across numpy versions), so a fixture stores only outputs plus an input
checksum that detects generator drift.  ``make_golden.py`` (run where the
reference project is importable) turns each spec into a fixture by running
the reference's own ``torch_fallback`` functions.
"""
from __future__ import annotations

import os
import sys

import numpy as np

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if _ROOT not in sys.path:
    sys.path.insert(0, _ROOT)

from oracle import kmeans_oracle as ko  # noqa: E402

GOLDEN_DIR = os.path.dirname(os.path.abspath(__file__))

# kind, name, dtype, shape/params
ASSIGN_CASES = [
    dict(name="assign_f32_small", dtype="float32", B=2, N=257, K=19, D=32, seed=11),
    dict(name="assign_f16_d100", dtype="float16", B=1, N=1000, K=37, D=100, seed=12),
    dict(name="assign_bf16_small", dtype="bfloat16", B=2, N=300, K=64, D=64, seed=13),
    dict(name="assign_f16_d17", dtype="float16", B=1, N=513, K=33, D=17, seed=14),
    dict(name="assign_f16_dupcent", dtype="float16", B=1, N=200, K=16, D=32, seed=15, dup=True),
    dict(name="assign_f16_xsqf32", dtype="float16", B=1, N=700, K=40, D=64, seed=16, xsq_f32=True),
    dict(name="assign_f16_8193x1031", dtype="float16", B=1, N=8193, K=1031, D=128, seed=17),
    dict(name="assign_f32_8193x1031_d96", dtype="float32", B=1, N=8193, K=1031, D=96, seed=18),
    dict(name="assign_f32_d513", dtype="float32", B=1, N=600, K=70, D=513, seed=19),
    # BASELINE config 4's feature size (split-D, 3xTF32): D=2048, float32
    dict(name="assign_f32_d2048", dtype="float32", B=1, N=2048, K=256, D=2048, seed=20),
    # float16 overflow: rows whose x_sq is inf, centroids whose c_sq is inf and
    # cross products whose doubling leaves the float16 range, so distances
    # reach inf and NaN (argmin then takes the first NaN, else the first minimum)
    dict(name="assign_f16_overflow", dtype="float16", B=1, N=600, K=64, D=64, seed=25,
         overflow=True),
]

UPDATE_CASES = [
    dict(name="update_f32_small", dtype="float32", B=2, N=500, K=23, D=48, seed=21, holes=5),
    dict(name="update_f16_4096x300", dtype="float16", B=1, N=4096, K=300, D=64, seed=22, holes=7),
    dict(name="update_bf16_small", dtype="bfloat16", B=2, N=777, K=40, D=40, seed=23, holes=3),
    dict(name="update_f16_d17", dtype="float16", B=1, N=513, K=33, D=17, seed=24, holes=2),
]

LLOYD_CASES = [
    dict(name="lloyd_f32_gmm", dtype="float32", B=2, N=2048, K=32, D=64, seed=31,
         gen="gmm", comps=32, mean_std=2.0, iters=5, tol=0.0),
    dict(name="lloyd_f16_randn", dtype="float16", B=2, N=3000, K=50, D=128, seed=32,
         gen="randn", iters=4, tol=0.0),
    dict(name="lloyd_f16_tolbreak", dtype="float16", B=1, N=2000, K=8, D=16, seed=33,
         gen="gmm", comps=8, mean_std=6.0, iters=50, tol=1e-2),
    # BASELINE config 1 at full size: B=2, N=16384, D=128, K=256, fp32, 10 iters, tol=0
    dict(name="lloyd_cfg1_f32", dtype="float32", B=2, N=16384, K=256, D=128, seed=34,
         gen="gmm", comps=256, mean_std=2.0, iters=10, tol=0.0),
]


def assign_inputs(spec):
    rng = np.random.default_rng(spec["seed"])
    B, N, K, D, dt = spec["B"], spec["N"], spec["K"], spec["D"], spec["dtype"]
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    if spec.get("dup"):
        base = ko.round_to(rng.standard_normal((B, K // 2, D), dtype=np.float32), dt)
        c = np.concatenate([base, base], axis=1)
    else:
        c = ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    if spec.get("overflow"):
        # rows N/3.. scaled by 30 (x_sq finite, some cross products overflow
        # when doubled), rows 2N/3.. by 100 (x_sq = inf); a quarter of the
        # centroids scaled by 100 (c_sq = inf), at random positions
        scale = np.ones((B, N, 1), np.float32)
        scale[:, N // 3:2 * N // 3] = 30.0
        scale[:, 2 * N // 3:] = 100.0
        x = ko.round_to(x * scale, dt)
        big = rng.choice(K, size=K // 4, replace=False)
        c[:, big] = ko.round_to(c[:, big] * np.float32(100.0), dt)
    if spec.get("xsq_f32"):
        xsq = np.square(x).sum(-1, dtype=np.float32)
        xsq_dtype = "float32"
    else:
        xsq = ko.row_sqnorm(x, dt)
        xsq_dtype = dt
    return x, c, xsq, xsq_dtype


def update_inputs(spec):
    rng = np.random.default_rng(spec["seed"])
    B, N, K, D, dt = spec["B"], spec["N"], spec["K"], spec["D"], spec["dtype"]
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    old = ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    ids = rng.integers(0, K, size=(B, N)).astype(np.int32)
    holes = rng.choice(K, size=spec["holes"], replace=False)
    nonholes = np.setdiff1d(np.arange(K), holes)
    mask = np.isin(ids, holes)  # guarantee some empty clusters
    ids[mask] = rng.choice(nonholes, size=int(mask.sum())).astype(np.int32)
    return x, ids, old


def lloyd_inputs(spec):
    rng = np.random.default_rng(spec["seed"])
    B, N, K, D, dt = spec["B"], spec["N"], spec["K"], spec["D"], spec["dtype"]
    if spec["gen"] == "gmm":
        x = ko.gmm_points(rng, B, N, D, spec["comps"], spec["mean_std"])
    else:
        x = rng.standard_normal((B, N, D), dtype=np.float32)
    x = ko.round_to(x, dt)
    c0 = ko.init_from_points(rng, x, K, replace=False)
    return x, c0


def checksum(*arrays) -> float:
    """Sum of the finite values plus the number of non-finite ones (inputs of
    the overflow cases hold inf)."""
    total = 0.0
    for a in arrays:
        a = np.asarray(a, dtype=np.float64)
        fin = np.isfinite(a)
        total += float(a[fin].sum()) + float((~fin).sum())
    return total


def path(name: str) -> str:
    return os.path.join(GOLDEN_DIR, name + ".npz")


# cosine / dot-product k-means (the reference's batch_kmeans_Cosine / _Dot path)
NORMALIZE_CASES = [
    dict(name="normalize_f16", dtype="float16", B=2, N=333, D=100, seed=41),
    dict(name="normalize_bf16", dtype="bfloat16", B=1, N=500, D=64, seed=42),
    dict(name="normalize_f32", dtype="float32", B=2, N=257, D=33, seed=43),
]

SIM_ASSIGN_CASES = [
    dict(name="cos_assign_f16", dtype="float16", B=2, N=1000, K=70, D=128, seed=51, cosine=True),
    dict(name="cos_assign_bf16", dtype="bfloat16", B=1, N=1500, K=300, D=64, seed=52, cosine=True),
    dict(name="cos_assign_f32", dtype="float32", B=2, N=700, K=45, D=96, seed=53, cosine=True),
    dict(name="dot_assign_f16_d17", dtype="float16", B=1, N=513, K=33, D=17, seed=54, cosine=False,
         neg=True),
    dict(name="dot_assign_f32_k1031", dtype="float32", B=1, N=2049, K=1031, D=128, seed=55,
         cosine=False),
]

SIM_UPDATE_CASES = [
    dict(name="cos_update_f16", dtype="float16", B=2, N=900, K=40, D=64, seed=61, holes=4),
    dict(name="cos_update_bf16", dtype="bfloat16", B=1, N=1200, K=100, D=128, seed=62, holes=6),
    dict(name="cos_update_f32", dtype="float32", B=2, N=500, K=23, D=48, seed=63, holes=3),
]

SIM_LLOYD_CASES = [
    dict(name="cos_lloyd_f16", dtype="float16", B=2, N=3000, K=40, D=64, seed=71,
         comps=40, mean_std=2.0, iters=4, cosine=True),
    dict(name="cos_lloyd_f32", dtype="float32", B=1, N=2048, K=32, D=128, seed=72,
         comps=32, mean_std=2.0, iters=4, cosine=True),
    dict(name="dot_lloyd_f16", dtype="float16", B=1, N=2000, K=16, D=32, seed=73,
         comps=16, mean_std=2.0, iters=3, cosine=False),
]


def normalize_inputs(spec):
    """Gaussian rows in the dtype, row 5 of batch 0 all zeros (the eps clamp)."""
    rng = np.random.default_rng(spec["seed"])
    x = ko.round_to(rng.standard_normal((spec["B"], spec["N"], spec["D"]), dtype=np.float32)
                    * 3.0, spec["dtype"])
    x[0, 5] = 0.0
    return x


def sim_assign_inputs(spec):
    """Points and centroids in the dtype (normalised by F.normalize afterwards
    when ``cosine``).  ``neg``: non-negative points and non-positive
    centroids, so every score, the winning one included, is negative."""
    rng = np.random.default_rng(spec["seed"])
    B, N, K, D, dt = spec["B"], spec["N"], spec["K"], spec["D"], spec["dtype"]
    x = rng.standard_normal((B, N, D), dtype=np.float32)
    c = rng.standard_normal((B, K, D), dtype=np.float32)
    if spec.get("neg"):
        x, c = np.abs(x), -np.abs(c)
    return ko.round_to(x, dt), ko.round_to(c, dt)


def sim_update_inputs(spec):
    return update_inputs(spec)


def sim_lloyd_inputs(spec):
    rng = np.random.default_rng(spec["seed"])
    B, N, K, D, dt = spec["B"], spec["N"], spec["K"], spec["D"], spec["dtype"]
    x = ko.round_to(ko.gmm_points(rng, B, N, D, spec["comps"], spec["mean_std"]), dt)
    c0 = ko.init_from_points(rng, x, K, replace=False)
    return x, c0
