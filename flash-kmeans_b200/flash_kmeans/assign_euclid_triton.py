"""Nearest-centroid assignment, drop-in for flash_kmeans.assign_euclid_triton.

The module keeps the reference's name so ``from flash_kmeans.assign_euclid_triton
import euclid_assign_triton`` keeps working; the kernel behind it is the
sm_100a tcgen05 assignment of libflashkmeans_b200.so, not Triton.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _ops


def euclid_assign(x: torch.Tensor, centroids: torch.Tensor, x_sq: torch.Tensor,
                  out: Optional[torch.Tensor] = None, c_sq: Optional[torch.Tensor] = None
                  ) -> torch.Tensor:
    """Nearest centroid (squared Euclidean) for every point; int32 (B, N).

    x (B, N, D) and centroids (B, K, D) in float16 / bfloat16 / float32;
    x_sq (B, N) = ||x||^2 (any float dtype; when it has x's 16-bit dtype the
    distance is evaluated with that dtype's rounding, as the reference torch
    path does); c_sq (B, K) optional.  Ties go to the lowest index.
    Arbitrary strides are accepted; rows that are not 16-byte addressable are
    repacked first.
    """
    assert x.is_cuda and centroids.is_cuda and x_sq.is_cuda, "All tensors must be on CUDA"
    assert centroids.dtype == x.dtype, "centroids dtype mismatch"
    B, N, D = x.shape
    K = centroids.shape[1]
    assert centroids.shape == (B, K, D), "centroids shape mismatch"
    assert x_sq.shape == (B, N), "x_sq shape mismatch"
    if out is None:
        out = torch.empty((B, N), device=x.device, dtype=torch.int32)
    if c_sq is not None:
        assert c_sq.shape == (B, K), "c_sq shape mismatch"
    return _ops.assign(_ops.ensure_tma(x), _ops.ensure_tma(centroids), x_sq, out=out, c_sq=c_sq)


def euclid_assign_triton(
    x: torch.Tensor,
    centroids: torch.Tensor,
    x_sq: torch.Tensor,
    out: torch.Tensor = None,
    c_sq: torch.Tensor = None,
    *,
    BLOCK_N: int = 128,
    BLOCK_K: int = 128,
    num_warps: Optional[int] = None,
    num_stages: Optional[int] = None,
    config: Optional[dict] = None,
    use_heuristic: bool = True,
) -> torch.Tensor:
    """Signature of the reference wrapper (assign_euclid_triton.py:1238-1251).

    The tuning keywords are accepted for compatibility and ignored: the
    B200 kernel has one fixed tiling.  As in the reference, ``num_warps`` and
    ``num_stages`` must be given together.
    """
    if (num_warps is None) != (num_stages is None) and config is None:
        raise ValueError("num_warps and num_stages must be set together")
    return euclid_assign(x, centroids, x_sq, out=out, c_sq=c_sq)


def cosine_assign_triton(x: torch.Tensor, centroids: torch.Tensor, out: torch.Tensor = None,
                         *, BLOCK_N: int = 128, BLOCK_K: int = 128) -> torch.Tensor:
    """Centroid of the largest dot product for every point; int32 (B, N).

    Signature and contract of the reference wrapper (assign_euclid_triton.py:
    1415-1498): x (B, N, D) and centroids (B, K, D) of one float dtype; with
    normalised inputs this is the cosine assignment of batch_kmeans_Cosine,
    otherwise the dot-product assignment of batch_kmeans_Dot.  Scores are
    float32 dot products (3xTF32 for float32 inputs), ties go to the lowest
    index.  The block sizes are accepted and ignored (one fixed tiling).
    """
    assert x.is_cuda and centroids.is_cuda, "All tensors must be on CUDA"
    assert centroids.dtype == x.dtype, "centroids dtype mismatch"
    B, N, D = x.shape
    K = centroids.shape[1]
    assert centroids.shape == (B, K, D), "centroids shape mismatch"
    if out is None:
        out = torch.empty((B, N), device=x.device, dtype=torch.int32)
    return _ops.assign_dot(_ops.ensure_tma(x), _ops.ensure_tma(centroids), out=out)
