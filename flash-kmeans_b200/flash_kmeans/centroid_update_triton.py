"""Centroid update, drop-in for flash_kmeans.centroid_update_triton.

Backed by the counting-sort segmented-sum kernels of libflashkmeans_b200.so.
"""
from __future__ import annotations

import torch

from . import _ops


def centroid_update_euclid(x: torch.Tensor, cluster_ids: torch.Tensor, old_centroids: torch.Tensor,
                           *, centroid_sums: torch.Tensor = None,
                           centroid_cnts: torch.Tensor = None, calculate_new: bool = True):
    """Per-cluster means of x grouped by cluster_ids; empty clusters keep old.

    x (B, N, D); cluster_ids (B, N) int32 or int64 in [0, K); old_centroids
    (B, K, D).  With ``centroid_sums`` (float32 (B, K, D)) / ``centroid_cnts``
    (int32 (B, K)) the sums and counts are ADDED to those buffers, which lets a
    caller accumulate over several blocks; ``calculate_new=False`` returns None
    after accumulating.  Sums are float32; the result has x's dtype.
    """
    assert x.is_cuda and cluster_ids.is_cuda, "Inputs must be on CUDA device"
    B, N, D = x.shape
    K = old_centroids.shape[1]
    if centroid_sums is None:
        centroid_sums = torch.zeros((B, K, D), device=x.device, dtype=torch.float32)
    else:
        assert centroid_sums.shape == (B, K, D)
    if centroid_cnts is None:
        centroid_cnts = torch.zeros((B, K), device=x.device, dtype=torch.int32)
    else:
        assert centroid_cnts.shape == (B, K)
    if cluster_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("cluster_ids must be int32 or int64")
    sums = centroid_sums if (centroid_sums.is_contiguous()
                             and centroid_sums.dtype == torch.float32) else None
    cnts = centroid_cnts if (centroid_cnts.is_contiguous()
                             and centroid_cnts.dtype == torch.int32) else None
    s_buf = sums if sums is not None else torch.zeros((B, K, D), device=x.device,
                                                      dtype=torch.float32)
    c_buf = cnts if cnts is not None else torch.zeros((B, K), device=x.device, dtype=torch.int32)
    _ops.accumulate(x, cluster_ids, s_buf, c_buf)
    if sums is None:
        centroid_sums.add_(s_buf)
    if cnts is None:
        centroid_cnts.add_(c_buf)
    if not calculate_new:
        return None
    new = torch.empty((B, K, D), device=x.device, dtype=x.dtype)
    _ops.finalize(s_buf if sums is None else centroid_sums,
                  c_buf if cnts is None else centroid_cnts, old_centroids.to(x.dtype), new)
    return new


def triton_centroid_update_sorted_euclid(x: torch.Tensor, cluster_ids: torch.Tensor,
                                         old_centroids: torch.Tensor, *, BLOCK_N: int = 256,
                                         centroid_sums: torch.Tensor = None,
                                         centroid_cnts: torch.Tensor = None,
                                         calculate_new: bool = True):
    """Signature of the reference (centroid_update_triton.py:316-317); BLOCK_N is ignored."""
    return centroid_update_euclid(x, cluster_ids, old_centroids, centroid_sums=centroid_sums,
                                  centroid_cnts=centroid_cnts, calculate_new=calculate_new)


def triton_centroid_update_euclid(x: torch.Tensor, cluster_ids: torch.Tensor,
                                  old_centroids: torch.Tensor):
    """The reference's per-token atomic variant (centroid_update_triton.py:119-160):
    same result, served by the same kernels."""
    assert x.is_cuda and cluster_ids.is_cuda, "Input tensors must be on CUDA device"
    B, N, D = x.shape
    assert cluster_ids.shape == (B, N)
    return centroid_update_euclid(x, cluster_ids, old_centroids)


def centroid_update_cosine(x_norm: torch.Tensor, cluster_ids: torch.Tensor,
                           old_centroids: torch.Tensor) -> torch.Tensor:
    """Per-cluster means, L2-normalised (the update of cosine / dot-product k-means).

    Follows _centroid_update_torch_native with mode='cosine' (torch_fallback.py:
    72-109): float32 sums and counts, mean (the old centroid, as float32, for an
    empty cluster), F.normalize in float32, then cast to x's dtype.
    """
    assert x_norm.is_cuda and cluster_ids.is_cuda, "Inputs must be on CUDA device"
    B, N, D = x_norm.shape
    K = old_centroids.shape[1]
    assert cluster_ids.shape == (B, N)
    if cluster_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("cluster_ids must be int32 or int64")
    sums = torch.zeros((B, K, D), device=x_norm.device, dtype=torch.float32)
    cnts = torch.zeros((B, K), device=x_norm.device, dtype=torch.int32)
    _ops.accumulate(x_norm, cluster_ids, sums, cnts)
    new = torch.empty((B, K, D), device=x_norm.device, dtype=x_norm.dtype)
    _ops.finalize_normalized(sums, cnts, old_centroids.to(x_norm.dtype), new)
    return new


def triton_centroid_update_cosine(x_norm: torch.Tensor, cluster_ids: torch.Tensor,
                                  old_centroids: torch.Tensor) -> torch.Tensor:
    """The reference's per-token variant (centroid_update_triton.py:73-119)."""
    return centroid_update_cosine(x_norm, cluster_ids, old_centroids)


def triton_centroid_update_sorted_cosine(x_norm: torch.Tensor, cluster_ids: torch.Tensor,
                                         old_centroids: torch.Tensor, *,
                                         BLOCK_N: int = 256) -> torch.Tensor:
    """Signature of the reference (centroid_update_triton.py:268-313); BLOCK_N is ignored."""
    return centroid_update_cosine(x_norm, cluster_ids, old_centroids)
