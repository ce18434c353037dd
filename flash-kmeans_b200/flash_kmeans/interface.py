"""sklearn/faiss-style facade, drop-in for flash_kmeans.interface.FlashKMeans.

Routing follows the reference (interface.py:106-262): host-resident data with
more than ``chunk_size_data_cpu`` points goes through the out-of-core
``kmeans_largeN`` path; everything else is moved to ``device`` in the compute
dtype and clustered by ``batch_kmeans_Euclid``.  Batched (B, N, D) host data
takes the out-of-core path too (the reference asserts it unsupported,
interface.py:138 and :225; ``kmeans_largeN`` here takes batched input).  This build has no
PyTorch/CPU fallback: ``use_triton=False`` or a machine without CUDA raises a
RuntimeError at ``train``/``predict`` time instead of silently switching paths.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _ops
from .assign_euclid_triton import euclid_assign
from .kmeans_large import kmeans_largeN, kmeans_largeN_assign
from .kmeans_triton_impl import batch_kmeans_Euclid


def _require_cuda(use_kernels: bool) -> None:
    if not use_kernels:
        raise RuntimeError(
            "FlashKMeans(use_triton=False) asks for the PyTorch fallback, which this B200 build "
            "does not ship; use use_triton=True")
    if not torch.cuda.is_available():
        raise RuntimeError("FlashKMeans needs a CUDA device (this build has no CPU fallback)")


class FlashKMeans:
    """Batched k-means on B200.

    Parameters mirror the reference (interface.py:63-104): d, k, niter=25,
    tol=1e-8, use_triton=True, seed=0, chunk_size_data=32768,
    chunk_size_centroids=1024 (accepted; only the reference's torch fallback
    used them), chunk_size_data_cpu=1048576, verbose=False, dtype=None,
    device=None.
    """

    def __init__(
        self,
        d: int,
        k: int,
        niter: int = 25,
        tol: float = 1e-8,
        use_triton: bool = True,
        seed: int = 0,
        chunk_size_data: int = 32768,
        chunk_size_centroids: int = 1024,
        chunk_size_data_cpu: int = 1048576,
        verbose: bool = False,
        dtype: Optional[torch.dtype] = None,
        device: Optional[torch.device] = None,
    ):
        self.d = int(d)
        self.k = int(k)
        self.niter = int(niter)
        self.tol = float(tol)
        self.use_triton = bool(use_triton)
        self.seed = int(seed)
        self.chunk_size_data = int(chunk_size_data)
        self.chunk_size_centroids = int(chunk_size_centroids)
        self.chunk_size_data_cpu = int(chunk_size_data_cpu)
        self.verbose = bool(verbose)
        self.dtype = dtype
        self._raw_device = device
        if device is None:
            self.device = torch.device("cuda:0" if torch.cuda.is_available() else "cpu")
        else:
            self.device = device
        self.centroids_b = None
        self.cluster_ids_b = None
        self._batch_size = None

    @staticmethod
    def _as_batched(data: torch.Tensor):
        if data.ndim == 2:
            N, D = data.shape
            return None, N, D, data.unsqueeze(0)
        if data.ndim == 3:
            B, N, D = data.shape
            return B, N, D, data
        raise ValueError(
            "data must be of shape (n_samples, n_features) or (batch_size, n_samples, n_features)")

    def train(self, data: torch.Tensor):
        """Fit on (N, D) or (B, N, D) data; stores centroids_b / cluster_ids_b."""
        B, N, D, x_b = self._as_batched(data)
        _require_cuda(self.use_triton)
        torch.manual_seed(self.seed)
        torch.cuda.manual_seed_all(self.seed)

        if data.device.type == "cpu" and N > self.chunk_size_data_cpu:
            # 2-D data goes in as (N, D), so the random init draws exactly what
            # the reference's kmeans_largeN draws for the same seed
            cluster_ids_b, centroids_b = kmeans_largeN(
                x_b if B is not None else data,
                self.k,
                max_iters=self.niter,
                tol=self.tol,
                verbose=self.verbose,
                dtype=self.dtype,
                BLOCK_N=self.chunk_size_data_cpu,
                device=self._raw_device,
            )
            if B is None:
                cluster_ids_b, centroids_b = cluster_ids_b.unsqueeze(0), centroids_b.unsqueeze(0)
        else:
            compute_dtype = self.dtype or x_b.dtype
            x_b = x_b.to(device=self.device, dtype=compute_dtype, copy=False)
            cluster_ids_b, centroids_b, _ = batch_kmeans_Euclid(
                x_b,
                self.k,
                max_iters=self.niter,
                tol=self.tol,
                init_centroids=None,
                verbose=self.verbose,
            )
        self.centroids_b = centroids_b
        self.cluster_ids_b = cluster_ids_b
        self._batch_size = B

    def fit(self, data: torch.Tensor):
        """Alias for train; returns self."""
        self.train(data)
        return self

    def predict(self, data: torch.Tensor) -> torch.Tensor:
        """Nearest trained centroid for each point; int32 (N,) or (B, N)."""
        if self.centroids_b is None:
            raise RuntimeError("Model not trained. Call train() or fit() first.")
        B, N, D, x_b = self._as_batched(data)
        if B != self._batch_size:
            raise ValueError(
                f"Model was trained with batch size B={self._batch_size}, "
                f"but predict received B={B}. Provide matching batch size.")
        _require_cuda(self.use_triton)
        if data.device.type == "cpu" and N > self.chunk_size_data_cpu:
            labels_b = kmeans_largeN_assign(
                x_b,
                self.centroids_b,
                dtype=self.dtype,
                BLOCK_N=self.chunk_size_data_cpu,
                device=self._raw_device,
            )
            return labels_b.squeeze(0) if B is None else labels_b
        compute_dtype = self.dtype or x_b.dtype
        x_b = x_b.to(device=self.device, dtype=compute_dtype, copy=False)
        cent = self.centroids_b.to(device=x_b.device, dtype=compute_dtype)
        x_k = _ops.ensure_tma(x_b)
        x_sq = _ops.row_sqnorm(x_k)
        labels_b = euclid_assign(x_k, cent, x_sq)
        if B is None:
            return labels_b.squeeze(0)
        return labels_b

    def fit_predict(self, data: torch.Tensor) -> torch.Tensor:
        """train() then return the training labels ((N,) or (B, N), int32)."""
        self.train(data)
        return self.cluster_ids_b.squeeze(0) if self._batch_size is None else self.cluster_ids_b
