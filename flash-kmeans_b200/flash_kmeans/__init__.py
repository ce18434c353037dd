"""Flash-KMeans for NVIDIA B200 (sm_100a).

Drop-in replacement for the Euclidean Lloyd path of the reference package
(``flash_kmeans/__init__.py:37-46`` exports the same names).  Compute runs in
hand-written tcgen05/TMA kernels of ``_lib/libflashkmeans_b200.so`` reached
through a C ABI (``include/flash_kmeans_b200.h``).  Unlike the reference there
is no import-time fallback to a PyTorch implementation: calls without the
native library or without CUDA raise RuntimeError.
"""
from .interface import FlashKMeans
from .kmeans_triton_impl import batch_kmeans_Euclid, batch_kmeans_Cosine, batch_kmeans_Dot
from .centroid_update_triton import (
    triton_centroid_update_euclid,
    triton_centroid_update_sorted_euclid,
)
from .kmeans_large import kmeans_largeN, kmeans_largeN_assign

__all__ = [
    "batch_kmeans_Euclid",
    "batch_kmeans_Cosine",
    "batch_kmeans_Dot",
    "triton_centroid_update_euclid",
    "triton_centroid_update_sorted_euclid",
    "FlashKMeans",
    "kmeans_largeN",
    "kmeans_largeN_assign",
]

__version__ = "0.3.0+b200"
