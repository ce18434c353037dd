"""Tensor-level wrappers over the C ABI.

PyTorch supplies device memory (the caching allocator, so per-call scratch is
cheap and stream-ordered) and the current stream; every computation is one of
the library's sm_100a kernels.
"""
from __future__ import annotations

import torch

from . import _native as nat

_FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("flash_kmeans kernels need CUDA tensors (no CPU fallback)")


def row_align(dtype: torch.dtype) -> int:
    """Elements per 16 bytes: the row-stride granularity TMA needs."""
    return 16 // torch.empty((), dtype=dtype).element_size()


def tma_compatible(t: torch.Tensor) -> bool:
    """True if a (B, M, D) tensor can be read by the assignment kernel as is."""
    if t.dtype not in _FLOAT_DTYPES or t.dim() != 3:
        return False
    B, M, D = t.shape
    st = list(t.stride())
    if D == 1:
        st[2] = 1
    if M == 1:
        st[1] = -(-D // row_align(t.dtype)) * row_align(t.dtype)
    if B == 1:
        st[0] = M * st[1]
    return bool(nat.load().fk_tma_compatible(nat.ptr(t), nat.dtype_code(t.dtype), D,
                                             (nat.ctypes.c_int64 * 3)(*st)))


def empty_rows(B: int, M: int, D: int, dtype, device) -> torch.Tensor:
    """(B, M, D) view over a buffer whose rows are padded to 16 bytes."""
    al = row_align(dtype)
    Dp = -(-D // al) * al
    buf = torch.empty((B, M, Dp), dtype=dtype, device=device)
    return buf if Dp == D else buf[..., :D]


def pack_rows(x: torch.Tensor) -> torch.Tensor:
    """Copy x (B, M, D) into 16-byte padded rows (kernel fk_pack_rows)."""
    _require_cuda(x)
    B, M, D = x.shape
    out = empty_rows(B, M, D, x.dtype, x.device)
    Dp = out.stride(1)
    lib = nat.load()
    with torch.cuda.device(x.device):
        nat.check(lib.fk_pack_rows(nat.ptr(x), nat.dtype_code(x.dtype), B, M, D,
                                   nat.strides(x, 3), nat.ptr(out), Dp,
                                   nat.stream_handle(x.device)), "fk_pack_rows")
    return out


def ensure_tma(x: torch.Tensor) -> torch.Tensor:
    return x if tma_compatible(x) else pack_rows(x)


def row_sqnorm(x: torch.Tensor, out_dtype=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """(x ** 2).sum(-1) over (B, N, D) with the reference's rounding (kernel fk_row_sqnorm)."""
    _require_cuda(x)
    B, N, D = x.shape
    out_dtype = out_dtype or x.dtype
    if out is None:
        out = torch.empty((B, N), dtype=out_dtype, device=x.device)
    lib = nat.load()
    with torch.cuda.device(x.device):
        nat.check(lib.fk_row_sqnorm(nat.ptr(x), nat.dtype_code(x.dtype), B, N, D,
                                    nat.strides(x, 3), nat.ptr(out), nat.dtype_code(out.dtype),
                                    nat.strides(out, 2), nat.stream_handle(x.device)),
                  "fk_row_sqnorm")
    return out


def row_normalize(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """F.normalize(x, p=2, dim=-1) over (B, N, D) in x's dtype (kernel fk_row_normalize)."""
    _require_cuda(x)
    B, N, D = x.shape
    if out is None:
        out = empty_rows(B, N, D, x.dtype, x.device)
    lib = nat.load()
    with torch.cuda.device(x.device):
        nat.check(lib.fk_row_normalize(nat.ptr(x), nat.dtype_code(x.dtype), B, N, D,
                                       nat.strides(x, 3), nat.ptr(out), nat.strides(out, 3),
                                       nat.stream_handle(x.device)), "fk_row_normalize")
    return out


class DeviceStatus:
    """Per-device int32 word that kernels set on asynchronous errors."""

    _words: dict = {}

    @classmethod
    def word(cls, device) -> torch.Tensor:
        dev = torch.device(device)
        key = dev.index if dev.index is not None else torch.cuda.current_device()
        w = cls._words.get(key)
        if w is None:
            w = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", key))
            cls._words[key] = w
        return w

    @classmethod
    def raise_if_set(cls, device) -> None:
        w = cls.word(device)
        code = int(w[0].item())
        if code:
            w.zero_()
            raise RuntimeError(f"flash_kmeans device error {code}: {nat.device_status_message(code)}")


def assign(x, centroids, x_sq, out=None, c_sq=None, counts=None, status=None) -> torch.Tensor:
    """Launch fk_assign.  x / centroids must already be TMA-compatible."""
    B, N, D = x.shape
    K = centroids.shape[1]
    if out is None:
        out = torch.empty((B, N), dtype=torch.int32, device=x.device)
    lib = nat.load()
    ws_bytes = lib.fk_assign_workspace_size(B, K, D, nat.dtype_code(x.dtype))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if status is None:
        status = DeviceStatus.word(x.device)
    with torch.cuda.device(x.device):
        _assign_call(lib, x, centroids, x_sq, out, c_sq, counts, ws, ws_bytes, status)
    return out


def _assign_call(lib, x, centroids, x_sq, out, c_sq, counts, ws, ws_bytes, status):
    B, N, D = x.shape
    K = centroids.shape[1]
    nat.check(lib.fk_assign(
        nat.ptr(x), nat.ptr(centroids), nat.ptr(x_sq), nat.ptr(c_sq), nat.ptr(out), nat.ptr(counts),
        nat.dtype_code(x.dtype), nat.dtype_code(x_sq.dtype),
        nat.dtype_code(c_sq.dtype) if c_sq is not None else 0,
        B, N, K, D, nat.strides(x, 3), nat.strides(centroids, 3), nat.strides(x_sq, 2),
        nat.strides(c_sq, 2) if c_sq is not None else None, nat.strides(out, 2),
        nat.ptr(ws), ws_bytes, nat.ptr(status), nat.stream_handle(x.device)), "fk_assign")


def assign_accumulate(x, centroids, x_sq, out, counts, sums, c_sq=None, status=None) -> None:
    """Launch fk_assign_accumulate: labels into `out`, their histogram added to
    `counts` and the rows of x added to sums[label] (one Lloyd iteration's
    assignment and accumulation)."""
    B, N, D = x.shape
    K = centroids.shape[1]
    lib = nat.load()
    ws_bytes = lib.fk_assign_accumulate_workspace_size(B, N, K, D, nat.dtype_code(x.dtype))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if status is None:
        status = DeviceStatus.word(x.device)
    with torch.cuda.device(x.device):
        nat.check(lib.fk_assign_accumulate(
            nat.ptr(x), nat.ptr(centroids), nat.ptr(x_sq), nat.ptr(c_sq), nat.ptr(out),
            nat.ptr(counts), nat.ptr(sums), nat.dtype_code(x.dtype), nat.dtype_code(x_sq.dtype),
            nat.dtype_code(c_sq.dtype) if c_sq is not None else 0, B, N, K, D,
            nat.strides(x, 3), nat.strides(centroids, 3), nat.strides(x_sq, 2),
            nat.strides(c_sq, 2) if c_sq is not None else None, nat.strides(out, 2),
            nat.ptr(ws), ws_bytes, nat.ptr(status), nat.stream_handle(x.device)),
            "fk_assign_accumulate")


def accumulate(x, ids, sums, counts, hist=None, status=None) -> None:
    """Launch fk_centroid_accumulate: sums += per-cluster row sums, counts += sizes."""
    B, N, D = x.shape
    K = sums.shape[1]
    lib = nat.load()
    ws_bytes = lib.fk_centroid_accumulate_workspace_size(B, N, K)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if status is None:
        status = DeviceStatus.word(x.device)
    with torch.cuda.device(x.device):
        nat.check(lib.fk_centroid_accumulate(
            nat.ptr(x), nat.dtype_code(x.dtype), B, N, K, D, nat.strides(x, 3), nat.ptr(ids),
            nat.dtype_code(ids.dtype), nat.strides(ids, 2), nat.ptr(hist), nat.ptr(sums),
            nat.ptr(counts), nat.ptr(ws), ws_bytes, nat.ptr(status), nat.stream_handle(x.device)),
            "fk_centroid_accumulate")


def finalize(sums, counts, old, new, csq_out=None, shift_out=None, reset=False) -> None:
    """Launch fk_centroid_finalize: new = counts ? sums / counts : old (cast)."""
    B, K, D = old.shape
    lib = nat.load()
    with torch.cuda.device(old.device):
        nat.check(lib.fk_centroid_finalize(
            nat.ptr(sums), nat.ptr(counts), nat.ptr(old), nat.ptr(new), nat.dtype_code(old.dtype),
            B, K, D, nat.strides(old, 3), nat.strides(new, 3), nat.ptr(csq_out),
            nat.ptr(shift_out), 1 if reset else 0, nat.stream_handle(old.device)),
            "fk_centroid_finalize")


def assign_dot(x, centroids, out=None, counts=None, status=None) -> torch.Tensor:
    """Launch fk_assign_dot (argmax of x.c).  x / centroids must be TMA-compatible."""
    B, N, D = x.shape
    K = centroids.shape[1]
    if out is None:
        out = torch.empty((B, N), dtype=torch.int32, device=x.device)
    lib = nat.load()
    ws_bytes = lib.fk_assign_workspace_size(B, K, D, nat.dtype_code(x.dtype))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    if status is None:
        status = DeviceStatus.word(x.device)
    with torch.cuda.device(x.device):
        nat.check(lib.fk_assign_dot(
            nat.ptr(x), nat.ptr(centroids), nat.ptr(out), nat.ptr(counts), nat.dtype_code(x.dtype),
            B, N, K, D, nat.strides(x, 3), nat.strides(centroids, 3), nat.strides(out, 2),
            nat.ptr(ws), ws_bytes, nat.ptr(status), nat.stream_handle(x.device)), "fk_assign_dot")
    return out


def finalize_normalized(sums, counts, old, new, shift_out=None, reset=False) -> None:
    """Launch fk_centroid_finalize_normalized: new = normalize(counts ? sums / counts : old)."""
    B, K, D = old.shape
    lib = nat.load()
    with torch.cuda.device(old.device):
        nat.check(lib.fk_centroid_finalize_normalized(
            nat.ptr(sums), nat.ptr(counts), nat.ptr(old), nat.ptr(new), nat.dtype_code(old.dtype),
            B, K, D, nat.strides(old, 3), nat.strides(new, 3), nat.ptr(shift_out),
            1 if reset else 0, nat.stream_handle(old.device)), "fk_centroid_finalize_normalized")
