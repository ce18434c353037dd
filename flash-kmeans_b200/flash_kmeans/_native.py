"""ctypes binding of libflashkmeans_b200.so (declared in include/flash_kmeans_b200.h).

Every compute call of this package goes through these functions; there is no
CPU or PyTorch fallback.  If the library is missing or cannot be loaded the
first call raises ``RuntimeError`` with the build command.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_NAME = "libflashkmeans_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", LIB_NAME)

FK_F16, FK_BF16, FK_F32, FK_I32, FK_I64 = 0, 1, 2, 3, 4
FK_F32_XSPLIT = 5   # float32 x split once into tf32 halves (the *_accumulate entry points)
# Widest rows for which the drivers use FK_F32_XSPLIT: measured 11 % faster at
# D = 128 and 256, 4 % at 512, no faster at 2048 (there the stages are fed from
# L2 and the extra TMA load costs what the shared-memory split did)
XSPLIT_MAX_D = 512


def accumulate_x_code(lib, dtype, B: int, N: int, K: int, D: int, free_bytes: int,
                      share: float) -> tuple:
    """(dtype code, workspace bytes) for fk_assign_accumulate: FK_F32_XSPLIT
    for float32 rows of at most XSPLIT_MAX_D elements when its extra workspace
    (x's two tf32 halves) takes at most `share` of `free_bytes`, else the
    plain code of `dtype`."""
    code = dtype_code(dtype)
    ws = lib.fk_assign_accumulate_workspace_size(B, N, K, D, code)
    if code == FK_F32 and D <= XSPLIT_MAX_D:
        split = lib.fk_assign_accumulate_workspace_size(B, N, K, D, FK_F32_XSPLIT)
        if split - ws <= free_bytes * share:
            return FK_F32_XSPLIT, split
    return code, ws
FK_ACC_PRIVATISED, FK_ACC_FUSED, FK_ACC_SORTED = 0, 1, 2  # fk_assign_accumulate_method
FK_OK = 0
FK_DEV_BAD_LABEL = 101
FK_DEV_WAIT_TIMEOUT = 102

_DTYPE_CODE = {
    torch.float16: FK_F16,
    torch.bfloat16: FK_BF16,
    torch.float32: FK_F32,
    torch.int32: FK_I32,
    torch.int64: FK_I64,
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_S = ctypes.c_size_t
_PL = ctypes.POINTER(ctypes.c_int64)

# name -> (restype, argtypes); mirrors include/flash_kmeans_b200.h
SIGNATURES = {
    "fk_abi_version": (_I, []),
    "fk_status_string": (ctypes.c_char_p, [_I]),
    "fk_last_error": (ctypes.c_char_p, []),
    "fk_device_sm_count": (_I, []),
    "fk_tma_compatible": (_I, [_P, _I, _L, _PL]),
    "fk_row_sqnorm": (_I, [_P, _I, _L, _L, _L, _PL, _P, _I, _PL, _P]),
    "fk_row_normalize": (_I, [_P, _I, _L, _L, _L, _PL, _P, _PL, _P]),
    "fk_pack_rows": (_I, [_P, _I, _L, _L, _L, _PL, _P, _L, _P]),
    "fk_assign_workspace_size": (_S, [_L, _L, _L, _I]),
    "fk_assign": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _PL, _PL, _PL, _PL,
                       _PL, _P, _S, _P, _P]),
    "fk_assign_dot": (_I, [_P, _P, _P, _P, _I, _L, _L, _L, _L, _PL, _PL, _PL, _P, _S, _P, _P]),
    "fk_assign_dot_accumulate": (_I, [_P, _P, _P, _P, _P, _I, _L, _L, _L, _L, _PL, _PL, _PL, _P,
                                      _S, _P, _P]),
    "fk_assign_accumulate_workspace_size": (_S, [_L, _L, _L, _L, _I]),
    "fk_assign_accumulate_method": (_I, [_L, _L, _I]),
    "fk_assign_accumulate": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _PL, _PL,
                                  _PL, _PL, _PL, _P, _S, _P, _P]),
    "fk_assign_accumulate_split_x": (_I, [_P, _L, _L, _L, _L, _PL, _P, _S, _P]),
    "fk_assign_static_scratch": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _L, _L, _L, _L, _PL,
                                      _PL, _PL, _PL, _PL, _P, _P]),
    "fk_centroid_accumulate_workspace_size": (_S, [_L, _L, _L]),
    "fk_centroid_accumulate": (_I, [_P, _I, _L, _L, _L, _L, _PL, _P, _I, _PL, _P, _P, _P, _P,
                                    _S, _P, _P]),
    "fk_centroid_finalize": (_I, [_P, _P, _P, _P, _I, _L, _L, _L, _PL, _PL, _P, _P, _I, _P]),
    "fk_centroid_finalize_normalized": (_I, [_P, _P, _P, _P, _I, _L, _L, _L, _PL, _PL, _P, _I,
                                             _P]),
}

ABI_VERSION = 2

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load (once) and return the native library; raise if it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"flash_kmeans native library not found at {LIB_PATH}; build it with "
                "`make -C flash-kmeans_b200` (or `python __graft_entry__.py`). "
                "This package has no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.fk_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_NAME}: ABI version {lib.fk_abi_version()} != {ABI_VERSION}")
        _lib = lib
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def strides(t: torch.Tensor, n: int):
    st = tuple(t.stride())
    assert len(st) == n
    return (ctypes.c_int64 * n)(*st)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_handle(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check(status: int, what: str) -> None:
    if status != FK_OK:
        lib = load()
        msg = lib.fk_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed: {lib.fk_status_string(status).decode()} ({msg})")


def device_status_message(code: int) -> str:
    return load().fk_status_string(int(code)).decode()
