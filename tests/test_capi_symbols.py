"""The C-ABI library loads without a GPU and exports every declared symbol.

No compute call is made here (this runs on CPU-only machines); only pure host
entry points (version, status strings, the TMA layout predicate, workspace
sizes) are exercised.
"""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flash_kmeans_b200.h")


def _declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fk_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from flash_kmeans import _native
    return _native.load()


def test_header_declares_the_api():
    names = _declared()
    for must in ("fk_assign", "fk_centroid_accumulate", "fk_centroid_finalize", "fk_row_sqnorm",
                 "fk_pack_rows", "fk_abi_version"):
        assert must in names


def test_every_declared_symbol_is_exported(lib):
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    from flash_kmeans import _native
    assert set(_native.SIGNATURES) == set(_declared())


def test_host_only_entry_points(lib):
    assert lib.fk_abi_version() == 2
    assert lib.fk_status_string(0) == b"ok"
    assert b"workspace" in lib.fk_status_string(3)
    # padded c_sq, then the -2c operand for 16-bit x (none for float32)
    assert lib.fk_assign_workspace_size(32, 1000, 128, 0) >= 32 * 1024 * 4 + 32 * 1000 * 128 * 2
    assert lib.fk_assign_workspace_size(32, 1000, 100, 1) >= 32 * 1024 * 4 + 32 * 1000 * 104 * 2
    # float32: the centroids' tf32 hi and lo halves (B, K, D padded to 8) besides c_sq
    assert lib.fk_assign_workspace_size(32, 1000, 128, 2) >= 32 * 1024 * 4 + 2 * 32 * 1000 * 128 * 4
    assert lib.fk_assign_workspace_size(32, 1000, 128, 2) < 32 * 1024 * 4 + 2 * 32 * 1000 * 128 * 4 + 2048
    assert lib.fk_centroid_accumulate_workspace_size(32, 75600, 1000) >= 2 * 32 * 75600 * 4
    st = (ctypes.c_int64 * 3)(75600 * 128, 128, 1)
    assert lib.fk_tma_compatible(ctypes.c_void_p(1 << 20), 0, 128, st) == 1
    st_bad = (ctypes.c_int64 * 3)(75600 * 100, 100, 1)  # 200-byte rows
    assert lib.fk_tma_compatible(ctypes.c_void_p(1 << 20), 0, 100, st_bad) == 0
    assert lib.fk_tma_compatible(ctypes.c_void_p((1 << 20) + 8), 0, 128, st) == 0


def test_invalid_arguments_fail_on_host(lib):
    """Argument validation happens before any CUDA call."""
    from flash_kmeans import _native
    st = (ctypes.c_int64 * 3)(1, 1, 1)
    rc = lib.fk_assign(None, None, None, None, None, None, 0, 0, 0, 1, 1, 0, 1, st, st, st, st, st,
                       None, 0, None, None)
    assert rc == 1
    with pytest.raises(RuntimeError, match="invalid argument"):
        _native.check(rc, "fk_assign")
    assert b"bad sizes" in lib.fk_last_error()
    rc = lib.fk_centroid_accumulate(None, 0, 1, 1, 4, 8, st, None, 3, st, None, None, None, None,
                                    0, None, None)
    assert rc == 1


def test_similarity_entry_points_validate_on_host(lib):
    """The cosine / dot-product entry points reject bad calls before any CUDA call."""
    st3 = (ctypes.c_int64 * 3)(1, 1, 1)
    st2 = (ctypes.c_int64 * 2)(1, 1)
    # K = 0, then null pointers with valid sizes
    assert lib.fk_assign_dot(None, None, None, None, 0, 1, 4, 0, 8, st3, st3, st2, None, 0, None,
                             None) == 1
    assert b"bad sizes" in lib.fk_last_error()
    assert lib.fk_assign_dot(None, None, None, None, 0, 1, 4, 2, 8, st3, st3, st2, None, 0, None,
                             None) == 1
    assert b"null pointer" in lib.fk_last_error()
    # the fused variant needs counts and sums
    assert lib.fk_assign_dot_accumulate(None, None, None, None, None, 0, 1, 4, 2, 8, st3, st3, st2,
                                        None, 0, None, None) == 1
    assert b"counts and sums" in lib.fk_last_error()
    assert lib.fk_row_normalize(None, 0, 1, 4, 0, st3, None, st3, None) == 1
    assert lib.fk_row_normalize(None, 0, 1, 4, 8, st3, None, st3, None) == 1
    assert b"null pointer" in lib.fk_last_error()
    assert lib.fk_row_normalize(ctypes.c_void_p(16), 0, 1, 1 << 31, 8, st3, ctypes.c_void_p(16),
                                st3, None) == 2   # unsupported: N >= 2^31
    # finalize: K = 0, null pointers, and new aliasing old
    assert lib.fk_centroid_finalize_normalized(None, None, None, None, 0, 1, 0, 8, st3, st3, None, 0,
                                               None) == 1
    assert lib.fk_centroid_finalize_normalized(None, None, None, None, 0, 1, 2, 8, st3, st3, None, 0,
                                               None) == 1
    p = ctypes.c_void_p(256)
    assert lib.fk_centroid_finalize_normalized(p, p, p, p, 0, 1, 2, 8, st3, st3, None, 0, None) == 1
    assert b"aliases" in lib.fk_last_error()


def test_accumulate_method_codes_are_stable(lib):
    from flash_kmeans import _native
    assert (_native.FK_ACC_PRIVATISED, _native.FK_ACC_FUSED, _native.FK_ACC_SORTED) == (0, 1, 2)
    # K <= 128 with 16-bit x and D <= 128: one kernel, one-hot sums on the tensor core
    assert lib.fk_assign_accumulate_method(128, 128, 0) == _native.FK_ACC_FUSED
    assert lib.fk_assign_accumulate_method(200, 128, 0) == _native.FK_ACC_PRIVATISED
    assert lib.fk_assign_accumulate_method(128, 128, 2) == _native.FK_ACC_PRIVATISED
    assert lib.fk_assign_accumulate_method(1000, 128, 0) == _native.FK_ACC_FUSED
    assert lib.fk_assign_accumulate_method(1024, 2048, 2) == _native.FK_ACC_SORTED


def test_xsplit_workspace_and_validation(lib):
    """FK_F32_XSPLIT: FK_F32's accumulate workspace plus x's (2B, N, Dx) float32
    halves (Dx = D rounded up to 4), the same method as FK_F32, and host-side
    argument checks of fk_assign_accumulate_split_x (no launch)."""
    from flash_kmeans import _native
    X = _native.FK_F32_XSPLIT
    for B, N, K, D in [(1, 262144, 1024, 2048), (3, 333, 70, 37), (2, 1000, 300, 128)]:
        base = lib.fk_assign_accumulate_workspace_size(B, N, K, D, 2)
        dx = (D + 3) // 4 * 4
        got = lib.fk_assign_accumulate_workspace_size(B, N, K, D, X)
        assert got >= base + 2 * B * N * dx * 4
        assert got < base + 2 * B * N * dx * 4 + 1024
        assert lib.fk_assign_accumulate_method(K, D, X) == lib.fk_assign_accumulate_method(K, D, 2)
    st3 = (ctypes.c_int64 * 3)(1000 * 128, 128, 1)
    p = ctypes.c_void_p(1 << 20)
    small = lib.fk_assign_accumulate_workspace_size(2, 1000, 300, 128, 2)
    assert lib.fk_assign_accumulate_split_x(None, 2, 1000, 300, 128, st3, p, 1 << 30, None) == 1
    assert lib.fk_assign_accumulate_split_x(p, 2, 1000, 0, 128, st3, p, 1 << 30, None) == 1
    assert lib.fk_assign_accumulate_split_x(p, 2, 1000, 300, 128, st3, p, small, None) == 3
    assert lib.fk_assign_accumulate_split_x(p, 0, 1000, 300, 128, st3, None, 0, None) == 0


def test_split_x_choice(lib):
    """The drivers' choice of the split-x form: float32 rows of at most
    XSPLIT_MAX_D elements, and only when x's halves fit the given share of the
    free device memory; 16-bit x and wider rows keep their plain code."""
    import torch
    from flash_kmeans import _native
    B, N, K, D = 1, 1 << 20, 8192, 128
    extra = 2 * B * N * D * 4
    code, ws = _native.accumulate_x_code(lib, torch.float32, B, N, K, D, 4 * extra, 0.25)
    assert code == _native.FK_F32_XSPLIT
    assert ws == lib.fk_assign_accumulate_workspace_size(B, N, K, D, _native.FK_F32_XSPLIT)
    code, ws = _native.accumulate_x_code(lib, torch.float32, B, N, K, D, 2 * extra, 0.25)
    assert code == _native.FK_F32
    assert ws == lib.fk_assign_accumulate_workspace_size(B, N, K, D, _native.FK_F32)
    code, _ = _native.accumulate_x_code(lib, torch.float32, 1, 262144, 1024, 2048, 1 << 40, 0.5)
    assert code == _native.FK_F32                       # D above XSPLIT_MAX_D
    code, ws = _native.accumulate_x_code(lib, torch.float16, B, N, K, D, 1 << 40, 0.5)
    assert code == _native.FK_F16
    assert ws == lib.fk_assign_accumulate_workspace_size(B, N, K, D, _native.FK_F16)
