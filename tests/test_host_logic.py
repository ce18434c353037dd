"""Host-side logic of the drop-in package, CPU only (no kernel launches)."""
import math

import numpy as np
import pytest
import torch

import flash_kmeans
from flash_kmeans import kmeans_large
from flash_kmeans.kmeans_triton_impl import _round_tol


def _reference_partition(N, BLOCK_N, G):
    # formula of kmeans_large.py:69-80 in the reference, restated
    nb = (N + BLOCK_N - 1) // BLOCK_N
    bpg = [nb // G + (1 if g < nb % G else 0) for g in range(G)]
    starts = [sum(bpg[:g]) * BLOCK_N for g in range(G)]
    ends = [min(starts[g] + bpg[g] * BLOCK_N, N) for g in range(G)]
    return bpg, starts, ends


@pytest.mark.parametrize("N", [1, 1000, 1 << 20, (1 << 22) + 7, 1 << 26])
@pytest.mark.parametrize("BLOCK_N", [1 << 16, 1 << 20])
@pytest.mark.parametrize("G", [1, 2, 3, 4, 8])
def test_partition_matches_reference_and_covers(N, BLOCK_N, G):
    bpg, ps, pe = kmeans_large.partition_blocks(N, BLOCK_N, G)
    assert (bpg, ps, pe) == _reference_partition(N, BLOCK_N, G)
    covered = sorted((ps[g], pe[g]) for g in range(G) if bpg[g] > 0)
    assert covered[0][0] == 0 and covered[-1][1] == N
    for (a0, a1), (b0, b1) in zip(covered, covered[1:]):
        assert a1 == b0
    assert max(bpg) - min(bpg) <= 1
    assert sum(bpg) == math.ceil(N / BLOCK_N)


def test_exports_match_reference_all():
    assert flash_kmeans.__all__ == [
        "batch_kmeans_Euclid", "batch_kmeans_Cosine", "batch_kmeans_Dot",
        "triton_centroid_update_euclid", "triton_centroid_update_sorted_euclid",
        "FlashKMeans", "kmeans_largeN", "kmeans_largeN_assign"]
    for name in flash_kmeans.__all__:
        assert callable(getattr(flash_kmeans, name))
    # the reference's module paths import too
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton  # noqa: F401
    from flash_kmeans.centroid_update_triton import triton_centroid_update_sorted_euclid  # noqa
    from flash_kmeans.kmeans_large import _resolve_devices  # noqa: F401


def test_no_cpu_fallback():
    x = torch.randn(2, 100, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        flash_kmeans.batch_kmeans_Euclid(x, 4, max_iters=2)
    km = flash_kmeans.FlashKMeans(d=8, k=4, use_triton=False)
    with pytest.raises(RuntimeError, match="fallback"):
        km.train(x)
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="CUDA"):
            flash_kmeans.kmeans_largeN(x[0], 4, max_iters=1)


def test_flashkmeans_validation_errors():
    km = flash_kmeans.FlashKMeans(d=8, k=4)
    with pytest.raises(RuntimeError, match="not trained"):
        km.predict(torch.randn(10, 8))
    with pytest.raises(ValueError, match="shape"):
        km.train(torch.randn(8))
    km.centroids_b = torch.zeros(1, 4, 8)
    km._batch_size = None
    with pytest.raises(ValueError, match="batch size"):
        km.predict(torch.randn(2, 10, 8))
    assert km.fit is not None and km.fit_predict is not None


def test_cosine_and_dot_have_no_cpu_fallback():
    for fn in (flash_kmeans.batch_kmeans_Cosine, flash_kmeans.batch_kmeans_Dot):
        with pytest.raises(RuntimeError, match="no CPU fallback"):
            fn(torch.randn(1, 4, 4), 2)


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16, torch.float32])
def test_tol_rounds_like_a_zero_dim_tensor_comparison(dt):
    # reference: `center_shift < tol` with a 0-dim tensor of x.dtype
    for tol in (1e-4, 1e-8, 0.3, 0.0, -1.0):
        for shift in (9.99e-5, 1.0e-4, 1.0001e-4, 0.29999, 0.0):
            want = bool(torch.tensor(shift, dtype=dt) < tol)
            got = float(torch.tensor(shift, dtype=dt)) < _round_tol(tol, dt)
            assert got == want, (dt, tol, shift)


def test_tma_layout_predicate():
    from flash_kmeans import _ops
    assert _ops.row_align(torch.float16) == 8 and _ops.row_align(torch.float32) == 4
    x = torch.empty(2, 10, 128, dtype=torch.float16)
    assert _ops.tma_compatible(x)
    assert not _ops.tma_compatible(torch.empty(2, 10, 100, dtype=torch.float16))
    assert _ops.tma_compatible(_ops.empty_rows(2, 10, 100, torch.float16, "cpu"))
    assert not _ops.tma_compatible(x.transpose(1, 2))
    assert _ops.tma_compatible(torch.empty(1, 1, 3, dtype=torch.float32)[..., :3]) in (True, False)


def test_oracle_never_imported_by_package():
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import sys; sys.path.insert(0, 'flash-kmeans_b200'); import flash_kmeans; "
            "import flash_kmeans.kmeans_large, flash_kmeans.interface; "
            "assert not [m for m in sys.modules if m.startswith('oracle')]")
    subprocess.run([sys.executable, "-c", code], cwd=root, check=True)


@pytest.mark.parametrize("K,D,dt", [(128, 128, 0), (380, 128, 0), (400, 128, 0), (1000, 128, 0),
                                    (1000, 128, 1), (1000, 192, 0), (64, 32, 2), (8192, 128, 2),
                                    (300, 100, 2), (100, 512, 0), (100, 600, 0)])
def test_accumulate_method_matches_workspace(K, D, dt):
    """fk_assign_accumulate_method is the choice fk_assign_accumulate makes: only the
    sorted method needs workspace beyond the assignment's; the engine's launch count
    follows it."""
    from flash_kmeans import _native as nat
    lib = nat.load()
    m = lib.fk_assign_accumulate_method(K, D, dt)
    assert m in (nat.FK_ACC_PRIVATISED, nat.FK_ACC_FUSED, nat.FK_ACC_SORTED)
    extra = (lib.fk_assign_accumulate_workspace_size(2, 5000, K, D, dt)
             - lib.fk_assign_workspace_size(2, K, D, dt))
    assert (extra > 0) == (m == nat.FK_ACC_SORTED)
    if m == nat.FK_ACC_FUSED:
        assert dt in (0, 1) and D <= 128
    if m == nat.FK_ACC_PRIVATISED:
        assert K * D * 4 <= 200 * 1024
