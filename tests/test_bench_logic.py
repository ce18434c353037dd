"""Host logic of bench.py (CPU only): the batch split over ranks and the choice
of the binding roofline."""
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


@pytest.mark.parametrize("B", [1, 7, 32, 33])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_batch_range_partitions_every_batch_once(B, world):
    if world > B:
        pytest.skip("more ranks than batches is refused by the bench")
    ranges = [bench._batch_range(B, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == B
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a0 < a1
    sizes = [b - a for a, b in ranges]
    assert max(sizes) - min(sizes) <= 1


def _workload_bytes_flops(name):
    w = bench.WORKLOADS[name]
    es = 2 if w["dtype"] != "float32" else 4
    B, N, D, K = w["B"], w["N"], w["D"], w["K"]
    alg = B * N * D * es + B * N * es + B * K * D * es + B * N * 4 + B * K * D * 4
    return alg, bench._flops(w)


@pytest.mark.parametrize("name,bound", [("cfg2", "tensor"), ("cfg3", "hbm"), ("cfg4", "tensor")])
def test_binding_roofline_per_workload(name, bound):
    burst, hbm = 1675.9, 6443.5   # the measured peaks' magnitudes
    alg, flops = _workload_bytes_flops(name)
    hbm_bound = bench._hbm_bound(alg, flops, burst, hbm)
    assert ("hbm" if hbm_bound else "tensor") == bound
    ms = 1.0
    r = bench._roofline(hbm_bound, flops / (ms * 1e-3) / 1e12, alg, ms, burst, burst * 0.85, hbm,
                        "measured", None)
    assert r["bound"] == bound
    assert r["unit"] == ("GB/s" if bound == "hbm" else "TFLOP/s")
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-3
    assert r["algorithmic_bytes"] == int(alg)
