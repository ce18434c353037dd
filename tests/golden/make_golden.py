"""Generate the golden vectors in ``tests/golden/`` from the reference itself.

Run once, on a machine where the reference Flash-KMeans checkout is
importable (CPU is enough)::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py /path/to/flash-kmeans

It imports the reference's pure-torch path (``flash_kmeans/torch_fallback.py``,
the project's parity oracle) and records, for every spec in ``cases.py``:

* assignment: ``euclid_assign_torch_native_chunked`` labels
  (torch_fallback.py:4-52);
* update: ``_centroid_update_torch_native`` centroids (torch_fallback.py:72-108);
* Lloyd: per-iteration ``_euclid_iter_torch_naive`` outputs
  (torch_fallback.py:111-135) and the final ``batch_kmeans_Euclid_torch_native``
  result (torch_fallback.py:137-178).

Inputs are rebuilt from their seeds by ``cases.py``; fixtures store outputs and
an input checksum.  Nothing at test time reads the reference checkout.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases  # noqa: E402

TORCH_DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _t(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(TORCH_DT[dt])


def _np(t):
    return t.detach().to(torch.float32).numpy()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from flash_kmeans import torch_fallback as tf  # the reference's oracle

    torch.set_num_threads(max(1, os.cpu_count() or 1))

    for spec in cases.ASSIGN_CASES:
        x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
        dt = spec["dtype"]
        ids = tf.euclid_assign_torch_native_chunked(_t(x, dt), _t(c, dt), _t(xsq, xsq_dtype))
        np.savez_compressed(cases.path(spec["name"]), ids=ids.numpy().astype(np.int32),
                            checksum=cases.checksum(x, c, xsq))
        print("wrote", spec["name"])

    for spec in cases.UPDATE_CASES:
        x, ids, old = cases.update_inputs(spec)
        dt = spec["dtype"]
        new = tf._centroid_update_torch_native(_t(x, dt), torch.from_numpy(ids).long(), _t(old, dt))
        np.savez_compressed(cases.path(spec["name"]), centroids=_np(new),
                            checksum=cases.checksum(x, ids, old))
        print("wrote", spec["name"])

    for spec in cases.LLOYD_CASES:
        x, c0 = cases.lloyd_inputs(spec)
        dt = spec["dtype"]
        xt, ct = _t(x, dt), _t(c0, dt)
        # per-iteration trace (teacher-forced chain of the oracle itself)
        x_sq = (xt ** 2).sum(dim=-1)
        shifts, ids_hist = [], []
        cent = ct
        trace_iters = min(spec["iters"], 3)
        for _ in range(trace_iters):
            new, shift, ids = tf._euclid_iter_torch_naive(xt, x_sq, cent)
            shifts.append(float(shift))
            ids_hist.append(ids.numpy().astype(np.int32))
            cent = new.clone()
        ids_f, cent_f, n_it = tf.batch_kmeans_Euclid_torch_native(
            xt, spec["K"], max_iters=spec["iters"], tol=spec["tol"], init_centroids=ct)
        K = spec["K"]
        id_dtype = np.int16 if K < 32768 else np.int32
        np.savez_compressed(
            cases.path(spec["name"]),
            trace_ids=np.stack(ids_hist).astype(id_dtype),
            trace_shifts=np.asarray(shifts, np.float32),
            ids=ids_f.numpy().astype(id_dtype),
            centroids=_np(cent_f),
            n_iters=np.int32(n_it),
            checksum=cases.checksum(x, c0))
        print("wrote", spec["name"], "n_iters", n_it)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py /path/to/flash-kmeans-checkout")
    main(sys.argv[1])
