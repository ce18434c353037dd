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
  result (torch_fallback.py:137-178);
* cosine / dot: ``F.normalize`` rows (kmeans_triton_impl.py:135), the argmax of
  the float32 einsum the reference checks ``cosine_assign_triton`` against
  (examples/test_assign_dtype_d.py:101-106), ``_centroid_update_torch_native``
  with ``mode='cosine'`` (torch_fallback.py:72-109), and Lloyd chains made of
  those steps in the order of ``_cosine_iter`` / ``_dot_iter``
  (kmeans_triton_impl.py:19-35) driven as ``batch_kmeans_Cosine`` / ``_Dot``
  drive them (kmeans_triton_impl.py:118-188).

An optional second argument names the groups to (re)write, comma separated:
``assign,update,lloyd,normalize,sim`` (default: all); an optional third one
names the cases to (re)write within those groups (default: all).

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


GROUPS = ("assign", "update", "lloyd", "normalize", "sim")


def main(ref_root: str, groups=GROUPS, only=None) -> None:
    sys.path.insert(0, ref_root)
    from flash_kmeans import torch_fallback as tf  # the reference's oracle

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if "assign" in groups:
        _assign(tf, only)
    if "update" in groups:
        _update(tf)
    if "lloyd" in groups:
        _lloyd(tf)
    if "normalize" in groups:
        _normalize()
    if "sim" in groups:
        _similarity(tf)


def _assign(tf, only=None):
    for spec in cases.ASSIGN_CASES:
        if only and spec["name"] not in only:
            continue
        x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
        dt = spec["dtype"]
        ids = tf.euclid_assign_torch_native_chunked(_t(x, dt), _t(c, dt), _t(xsq, xsq_dtype))
        np.savez_compressed(cases.path(spec["name"]), ids=ids.numpy().astype(np.int32),
                            checksum=cases.checksum(x, c, xsq))
        print("wrote", spec["name"])


def _update(tf):
    for spec in cases.UPDATE_CASES:
        x, ids, old = cases.update_inputs(spec)
        dt = spec["dtype"]
        new = tf._centroid_update_torch_native(_t(x, dt), torch.from_numpy(ids).long(), _t(old, dt))
        np.savez_compressed(cases.path(spec["name"]), centroids=_np(new),
                            checksum=cases.checksum(x, ids, old))
        print("wrote", spec["name"])


def _lloyd(tf):
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


def _normalize():
    import torch.nn.functional as F
    for spec in cases.NORMALIZE_CASES:
        x = cases.normalize_inputs(spec)
        y = F.normalize(_t(x, spec["dtype"]), p=2, dim=-1)
        np.savez_compressed(cases.path(spec["name"]), y=_np(y), checksum=cases.checksum(x))
        print("wrote", spec["name"])


def _scores_argmax(xs, c):
    # the float32 einsum + argmax of examples/test_assign_dtype_d.py:101-106
    return torch.einsum("bnd,bkd->bnk", xs.float(), c.float()).argmax(dim=-1)


def _similarity(tf):
    import torch.nn.functional as F
    for spec in cases.SIM_ASSIGN_CASES:
        x, c = cases.sim_assign_inputs(spec)
        xt, ct = _t(x, spec["dtype"]), _t(c, spec["dtype"])
        if spec["cosine"]:
            xt, ct = F.normalize(xt, dim=-1), F.normalize(ct, dim=-1)
        ids = _scores_argmax(xt, ct)
        np.savez_compressed(cases.path(spec["name"]), ids=ids.numpy().astype(np.int32),
                            checksum=cases.checksum(x, c))
        print("wrote", spec["name"])

    for spec in cases.SIM_UPDATE_CASES:
        x, ids, old = cases.sim_update_inputs(spec)
        dt = spec["dtype"]
        xs = F.normalize(_t(x, dt), dim=-1)
        new = tf._centroid_update_torch_native(xs, torch.from_numpy(ids).long(), _t(old, dt),
                                               mode="cosine")
        np.savez_compressed(cases.path(spec["name"]), centroids=_np(new),
                            checksum=cases.checksum(x, ids, old))
        print("wrote", spec["name"])

    for spec in cases.SIM_LLOYD_CASES:
        x, c0 = cases.sim_lloyd_inputs(spec)
        dt, cosine = spec["dtype"], spec["cosine"]
        B, K, D = spec["B"], spec["K"], spec["D"]
        xs = _t(x, dt)
        cent = _t(c0, dt).view(B, K, D)
        if cosine:
            xs, cent = F.normalize(xs, p=2, dim=-1), F.normalize(cent, p=2, dim=-1)
        init = cent.clone()
        ids_hist, cent_hist, shifts = [], [], []
        for _ in range(spec["iters"]):
            ids = _scores_argmax(xs, cent)
            new = tf._centroid_update_torch_native(xs, ids, cent, mode="cosine")
            shifts.append(float((new - cent).norm(dim=-1).max()))
            ids_hist.append(ids.numpy().astype(np.int16))
            cent_hist.append(_np(new))
            cent = new.clone()
        np.savez_compressed(cases.path(spec["name"]), init=_np(init),
                            trace_ids=np.stack(ids_hist), trace_centroids=np.stack(cent_hist),
                            trace_shifts=np.asarray(shifts, np.float32),
                            checksum=cases.checksum(x, c0))
        print("wrote", spec["name"], "shifts", shifts)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3, 4):
        sys.exit("usage: make_golden.py /path/to/flash-kmeans-checkout [group,...] [case,...]")
    main(sys.argv[1], tuple(sys.argv[2].split(",")) if len(sys.argv) >= 3 else GROUPS,
         set(sys.argv[3].split(",")) if len(sys.argv) == 4 else None)
