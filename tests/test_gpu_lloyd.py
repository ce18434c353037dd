"""GPU parity of the Lloyd drivers (batched, FlashKMeans API, out-of-core)."""
import numpy as np
import pytest
import torch

import cases
from _parity import assert_centroids, assert_labels, clusters_touched
from oracle import kmeans_oracle as ko

pytestmark = pytest.mark.gpu

TD = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _dev(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(TD[dt])


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(scope="module")
def fk():
    import flash_kmeans
    return flash_kmeans


def _teacher_forced(x, c0, K, dt, iters):
    """Run our iteration and the oracle's from the same centroids each step."""
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    B, N, D = x.shape
    xd = _dev(x, dt)
    eng = LloydEngine(B, N, K, D, TD[dt], "cuda")
    cent = ko.round_to(c0, dt)
    eng.load(xd, _dev(cent, dt))
    x_sq = ko.row_sqnorm(x, dt)
    for t in range(iters):
        eng.c_cur.copy_(_dev(cent, dt))   # teacher forcing
        eng.csq_valid = False
        eng.step()
        shift, code = eng.read_stat()
        assert code == 0
        ids = eng.ids.cpu().numpy()
        new = _np(eng.c_nxt)
        o_new, o_shift, o_ids = ko.lloyd_iter(x, x_sq, cent, dt)
        assert_labels(x, cent, ids, o_ids, dt, f"iter {t}")
        touched = clusters_touched(ids, o_ids, K)
        assert_centroids(new, o_new, f"iter {t}", skip=touched)
        # the update itself, fed the oracle's labels, matches to float rounding
        from flash_kmeans import triton_centroid_update_sorted_euclid as upd
        new2 = _np(upd(xd, torch.from_numpy(o_ids).cuda(), _dev(cent, dt)))
        assert_centroids(new2, o_new, f"iter {t} (oracle labels)")
        assert abs(shift - o_shift) <= 2e-3 * max(abs(o_shift), 1e-3) + 1e-6
        cent = o_new


@pytest.mark.parametrize("spec", cases.LLOYD_CASES, ids=lambda s: s["name"])
def test_lloyd_teacher_forced_vs_oracle(fk, spec):
    x, c0 = cases.lloyd_inputs(spec)
    _teacher_forced(ko.round_to(x, spec["dtype"]), c0, spec["K"], spec["dtype"], min(3, spec["iters"]))


@pytest.mark.parametrize("spec", cases.LLOYD_CASES, ids=lambda s: s["name"])
def test_lloyd_free_running_vs_reference(fk, spec):
    x, c0 = cases.lloyd_inputs(spec)
    dt = spec["dtype"]
    ids, cent, n_it = fk.batch_kmeans_Euclid(_dev(x, dt), spec["K"], max_iters=spec["iters"],
                                             tol=spec["tol"], init_centroids=_dev(c0, dt))
    g = np.load(cases.path(spec["name"]))
    assert ids.dtype == torch.int32 and ids.shape == (spec["B"], spec["N"])
    assert cent.dtype == TD[dt] and cent.shape == (spec["B"], spec["K"], spec["D"])
    assert n_it == int(g["n_iters"])
    # Untethered: a near-tie resolved differently early can steer later iterations,
    # so this is a loose agreement check (the strict bar is the teacher-forced test).
    agree = (ids.cpu().numpy() == g["ids"]).mean()
    assert agree >= 0.99, agree
    touched = clusters_touched(ids.cpu().numpy(), g["ids"], spec["K"])
    assert_centroids(_np(cent), g["centroids"], spec["name"], skip=touched, rtol=1e-2)


def test_lloyd_tol_break_returns_pre_update_centroids(fk):
    spec = next(s for s in cases.LLOYD_CASES if s["tol"] > 0)
    x, c0 = cases.lloyd_inputs(spec)
    dt = spec["dtype"]
    ids, cent, n_it = fk.batch_kmeans_Euclid(_dev(x, dt), spec["K"], max_iters=spec["iters"],
                                             tol=spec["tol"], init_centroids=_dev(c0, dt))
    hist = []
    o_ids, o_cent, o_n = ko.batch_kmeans_euclid(x, spec["K"], spec["iters"], spec["tol"],
                                                init_centroids=c0, dtype=dt, history=hist)
    assert n_it == o_n < spec["iters"]
    xq = ko.round_to(x, dt)
    assert_labels(xq, o_cent, ids.cpu().numpy(), o_ids, dt, "tol break")
    touched = clusters_touched(ids.cpu().numpy(), o_ids, spec["K"])
    assert_centroids(_np(cent), o_cent, "tol break", skip=touched)


def test_cfg2_slice_teacher_forced(fk):
    """BASELINE config 2 shapes (N=75600, K=1000, D=128, fp16), two batches, 2 iterations."""
    rng = np.random.default_rng(2)
    B, N, K, D = 2, 75600, 1000, 128
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), "float16")
    c0 = ko.init_from_points(rng, x, K, replace=True)
    _teacher_forced(x, c0, K, "float16", 2)


def test_random_init_uses_cuda_rng_like_reference(fk):
    """init_centroids=None draws randint(0, N, (B, K)) on x.device, as the reference."""
    torch.manual_seed(7)
    x = torch.randn(2, 4096, 64, device="cuda").half()
    ids, cent, _ = fk.batch_kmeans_Euclid(x, 32, max_iters=1)
    torch.manual_seed(7)
    _ = torch.randn(2, 4096, 64, device="cuda")
    idx = torch.randint(0, 4096, (2, 32), device="cuda")
    c0 = torch.gather(x, 1, idx[..., None].expand(-1, -1, 64))
    ids2, cent2, _ = fk.batch_kmeans_Euclid(x, 32, max_iters=1, init_centroids=c0)
    # the same initial centroids; the cluster sums are float atomics whose order
    # varies between runs, so the centroids agree to rounding, not bit for bit
    assert (ids == ids2).float().mean().item() >= 0.999
    torch.testing.assert_close(cent.float(), cent2.float(), rtol=2e-3, atol=2e-3)


def test_flashkmeans_api_matches_raw(fk):
    """Port of examples/testapi.py: fit_predict == batch_kmeans_Euclid under one seed."""
    B, N, K, D = 4, 20000, 200, 128
    data = torch.randn(B, N, D, device="cuda", dtype=torch.float16)
    km = fk.FlashKMeans(d=D, k=K, niter=8, seed=42, device=torch.device("cuda:0"))
    api = km.fit_predict(data)
    torch.manual_seed(42)
    torch.cuda.manual_seed_all(42)
    raw, cent, _ = fk.batch_kmeans_Euclid(data, n_clusters=K, max_iters=8, tol=1e-8)
    # Same seed -> same init and the same run.  Per-cluster sums are float32
    # atomics (as in the reference's Triton update), so the two runs may differ
    # in the last bit of a sum; compare at the parity bar, not bit for bit.
    agree = (api == raw).float().mean().item()
    assert agree >= 0.999, agree
    assert_centroids(_np(km.centroids_b), _np(cent), "api vs raw")
    pred = km.predict(data)
    # predict against the final centroids differs from the training labels only by
    # the last update; it must equal a fresh assignment
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign
    again = euclid_assign(data, km.centroids_b, _ops.row_sqnorm(data))
    assert torch.equal(pred, again)
    # 2-D input squeezes the batch axis
    km2 = fk.FlashKMeans(d=D, k=K, niter=3, seed=1)
    lab = km2.fit_predict(data[0])
    assert lab.shape == (N,) and lab.dtype == torch.int32
    assert km2.predict(data[0]).shape == (N,)
    with pytest.raises(ValueError):
        km2.predict(data)


def test_kmeans_largeN_single_gpu_vs_oracle(fk):
    rng = np.random.default_rng(4)
    N, K, D = 300_000, 64, 32
    x = rng.standard_normal((N, D), dtype=np.float32)
    c0 = x[rng.integers(0, N, K)]
    xt = torch.from_numpy(x).pin_memory()
    # one pass from the same centroids: the oracle's labels and update
    labels, cent = fk.kmeans_largeN(xt, K, max_iters=1, tol=-1, BLOCK_N=70_000,
                                    init_centroids=torch.from_numpy(c0), device="cuda:0")
    assert labels.is_cuda and labels.shape == (N,) and labels.dtype == torch.int32
    o_ids, o_cent = ko.kmeans_large_n(x, K, 1, -1.0, init_centroids=c0, dtype="float32")
    assert_labels(x[None], c0[None], labels.cpu().numpy()[None], o_ids[None], "float32", "largeN")
    touched = clusters_touched(labels.cpu().numpy()[None], o_ids[None], K)
    assert_centroids(_np(cent)[None], o_cent[None], "largeN", skip=touched)
    # several passes, free-running: float32 summation order moves near-tie points, and
    # the difference compounds, so check self-consistency (returned centroids are the
    # update of the returned labels) and near-agreement with the oracle
    labels4, cent4 = fk.kmeans_largeN(xt, K, max_iters=4, tol=-1, BLOCK_N=70_000,
                                      init_centroids=torch.from_numpy(c0), device="cuda:0")
    l4 = labels4.cpu().numpy()
    upd = ko.centroid_update(x[None], l4[None], _np(cent4)[None], "float32")
    assert_centroids(_np(cent4)[None], upd, "largeN x4 self-consistent")
    o4, _ = ko.kmeans_large_n(x, K, 4, -1.0, init_centroids=c0, dtype="float32")
    assert (l4 == o4).mean() >= 0.999
    # assign-only pipeline agrees with a direct assignment
    lab2 = fk.kmeans_largeN_assign(xt, cent, BLOCK_N=70_000, device="cuda:0")
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign
    xd = xt.cuda()[None]
    direct = euclid_assign(xd, cent[None], _ops.row_sqnorm(xd))[0]
    assert torch.equal(lab2, direct)


def test_kmeans_largeN_streaming_equals_resident(fk):
    """Slices that fit in HBM are copied once and kept resident (the default here); the
    streaming pipeline (double-buffered blocks, next pass prefetched) gives the same run."""
    rng = np.random.default_rng(12)
    x = ko.gmm_points(rng, 1, 200_000, 24, 16, 5.0)[0]
    c0 = torch.from_numpy(x[rng.integers(0, len(x), 16)])
    xt = torch.from_numpy(x).pin_memory()
    lab_r, cent_r = fk.kmeans_largeN(xt, 16, max_iters=5, tol=-1, BLOCK_N=30_000,
                                     init_centroids=c0, device="cuda:0")
    lab_s, cent_s = fk.kmeans_largeN(xt, 16, max_iters=5, tol=-1, BLOCK_N=30_000,
                                     init_centroids=c0, device="cuda:0", resident=False)
    # float32 atomics sum in a different order run to run, so a few near-tie points may
    # move over 5 free-running iterations: the north star's label / centroid bar
    assert (lab_r == lab_s).double().mean().item() >= 0.999
    assert_centroids(_np(cent_s)[None], _np(cent_r)[None], "streaming vs resident")


def test_kmeans_largeN_tol_break_returns_new_centroids(fk):
    """On a tolerance break kmeans_largeN returns the centroids UPDATED from the
    returned labels (kmeans_large.py:251-258), unlike batch_kmeans_Euclid."""
    rng = np.random.default_rng(8)
    x = ko.gmm_points(rng, 1, 50_000, 16, 8, 6.0)[0]
    c0 = x[rng.integers(0, len(x), 8)]
    labels, cent = fk.kmeans_largeN(torch.from_numpy(x), 8, max_iters=100, tol=1e-3,
                                    BLOCK_N=16_384, init_centroids=torch.from_numpy(c0),
                                    device="cuda:0")
    lab = labels.cpu().numpy()
    # the returned centroids are the means of the returned labelling ...
    upd = ko.centroid_update(x[None], lab[None], _np(cent)[None], "float32", exact_order=False)
    assert_centroids(_np(cent)[None], upd, "centroids are the update of the labels", rtol=1e-5)
    # ... and the run had converged: one more assignment barely moves anything
    again = ko.assign(x[None], _np(cent)[None], ko.row_sqnorm(x[None], "float32"), "float32")[0]
    assert (again == lab).mean() > 0.999


@pytest.mark.parametrize("metric,dt,K,D", [("euclid", "float16", 1000, 128),   # fused
                                           ("euclid", "float32", 700, 96),     # sorted
                                           ("euclid", "bfloat16", 64, 64),     # privatised
                                           ("dot", "float16", 1000, 128)])
def test_engine_graph_replay_matches_eager(fk, metric, dt, K, D):
    """Steps replayed from CUDA graphs give the eager steps' labels and
    centroids (well-separated clusters, so float-atomic order cannot flip a
    label), and the graphs are really used."""
    from flash_kmeans import _ops
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    rng = np.random.default_rng(77)
    B, N = 2, 6000
    x = ko.round_to(ko.gmm_points(rng, B, N, D, K, 8.0), dt)
    c0 = ko.init_from_points(rng, x, K, replace=False)
    xd, cd = _dev(x, dt), _dev(c0, dt)
    if metric == "dot":
        xd, cd = _ops.row_normalize(xd), _ops.row_normalize(cd)
    out = []
    for graphs in (False, True):
        eng = LloydEngine(B, N, K, D, TD[dt], "cuda", metric=metric, use_graphs=graphs)
        eng.load(xd, cd)
        shifts = []
        for _ in range(5):
            eng.step()
            shifts.append(eng.read_stat())
            eng.advance()
        assert all(code == 0 for _, code in shifts)
        out.append((eng.ids.cpu().numpy(), _np(eng.result_centroids()), [sh for sh, _ in shifts]))
        if graphs:
            assert eng.use_graphs and len(eng._graphs) == 3   # one pair per centroid buffer
    np.testing.assert_array_equal(out[0][0], out[1][0])
    assert_centroids(out[1][1], out[0][1], "graph vs eager", rtol=1e-5)
    # once converged the shift is float-atomic-order noise: compare on the
    # scale of the first shift
    np.testing.assert_allclose(out[1][2], out[0][2], rtol=1e-3, atol=1e-5 * max(out[0][2]))


@pytest.mark.gpu
def test_pipelined_run_break_semantics(fk, capsys):
    """batch_kmeans_Euclid queues iteration it+1 before reading iteration it's shift
    (LloydEngine.run); a break must still return iteration it's labels and the
    centroids that produced them, untouched by the discarded iteration."""
    from flash_kmeans.assign_euclid_triton import euclid_assign
    from flash_kmeans import _ops
    rng = np.random.default_rng(31)
    B, N, K, D = 2, 3000, 40, 64
    x = _dev(ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), "float16"), "float16")
    c0 = x[:, :K].clone()
    # break at the first check: the initial centroids and their labels, bit for bit
    ids, cent, n_it = fk.batch_kmeans_Euclid(x, K, max_iters=10, tol=1e9, init_centroids=c0,
                                             verbose=True)
    assert n_it == 1
    assert torch.equal(cent, c0)
    assert torch.equal(ids, euclid_assign(x, c0, _ops.row_sqnorm(x)))
    assert capsys.readouterr().out.splitlines()[0].startswith("Iter 0, center shift:")
    # no break: the last labels and the last update's centroids, as the synchronous loop
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    for iters in (1, 2, 5):
        ids, cent, n_it = fk.batch_kmeans_Euclid(x, K, max_iters=iters, tol=-1.0, init_centroids=c0,
                                                 verbose=True)
        lines = capsys.readouterr().out.splitlines()
        assert n_it == iters and len(lines) == iters
        eng = LloydEngine(B, N, K, D, x.dtype, x.device, use_graphs=False)
        eng.load(x, c0)
        for _ in range(iters):
            eng.step()
            _, code = eng.read_stat()
            assert code == 0
            ids_sync = eng.ids.clone()
            eng.advance()
        agree = (ids == ids_sync).double().mean().item()
        assert agree >= 0.999, agree   # float32 atomics: centroids may differ in the last bits
        assert_centroids(_np(cent), _np(eng.result_centroids()), f"{iters} iterations")
