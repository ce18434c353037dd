"""GPU parity of the cosine / dot-product k-means path against the oracle and
the reference's golden vectors.

The kernels (row normalisation, dot-product argmax assignment, normalised
finalize) run through the C ABI; the numpy oracle is the checker only.
"""
import zlib

import numpy as np
import pytest
import torch

import cases
from _parity import assert_centroids, assert_labels, clusters_touched
from oracle import kmeans_oracle as ko

pytestmark = pytest.mark.gpu

TD = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
# a unit of the dtype at 1.0: the per-element bound for a normalised row
ULP1 = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -23}


def _dev(a, dt):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(TD[dt])


def _np(t):
    return t.detach().float().cpu().numpy()


def _rng(*key):
    return np.random.default_rng(zlib.crc32(repr(key).encode()))


@pytest.fixture(scope="module")
def fk():
    import flash_kmeans
    from flash_kmeans import _native
    _native.load()
    return flash_kmeans


# ------------------------------------------------------------- normalisation
@pytest.mark.parametrize("spec", cases.NORMALIZE_CASES, ids=lambda s: s["name"])
def test_row_normalize_matches_golden(fk, spec):
    from flash_kmeans import _ops
    x = cases.normalize_inputs(spec)
    dt = spec["dtype"]
    got = _np(_ops.row_normalize(_dev(x, dt)))
    want = np.load(cases.path(spec["name"]))["y"]
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))  # the zero row
    ok = ~np.isnan(want)
    # the float32 norm's summation order can move the quotient by a unit or two
    err = np.abs(got[ok] - want[ok]) / np.maximum(np.abs(want[ok]), 1e-30)
    assert err.max() <= 2.01 * ULP1[dt] * 2, err.max()
    oracle = ko.normalize_rows(x, dt)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(oracle))
    assert (got[ok] != oracle[ok]).mean() < (0.3 if dt == "float32" else 0.02)


@pytest.mark.parametrize("dt", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("D", [1, 7, 64, 100, 128, 1000])
def test_row_normalize_shapes_and_strides(fk, dt, D):
    from flash_kmeans import _ops
    rng = _rng("norm", dt, D)
    x = ko.round_to(rng.standard_normal((3, 77, D), dtype=np.float32) * 5, dt)
    xd = _dev(x, dt)
    got = _np(_ops.row_normalize(xd))
    want = ko.normalize_rows(x, dt)
    err = np.abs(got - want) / np.maximum(np.abs(want), 1e-30)
    assert err.max() <= 2.01 * ULP1[dt] * 2
    # a strided (transposed-batch) view gives the same rows
    xt = xd.transpose(0, 1).contiguous().transpose(0, 1)
    assert torch.equal(_ops.row_normalize(xt), _ops.row_normalize(xd))


# ---------------------------------------------------------------- assignment
@pytest.mark.parametrize("spec", cases.SIM_ASSIGN_CASES, ids=lambda s: s["name"])
def test_dot_assign_matches_golden_and_oracle(fk, spec):
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import cosine_assign_triton
    x, c = cases.sim_assign_inputs(spec)
    dt = spec["dtype"]
    xd, cd = _dev(x, dt), _dev(c, dt)
    if spec["cosine"]:
        xd, cd = _ops.row_normalize(xd), _ops.row_normalize(cd)
    got = cosine_assign_triton(xd, cd).cpu().numpy()
    xs, cs = _np(xd), _np(cd)
    golden = np.load(cases.path(spec["name"]))["ids"]
    assert_labels(xs, cs, got, golden, dt, spec["name"] + " vs reference", metric="dot")
    assert_labels(xs, cs, got, ko.assign_dot(xs, cs), dt, spec["name"] + " vs oracle",
                  metric="dot")


SIM_SHAPES = [  # (B, N, K, D): tails in N, K and D; x-resident and split-D; one and many tiles
    (1, 1, 1, 16), (1, 5, 3, 8), (2, 127, 7, 64), (1, 129, 255, 128), (1, 300, 256, 32),
    (1, 257, 257, 96), (3, 200, 19, 100), (1, 1000, 513, 17), (1, 640, 70, 192),
    (1, 333, 300, 513), (2, 4099, 1000, 128),
]


@pytest.mark.parametrize("dt", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("shape", SIM_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("sign", ["mixed", "negative"])
def test_dot_assign_shapes_vs_oracle(fk, dt, shape, sign):
    """Raw dot products, including all-negative scores (the padded columns of
    the last centroid tile must never win) and one-centroid batches."""
    from flash_kmeans.assign_euclid_triton import cosine_assign_triton
    B, N, K, D = shape
    rng = _rng("dot", dt, shape, sign)
    x = rng.standard_normal((B, N, D), dtype=np.float32)
    c = rng.standard_normal((B, K, D), dtype=np.float32)
    if sign == "negative":
        x, c = np.abs(x), -np.abs(c)
    x, c = ko.round_to(x, dt), ko.round_to(c, dt)
    got = cosine_assign_triton(_dev(x, dt), _dev(c, dt)).cpu().numpy()
    assert got.min() >= 0 and got.max() < K
    assert_labels(x, c, got, ko.assign_dot(x, c), dt, f"{dt} {shape} {sign}", metric="dot")


def test_dot_assign_ties_take_lowest_index(fk):
    from flash_kmeans.assign_euclid_triton import cosine_assign_triton
    rng = _rng("dot-ties")
    base = ko.round_to(rng.standard_normal((1, 40, 64), dtype=np.float32), "float16")
    c = np.concatenate([base, base, base], axis=1)  # K = 120, three copies of each
    x = ko.round_to(rng.standard_normal((1, 3000, 64), dtype=np.float32), "float16")
    got = cosine_assign_triton(_dev(x, "float16"), _dev(c, "float16")).cpu().numpy()
    assert got.max() < 40, "equal scores must resolve to the first copy"
    want = ko.assign_dot(x, c)
    assert_labels(x, c, got, want, "float16", "ties", metric="dot")


def test_dot_assign_counts_and_out(fk):
    """fk_assign_dot's optional per-cluster counts equal the labels' histogram;
    ``out`` is written in place (strided)."""
    from flash_kmeans import _ops
    rng = _rng("dot-counts")
    B, N, K, D = 3, 5000, 300, 128
    x = _dev(rng.standard_normal((B, N, D), dtype=np.float32), "float16")
    c = _dev(rng.standard_normal((B, K, D), dtype=np.float32), "float16")
    counts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
    big = torch.full((B, 2 * N), -1, dtype=torch.int32, device="cuda")
    out = big[:, ::2]
    _ops.assign_dot(x, c, out=out, counts=counts)
    ids = out.cpu().numpy()
    assert (big[:, 1::2] == -1).all()
    for b in range(B):
        np.testing.assert_array_equal(counts[b].cpu().numpy(), np.bincount(ids[b], minlength=K))
    ref = _ops.assign_dot(x, c)
    assert torch.equal(ref, out)


def test_dot_assign_deterministic(fk):
    from flash_kmeans.assign_euclid_triton import cosine_assign_triton
    rng = _rng("dot-det")
    x = _dev(rng.standard_normal((4, 20000, 128), dtype=np.float32), "bfloat16")
    c = _dev(rng.standard_normal((4, 1000, 128), dtype=np.float32), "bfloat16")
    a = cosine_assign_triton(x, c)
    for _ in range(3):
        assert torch.equal(a, cosine_assign_triton(x, c))


# -------------------------------------------------------------------- update
@pytest.mark.parametrize("spec", cases.SIM_UPDATE_CASES, ids=lambda s: s["name"])
@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_cosine_update_matches_golden(fk, spec, idt):
    from flash_kmeans import _ops
    from flash_kmeans.centroid_update_triton import triton_centroid_update_sorted_cosine
    x, ids, old = cases.sim_update_inputs(spec)
    dt = spec["dtype"]
    xs = _ops.row_normalize(_dev(x, dt))
    new = triton_centroid_update_sorted_cosine(xs, torch.from_numpy(ids).to("cuda", idt),
                                               _dev(old, dt))
    assert new.dtype == TD[dt] and new.shape == (spec["B"], spec["K"], spec["D"])
    got = _np(new)
    golden = np.load(cases.path(spec["name"]))["centroids"]
    assert_centroids(got, golden, spec["name"] + " vs reference")
    want = ko.centroid_update_cosine(_np(xs), ids, old, dt)
    assert_centroids(got, want, spec["name"] + " vs oracle")
    # empty clusters: the old centroid, normalised
    cnt = np.stack([np.bincount(ids[b], minlength=spec["K"]) for b in range(spec["B"])])
    old_n = ko.finalize_normalized(np.zeros_like(old), np.zeros(cnt.shape), old, dt)
    assert_centroids(got[cnt == 0][None], old_n[cnt == 0][None], "empty clusters", rtol=2e-3)


@pytest.mark.parametrize("dt,B,N,K,D", [("float16", 2, 9000, 1000, 128),   # sorted path
                                        ("bfloat16", 1, 7000, 200, 64),    # privatised path
                                        ("float32", 2, 3000, 50, 300)])
def test_cosine_update_large_k_and_d(fk, dt, B, N, K, D):
    from flash_kmeans.centroid_update_triton import triton_centroid_update_cosine
    rng = _rng("cos-upd", dt, B, N, K, D)
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    ids = rng.integers(0, K, (B, N)).astype(np.int32)
    old = ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    got = _np(triton_centroid_update_cosine(_dev(x, dt), torch.from_numpy(ids).cuda(), _dev(old, dt)))
    want = ko.centroid_update_cosine(x, ids, old, dt, exact_order=False)
    assert_centroids(got, want, f"{dt} {B}x{N}x{K}x{D}")
    nrm = np.linalg.norm(got.astype(np.float64), axis=-1)
    assert np.abs(nrm - 1).max() < {"float16": 2e-3, "bfloat16": 1e-2, "float32": 1e-5}[dt]


# --------------------------------------------------------------------- Lloyd
def _engine_teacher_forced(xs, cent0, K, dt, golden):
    """Our dot-metric iteration from the reference chain's centroids at every step."""
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    B, N, D = xs.shape
    eng = LloydEngine(B, N, K, D, TD[dt], "cuda", metric="dot")
    eng.load(_dev(xs, dt), _dev(cent0, dt))
    cent = cent0
    for t in range(golden["trace_ids"].shape[0]):
        eng.c_cur.copy_(_dev(cent, dt))
        eng.step()
        shift, code = eng.read_stat()
        assert code == 0
        ids = eng.ids.cpu().numpy()
        assert_labels(xs, cent, ids, golden["trace_ids"][t], dt, f"iter {t} labels", metric="dot")
        touched = clusters_touched(ids, golden["trace_ids"][t], K)
        assert_centroids(_np(eng.c_nxt), golden["trace_centroids"][t], f"iter {t}", skip=touched)
        want_shift = float(golden["trace_shifts"][t])
        if not touched.any():
            assert abs(shift - want_shift) <= 2e-3 * max(want_shift, 1e-3) + 1e-6
        cent = golden["trace_centroids"][t]


@pytest.mark.parametrize("spec", cases.SIM_LLOYD_CASES, ids=lambda s: s["name"])
def test_similarity_lloyd_teacher_forced_vs_reference(fk, spec):
    from flash_kmeans import _ops
    x, c0 = cases.sim_lloyd_inputs(spec)
    dt = spec["dtype"]
    g = np.load(cases.path(spec["name"]))
    xs = _np(_ops.row_normalize(_dev(x, dt))) if spec["cosine"] else ko.round_to(x, dt)
    _engine_teacher_forced(xs, g["init"], spec["K"], dt, g)


@pytest.mark.parametrize("spec", cases.SIM_LLOYD_CASES, ids=lambda s: s["name"])
def test_similarity_drivers_free_running(fk, spec):
    x, c0 = cases.sim_lloyd_inputs(spec)
    dt = spec["dtype"]
    fn = fk.batch_kmeans_Cosine if spec["cosine"] else fk.batch_kmeans_Dot
    ids, cent, n_it = fn(_dev(x, dt), spec["K"], max_iters=spec["iters"],
                         init_centroids=_dev(c0, dt))
    assert ids.dtype == torch.int32 and ids.shape == (spec["B"], spec["N"])
    assert cent.dtype == TD[dt] and cent.shape == (spec["B"], spec["K"], spec["D"])
    assert n_it == spec["iters"]
    g = np.load(cases.path(spec["name"]))
    agree = (ids.cpu().numpy() == g["trace_ids"][-1]).mean()
    assert agree >= 0.99, agree
    touched = clusters_touched(ids.cpu().numpy(), g["trace_ids"][-1], spec["K"])
    assert_centroids(_np(cent), g["trace_centroids"][-1], spec["name"], skip=touched, rtol=1e-2)


def test_cosine_tol_break_returns_pre_update_centroids(fk):
    rng = _rng("cos-tol")
    B, N, K, D = 2, 4000, 12, 32
    x = ko.round_to(ko.gmm_points(rng, B, N, D, K, 6.0), "float16")
    c0 = ko.init_from_points(rng, x, K, replace=False)
    tol = 1e-3
    ids, cent, n_it = fk.batch_kmeans_Cosine(_dev(x, "float16"), K, max_iters=50, tol=tol,
                                             init_centroids=_dev(c0, "float16"))
    hist = []
    o_ids, o_cent, o_n = ko.batch_kmeans_similarity(x, K, 50, tol, init_centroids=c0,
                                                    dtype="float16", cosine=True, history=hist)
    assert n_it == o_n < 50
    xs = ko.normalize_rows(x, "float16")
    assert_labels(xs, o_cent, ids.cpu().numpy(), o_ids, "float16", "tol break", metric="dot")
    touched = clusters_touched(ids.cpu().numpy(), o_ids, K)
    assert_centroids(_np(cent), o_cent, "tol break", skip=touched)


def test_cosine_random_init_uses_cuda_rng_like_reference(fk):
    """init_centroids=None gathers randint(0, N, (B, K)) rows of the normalised x."""
    from flash_kmeans import _ops
    torch.manual_seed(11)
    x = torch.randn(2, 4096, 64, device="cuda").half()
    ids, cent, _ = fk.batch_kmeans_Cosine(x, 32, max_iters=2)
    torch.manual_seed(11)
    _ = torch.randn(2, 4096, 64, device="cuda")
    idx = torch.randint(0, 4096, (2, 32), device="cuda")
    c0 = torch.gather(_ops.row_normalize(x), 1, idx[..., None].expand(-1, -1, 64))
    ids2, cent2, _ = fk.batch_kmeans_Cosine(x, 32, max_iters=2, init_centroids=c0)
    # the same initial centroids; the cluster sums are float atomics whose order
    # varies between runs, so the centroids agree to rounding, not bit for bit
    assert (ids == ids2).float().mean().item() >= 0.999
    torch.testing.assert_close(cent.float(), cent2.float(), rtol=2e-3, atol=2e-3)


def test_cosine_engine_launch_count_and_no_allocation(fk):
    """A dot-metric step launches the kernels ``kernels_per_step`` names and
    allocates nothing from the caching allocator after the first step."""
    from flash_kmeans.kmeans_triton_impl import LloydEngine
    rng = _rng("cos-eng")
    B, N, K, D = 2, 8192, 256, 128
    x = _dev(rng.standard_normal((B, N, D), dtype=np.float32), "float16")
    eng = LloydEngine(B, N, K, D, torch.float16, "cuda", metric="dot")
    assert eng.kernels_per_step in (2, 3, 5)  # fused, privatised, sorted
    eng.load(x, x[:, :K])
    for _ in range(3):   # eager first step, then the graphs of both centroid buffers
        eng.step()
        eng.advance()
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    for _ in range(3):
        eng.step()
        eng.advance()
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == before


@pytest.mark.parametrize("dt,B,N,K,D", [
    ("float16", 2, 20000, 1000, 128),    # fused sums in the assignment kernel
    ("bfloat16", 1, 30000, 1000, 64),    # fused, D = 64
    ("float16", 3, 9000, 128, 128),      # fused one-hot sums, narrow tiles
    ("bfloat16", 1, 7000, 50, 100),      # fused one-hot, D = 100
    ("float16", 50, 900, 64, 64),        # fused one-hot, many batches (one flush each)
    ("float16", 1, 3000, 200, 192),      # privatised, split-D
    ("float16", 1, 5000, 2000, 192),     # sorted (D > 128)
    ("float32", 2, 4000, 700, 96),       # sorted, float32
    ("float32", 1, 3000, 40, 64),        # privatised, float32
])
def test_assign_dot_accumulate_every_method(fk, dt, B, N, K, D):
    """fk_assign_dot_accumulate (each accumulation method) gives the labels of
    fk_assign_dot and adds exactly those labels' counts and float32 row sums."""
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    rng = _rng("dot-acc", dt, B, N, K, D)
    x = _dev(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    c = _dev(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    x, c = _ops.ensure_tma(x), _ops.ensure_tma(c)
    lib = nat.load()
    code = nat.dtype_code(x.dtype)
    ws = torch.empty(lib.fk_assign_accumulate_workspace_size(B, N, K, D, code), dtype=torch.uint8,
                     device="cuda")
    ids = torch.empty((B, N), dtype=torch.int32, device="cuda")
    counts = torch.full((B, K), 5, dtype=torch.int32, device="cuda")   # added to, not overwritten
    sums = torch.ones((B, K, D), dtype=torch.float32, device="cuda")
    status = _ops.DeviceStatus.word(x.device)
    nat.check(lib.fk_assign_dot_accumulate(
        nat.ptr(x), nat.ptr(c), nat.ptr(ids), nat.ptr(counts), nat.ptr(sums), code, B, N, K, D,
        nat.strides(x, 3), nat.strides(c, 3), nat.strides(ids, 2), nat.ptr(ws), ws.numel(),
        nat.ptr(status), nat.stream_handle(x.device)), "fk_assign_dot_accumulate")
    _ops.DeviceStatus.raise_if_set(x.device)
    assert torch.equal(ids, _ops.assign_dot(x, c))
    idl = ids.long()
    want_cnt = torch.zeros((B, K), dtype=torch.int64, device="cuda")
    want_cnt.scatter_add_(1, idl, torch.ones_like(idl))
    assert torch.equal(counts.long() - 5, want_cnt)
    want = torch.zeros((B, K, D), dtype=torch.float64, device="cuda")
    want.scatter_add_(1, idl[..., None].expand(-1, -1, D), x.double())
    got = sums.double() - 1.0
    err = (got - want).abs().max().item()
    scale = x.double().abs().amax().item() * max(1, int(want_cnt.max()))
    assert err <= 1e-5 * scale, (err, scale)
