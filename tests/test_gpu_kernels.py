"""GPU parity of the sm_100a kernels against the CPU oracle and the golden vectors.

Every computation here goes through the C ABI (flash_kmeans._ops -> ctypes ->
libflashkmeans_b200.so); the oracle (numpy) is the checker only.
"""
import zlib

import numpy as np
import pytest
import torch

import cases
from _parity import assert_centroids, assert_labels, label_report
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
    from flash_kmeans import _native
    _native.load()
    return flash_kmeans


# ----------------------------------------------------------------- row norms
@pytest.mark.parametrize("dt", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("D", [1, 17, 128, 2048])
def test_row_sqnorm_matches_oracle(fk, dt, D):
    from flash_kmeans import _ops
    rng = np.random.default_rng(D)
    x = ko.round_to(rng.standard_normal((2, 301, D), dtype=np.float32), dt)
    got = _np(_ops.row_sqnorm(_dev(x, dt)))
    want = ko.row_sqnorm(x, dt)
    # float32 accumulation order differs; the final rounding may differ by one ulp
    rel = np.abs(got - want) / np.maximum(np.abs(want), 1e-6)
    ulp = {"float16": 2 ** -10, "bfloat16": 2 ** -7, "float32": 1e-5}[dt]
    assert rel.max() <= ulp * 1.01
    if dt != "float32":  # 16-bit results are rounded once: nearly always identical
        assert (got != want).mean() < 0.02


@pytest.mark.parametrize("dt", ["float16", "float32"])
def test_row_sqnorm_layouts_agree(fk, dt):
    """The vector kernel addresses rows directly when batches are back to back and
    through (batch, point) otherwise; both give the same bits, over enough rows that
    every warp runs several unrolled iterations and a ragged tail."""
    from flash_kmeans import _ops
    B, N, D = 3, 100003, 64
    big = torch.randn((B, N + 5, D), device="cuda").to(TD[dt])
    strided = big[:, :N]                      # batch stride (N+5)*D: the (batch, point) path
    flat = strided.contiguous()
    a = _ops.row_sqnorm(strided)
    b = _ops.row_sqnorm(flat)
    assert torch.equal(a, b)
    want = ko.row_sqnorm(_np(flat[:, :2000]), dt)
    rel = np.abs(_np(b[:, :2000]) - want) / np.maximum(np.abs(want), 1e-6)
    assert rel.max() <= {"float16": 2 ** -10, "float32": 1e-5}[dt] * 1.01


# ----------------------------------------------------------------- assignment
@pytest.mark.parametrize("spec", cases.ASSIGN_CASES, ids=lambda s: s["name"])
def test_assign_matches_golden_and_oracle(fk, spec):
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
    dt = spec["dtype"]
    ids = euclid_assign_triton(_dev(x, dt), _dev(c, dt), _dev(xsq, xsq_dtype))
    torch.cuda.synchronize()
    got = ids.cpu().numpy()
    golden = np.load(cases.path(spec["name"]))["ids"]
    assert_labels(x, c, got, golden, dt, spec["name"] + " vs reference")
    want = ko.assign(x, c, xsq, dt, xsq_dtype=xsq_dtype)
    assert_labels(x, c, got, want, dt, spec["name"] + " vs oracle")


def test_assign_duplicate_centroids_take_lowest_index(fk):
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    spec = next(s for s in cases.ASSIGN_CASES if s.get("dup"))
    x, c, xsq, xsq_dtype = cases.assign_inputs(spec)
    ids = euclid_assign_triton(_dev(x, "float16"), _dev(c, "float16"), _dev(xsq, "float16"))
    got = ids.cpu().numpy()
    assert got.max() < spec["K"] // 2
    np.testing.assert_array_equal(got, np.load(cases.path(spec["name"]))["ids"])


SHAPES = [  # (B, N, K, D): tails in every dimension, both x-resident and split-D paths
    (1, 1, 1, 16), (1, 5, 3, 8), (2, 127, 7, 64), (1, 129, 255, 128), (1, 300, 256, 32),
    (1, 257, 257, 96), (3, 200, 19, 100), (1, 1000, 513, 17), (1, 640, 70, 192),
    (1, 333, 300, 513), (1, 250, 64, 1000),
]


@pytest.mark.parametrize("dt", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_assign_shapes_vs_oracle(fk, dt, shape):
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    B, N, K, D = shape
    rng = np.random.default_rng(zlib.crc32(repr((dt,) + shape).encode()))  # stable across runs
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    c = ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    xd = _dev(x, dt)
    xsq = _ops.row_sqnorm(xd)
    ids = euclid_assign_triton(xd, _dev(c, dt), xsq).cpu().numpy()
    want = ko.assign(x, c, _np(xsq), dt)
    assert_labels(x, c, ids, want, dt, f"{dt} {shape}")


@pytest.mark.parametrize("dt,xsq_f32", [("float16", False), ("bfloat16", False), ("float16", True)])
def test_assign_narrow_tiles_across_batches(fk, dt, xsq_f32):
    """K <= 128: 128-column tiles with the batch's centroids resident in shared memory.
    256 point tiles over the persistent CTAs, so many CTAs' tile ranges cross batches and
    the centroids are reloaded mid-range."""
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    B, N, K, D = 64, 500, 100, 128
    rng = np.random.default_rng(17 + xsq_f32)
    x = ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt)
    c = ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt)
    xd = _dev(x, dt)
    xsq = (xd.float() ** 2).sum(-1) if xsq_f32 else _ops.row_sqnorm(xd)
    ids = euclid_assign_triton(xd, _dev(c, dt), xsq).cpu().numpy()
    want = ko.assign(x, c, _np(xsq), dt, xsq_dtype="float32" if xsq_f32 else None)
    assert_labels(x, c, ids, want, dt, f"narrow {dt} xsq_f32={xsq_f32}")


def test_assign_strided_inputs(fk):
    """Non-contiguous x (transposed storage) and a sliced batch go through packing."""
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    rng = np.random.default_rng(5)
    x = ko.round_to(rng.standard_normal((2, 64, 500), dtype=np.float32), "float16")
    c = ko.round_to(rng.standard_normal((2, 40, 64), dtype=np.float32), "float16")
    xt = _dev(x, "float16").transpose(1, 2)          # (2, 500, 64), stride_d = 500
    xs = ko.round_to(np.swapaxes(x, 1, 2), "float16")
    xsq = (xt.float() ** 2).sum(-1)
    ids = euclid_assign_triton(xt, _dev(c, "float16"), xsq).cpu().numpy()
    want = ko.assign(xs, c, _np(xsq), "float16", xsq_dtype="float32")
    assert_labels(xs, c, ids, want, "float16", "strided")


@pytest.mark.parametrize("dt,xsq32", [("float16", False), ("bfloat16", False), ("float16", True)])
def test_assign_out_and_csq_arguments(fk, dt, xsq32):
    """out= and c_sq= arguments; with c_sq given and dense centroids the -2c operand
    is staged by the vectorised kernel (the Lloyd engine's steady state), with it
    absent by the per-row kernel that also computes c_sq."""
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    rng = np.random.default_rng(6)
    x = ko.round_to(rng.standard_normal((2, 700, 64), dtype=np.float32), dt)
    c = ko.round_to(rng.standard_normal((2, 90, 64), dtype=np.float32), dt)
    xd, cd = _dev(x, dt), _dev(c, dt)
    xsq = (xd.float() ** 2).sum(-1) if xsq32 else _ops.row_sqnorm(xd)
    out = torch.full((2, 700), -1, dtype=torch.int32, device="cuda")
    csq = (cd.float() ** 2).sum(-1)
    r = euclid_assign_triton(xd, cd, xsq, out=out, c_sq=csq)
    assert r.data_ptr() == out.data_ptr()
    base = euclid_assign_triton(xd, cd, xsq)
    rep = label_report(x, c, out.cpu().numpy(), base.cpu().numpy(), dt)
    assert rep["bad"] == 0
    with pytest.raises(ValueError):
        euclid_assign_triton(xd, cd, xsq, num_warps=4)


def test_assign_deterministic(fk):
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(4, 20000, 128, device="cuda", generator=g).half()
    c = torch.randn(4, 1000, 128, device="cuda", generator=g).half()
    xsq = _ops.row_sqnorm(x)
    a = euclid_assign_triton(x, c, xsq)
    b = euclid_assign_triton(x, c, xsq)
    assert torch.equal(a, b)


# ------------------------------------------------------------------ update
@pytest.mark.parametrize("spec", cases.UPDATE_CASES, ids=lambda s: s["name"])
@pytest.mark.parametrize("idt", [torch.int32, torch.int64])
def test_update_matches_golden(fk, spec, idt):
    from flash_kmeans import triton_centroid_update_sorted_euclid
    x, ids, old = cases.update_inputs(spec)
    dt = spec["dtype"]
    new = triton_centroid_update_sorted_euclid(_dev(x, dt), torch.from_numpy(ids).to("cuda", idt),
                                               _dev(old, dt))
    got = _np(new)
    golden = np.load(cases.path(spec["name"]))["centroids"]
    assert_centroids(got, golden, spec["name"])
    # empty clusters are bit-identical to the old centroids
    cnt = np.stack([np.bincount(ids[b], minlength=spec["K"]) for b in range(spec["B"])])
    np.testing.assert_array_equal(got[cnt == 0], ko.round_to(old, dt)[cnt == 0])


def test_update_accumulate_over_blocks(fk):
    """Accumulating two halves equals the one-shot update (calculate_new=False path)."""
    from flash_kmeans import triton_centroid_update_sorted_euclid as upd
    rng = np.random.default_rng(9)
    B, N, K, D = 1, 5000, 77, 128
    x = _dev(rng.standard_normal((B, N, D), dtype=np.float32), "float32")
    ids = torch.from_numpy(rng.integers(0, K, (B, N)).astype(np.int32)).cuda()
    old = _dev(rng.standard_normal((B, K, D), dtype=np.float32), "float32")
    sums = torch.zeros((B, K, D), device="cuda")
    cnts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
    assert upd(x[:, :2000], ids[:, :2000], old, centroid_sums=sums, centroid_cnts=cnts,
               calculate_new=False) is None
    last = upd(x[:, 2000:], ids[:, 2000:], old, centroid_sums=sums, centroid_cnts=cnts,
               calculate_new=True)
    ref = ko.centroid_update(_np(x), ids.cpu().numpy(), _np(old), "float32")
    assert_centroids(_np(last), ref, "accumulate")
    np.testing.assert_array_equal(cnts.cpu().numpy()[0], np.bincount(ids.cpu().numpy()[0], minlength=K))


def test_update_bad_label_reports_device_status(fk):
    from flash_kmeans import _ops
    from flash_kmeans._ops import DeviceStatus
    x = torch.randn(1, 64, 32, device="cuda")
    ids = torch.zeros(1, 64, dtype=torch.int32, device="cuda")
    ids[0, 3] = 99  # K = 8
    sums = torch.zeros(1, 8, 32, device="cuda")
    cnt = torch.zeros(1, 8, dtype=torch.int32, device="cuda")
    _ops.accumulate(x, ids, sums, cnt)
    with pytest.raises(RuntimeError, match="outside"):
        DeviceStatus.raise_if_set(x.device)
    DeviceStatus.raise_if_set(x.device)  # cleared
    assert int(cnt.sum()) == 63


def _torch_sums(x, ids, K):
    """float32 per-cluster row sums and counts with torch (index_add / bincount)."""
    B, N, D = x.shape
    sums = torch.zeros((B, K, D), device=x.device)
    cnts = torch.zeros((B, K), dtype=torch.int32, device=x.device)
    for b in range(B):
        sums[b].index_add_(0, ids[b].long(), x[b].float())
        cnts[b] = torch.bincount(ids[b].long(), minlength=K).int()
    return sums, cnts


# K x D below / above the shared-memory privatisation limit (51200 floats)
@pytest.mark.parametrize("dt,B,N,K,D,idt", [
    ("float16", 2, 3000, 77, 128, torch.int32), ("float32", 1, 2000, 300, 100, torch.int64),
    ("float16", 2, 3000, 600, 128, torch.int64), ("bfloat16", 1, 2500, 700, 96, torch.int32)])
def test_accumulate_privatised_and_sorted_paths(fk, dt, B, N, K, D, idt):
    """fk_centroid_accumulate against torch index_add: the privatised shared-memory kernel
    (small K x D) and the counting-sort segmented sum (large K x D)."""
    from flash_kmeans import _ops
    g = torch.Generator(device="cuda").manual_seed(K + D)
    x = torch.randn((B, N, D), device="cuda", generator=g).to(getattr(torch, dt))
    ids = torch.randint(0, K, (B, N), device="cuda", generator=g).to(idt)
    ids[:, :N // 3] = K // 2  # a crowded cluster
    sums = torch.zeros((B, K, D), device="cuda")
    cnts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
    _ops.accumulate(x, ids, sums, cnts)
    ref_s, ref_c = _torch_sums(x, ids, K)
    assert torch.equal(cnts, ref_c)
    torch.testing.assert_close(sums, ref_s, rtol=1e-5, atol=1e-3)


# -------------------------------------------------- fused assign + accumulate
@pytest.mark.parametrize("dt,B,N,K,D", [
    ("float16", 3, 5000, 1000, 128), ("float16", 2, 700, 70, 64), ("bfloat16", 2, 900, 33, 100),
    ("float16", 1, 1000, 50, 17), ("float16", 1, 640, 40, 192), ("float32", 2, 800, 60, 48),
    ("bfloat16", 2, 900, 600, 100), ("float16", 1, 3000, 3100, 17), ("float16", 1, 640, 300, 192),
    ("float32", 1, 1200, 1100, 48),
    # CTA ranges that cross many batch boundaries, one long batch with K = 128, K = 1,
    # and float32 x_sq (mode 1)
    ("float16", 64, 1000, 100, 128), ("bfloat16", 40, 700, 17, 64),
    ("float16", 1, 300000, 128, 128), ("float16", 3, 129, 1, 8), ("float16-xsq32", 5, 3000, 60, 128),
    # one-hot form: every tile its own batch (each CTA flushes after every tile, both
    # epilogue warpgroups and both sums barriers), and three tiles per batch
    ("float16", 300, 100, 64, 128), ("bfloat16", 37, 260, 128, 96)])
def test_assign_accumulate_matches_separate_path(fk, dt, B, N, K, D):
    """fk_assign_accumulate (fused for 16-bit D<=128: one-hot tensor-core sums for K<=128,
    sum warps for larger K; privatised or sorted otherwise) equals fk_assign + torch
    index_add: labels bit-identical, counts exact, sums to fp32 order."""
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    lib = nat.load()
    xsq32 = dt.endswith("-xsq32")
    dt = dt.replace("-xsq32", "")
    rng = np.random.default_rng(B * 7 + D + K)
    x = _ops.ensure_tma(_dev(ko.round_to(rng.standard_normal((B, N, D), dtype=np.float32), dt), dt))
    c = _ops.ensure_tma(_dev(ko.round_to(rng.standard_normal((B, K, D), dtype=np.float32), dt), dt))
    xsq = (x.float() ** 2).sum(-1) if xsq32 else _ops.row_sqnorm(x)
    ref = _ops.assign(x, c, xsq)
    ref_s, ref_c = _torch_sums(x, ref, K)
    out = torch.full((B, N), -1, dtype=torch.int32, device="cuda")
    sums = torch.zeros((B, K, D), device="cuda")
    cnts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
    ws = torch.empty(lib.fk_assign_accumulate_workspace_size(B, N, K, D, nat.dtype_code(x.dtype)),
                     dtype=torch.uint8, device="cuda")
    status = torch.zeros(4, dtype=torch.int32, device="cuda")
    nat.check(lib.fk_assign_accumulate(
        nat.ptr(x), nat.ptr(c), nat.ptr(xsq), None, nat.ptr(out), nat.ptr(cnts), nat.ptr(sums),
        nat.dtype_code(x.dtype), nat.dtype_code(xsq.dtype), 0, B, N, K, D, nat.strides(x, 3),
        nat.strides(c, 3), nat.strides(xsq, 2), None, nat.strides(out, 2), nat.ptr(ws), ws.numel(),
        nat.ptr(status), nat.stream_handle(x.device)), "fk_assign_accumulate")
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    assert torch.equal(out, ref)
    assert torch.equal(cnts, ref_c)
    torch.testing.assert_close(sums, ref_s, rtol=1e-5, atol=1e-3)


# ------------------------------------------- float32 x split once (FK_F32_XSPLIT)
@pytest.mark.parametrize("metric", ["euclid", "dot"])
@pytest.mark.parametrize("B,N,K,D,layout", [
    (2, 1000, 300, 128, "dense"),      # 128-byte chunk rows, two stages
    (1, 700, 260, 640, "dense"),       # 64-byte chunk rows, four stages (D >= 512)
    (3, 333, 70, 37, "padded"),        # rows padded to 40 floats: the strided split
    (2, 500, 40, 48, "strided"),       # a non-contiguous view of x (every other column)
    (3, 700, 90, 128, "rowview")])     # rows 0..N-1 of a longer buffer: the row-wise split
def test_xsplit_matches_tile_split(fk, metric, B, N, K, D, layout):
    """fk_assign_accumulate / fk_assign_dot_accumulate with x split once per fit
    into the workspace (FK_F32_XSPLIT) give the same labels, counts and sums,
    bit for bit, as with each x tile split in shared memory (FK_F32): both use
    the same tf32 hi/lo halves and the same MMA order."""
    from flash_kmeans import _native as nat
    from flash_kmeans import _ops
    lib = nat.load()
    rng = np.random.default_rng(B * 31 + D + K)
    xa = rng.standard_normal((B, N, D), dtype=np.float32)
    if layout == "strided":
        big = torch.from_numpy(rng.standard_normal((B, N, 2 * D), dtype=np.float32)).cuda()
        big[..., ::2] = torch.from_numpy(xa).cuda()
        x = big[..., ::2]
        xt = _ops.ensure_tma(x.contiguous())
    elif layout == "rowview":
        big = torch.from_numpy(rng.standard_normal((B, N + 13, D), dtype=np.float32)).cuda()
        big[:, :N] = torch.from_numpy(xa).cuda()
        x = big[:, :N]
        xt = _ops.ensure_tma(x.contiguous())
    else:
        xt = _ops.ensure_tma(torch.from_numpy(xa).cuda())
        x = xt
    c = _ops.ensure_tma(torch.from_numpy(rng.standard_normal((B, K, D), dtype=np.float32)).cuda())
    xsq = _ops.row_sqnorm(xt) if metric == "euclid" else None
    status = torch.zeros(4, dtype=torch.int32, device="cuda")

    def run(code):
        out = torch.full((B, N), -1, dtype=torch.int32, device="cuda")
        sums = torch.zeros((B, K, D), device="cuda")
        cnts = torch.zeros((B, K), dtype=torch.int32, device="cuda")
        ws = torch.empty(lib.fk_assign_accumulate_workspace_size(B, N, K, D, code),
                         dtype=torch.uint8, device="cuda")
        s = nat.stream_handle(xt.device)
        if code == nat.FK_F32_XSPLIT:
            # the split reads x through its own strides (strided case: the view)
            nat.check(lib.fk_assign_accumulate_split_x(nat.ptr(x), B, N, K, D, nat.strides(x, 3),
                                                       nat.ptr(ws), ws.numel(), s),
                      "fk_assign_accumulate_split_x")
        if metric == "euclid":
            nat.check(lib.fk_assign_accumulate(
                nat.ptr(xt), nat.ptr(c), nat.ptr(xsq), None, nat.ptr(out), nat.ptr(cnts),
                nat.ptr(sums), code, nat.dtype_code(xsq.dtype), 0, B, N, K, D,
                nat.strides(xt, 3), nat.strides(c, 3), nat.strides(xsq, 2), None,
                nat.strides(out, 2), nat.ptr(ws), ws.numel(), nat.ptr(status), s),
                "fk_assign_accumulate")
        else:
            nat.check(lib.fk_assign_dot_accumulate(
                nat.ptr(xt), nat.ptr(c), nat.ptr(out), nat.ptr(cnts), nat.ptr(sums), code,
                B, N, K, D, nat.strides(xt, 3), nat.strides(c, 3), nat.strides(out, 2),
                nat.ptr(ws), ws.numel(), nat.ptr(status), s), "fk_assign_dot_accumulate")
        torch.cuda.synchronize()
        assert int(status[0]) == 0
        return out, cnts, sums

    o1, c1, s1 = run(nat.FK_F32)
    o2, c2, s2 = run(nat.FK_F32_XSPLIT)
    assert int((o1 < 0).sum()) == 0
    assert torch.equal(o1, o2)
    assert torch.equal(c1, c2)
    ref_s, _ = _torch_sums(xt, o1, K)
    torch.testing.assert_close(s2, ref_s, rtol=1e-5, atol=1e-3)
