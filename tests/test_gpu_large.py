"""GPU tests of the out-of-core path: FlashKMeans' host-data route, batched
kmeans_largeN, centroid staging order, and the multi-GPU reductions.

The reference checks that FlashKMeans on host data with N above
``chunk_size_data_cpu`` equals a direct ``kmeans_largeN`` run under the same
seed (examples/testapi.py:85-119); the route itself is interface.py:136-150
(train) and :223-235 (predict -> kmeans_largeN_assign).
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from _parity import assert_centroids, assert_labels, clusters_touched
from oracle import kmeans_oracle as ko

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def fk():
    import flash_kmeans
    return flash_kmeans


def _np(t):
    return t.detach().float().cpu().numpy()


def test_flashkmeans_cpu_largeN_route_matches_kmeans_largeN(fk):
    """Port of examples/testapi.py:85-119 at a smaller size: host data with N >
    chunk_size_data_cpu goes through kmeans_largeN (same seed, same run) and
    predict through kmeans_largeN_assign."""
    N, K, D, chunk = 3 * 65536 + 1234, 256, 64, 65536
    g = torch.Generator().manual_seed(5)
    data = torch.randn(N, D, generator=g, dtype=torch.float32)
    km = fk.FlashKMeans(d=D, k=K, niter=6, tol=-1, seed=42, chunk_size_data_cpu=chunk)
    api = km.fit_predict(data)
    assert api.shape == (N,) and api.dtype == torch.int32
    assert km.centroids_b.shape == (1, K, D)
    torch.manual_seed(42)
    torch.cuda.manual_seed_all(42)
    raw, cent = fk.kmeans_largeN(data, n_clusters=K, max_iters=6, tol=-1, BLOCK_N=chunk)
    # same seed -> same initial centroids; float32 atomics order the sums
    # differently run to run, so compare at the parity bar
    agree = (api.cpu() == raw.cpu()).double().mean().item()
    assert agree >= 0.999, agree
    touched = clusters_touched(api.cpu().numpy()[None], raw.cpu().numpy()[None], K)
    assert_centroids(_np(km.centroids_b), _np(cent)[None], "api vs kmeans_largeN", skip=touched)
    # predict routes to kmeans_largeN_assign: the same labels bit for bit
    pred = km.predict(data)
    direct = fk.kmeans_largeN_assign(data, km.centroids_b[0], BLOCK_N=chunk)
    assert pred.shape == (N,)
    assert torch.equal(pred.cpu(), direct.cpu())


def _batched_case(B=3, N=90_000, D=20, K=24, seed=9):
    rng = np.random.default_rng(seed)
    x = ko.gmm_points(rng, B, N, D, K, 5.0)
    c0 = np.stack([x[b][rng.integers(0, N, K)] for b in range(B)])
    return x, c0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("resident", [False, True])
def test_kmeans_largeN_batched_equals_per_batch(fk, dtype, resident):
    """Batched x (B, N, D) runs the B problems independently: one pass from the
    same centroids gives each batch's labels bit for bit and its centroids to
    float rounding: the float32 sums add in another order (other CTA ranges,
    atomics), so a stored float16 centroid may differ by one rounding step
    (2^-10 relative).  D=20 exercises padded rows; float16 the on-device
    conversion of streamed float32 blocks."""
    x, c0 = _batched_case()
    B, N, D = x.shape
    K = c0.shape[1]
    xt = torch.from_numpy(x).pin_memory()
    lab, cent = fk.kmeans_largeN(xt, K, max_iters=1, tol=-1, BLOCK_N=25_000,
                                 init_centroids=torch.from_numpy(c0), device="cuda:0",
                                 dtype=dtype, resident=resident)
    assert lab.shape == (B, N) and cent.shape == (B, K, D) and cent.dtype == dtype
    for b in range(B):
        lb, cb = fk.kmeans_largeN(xt[b], K, max_iters=1, tol=-1, BLOCK_N=25_000,
                                  init_centroids=torch.from_numpy(c0[b]), device="cuda:0",
                                  dtype=dtype, resident=resident)
        assert torch.equal(lab[b], lb)
        assert_centroids(_np(cent[b])[None], _np(cb)[None], f"batch {b}",
                         rtol=1e-5 if dtype == torch.float32 else 2.0 ** -10)
    # against the oracle (one teacher-forced pass)
    dt = "float32" if dtype == torch.float32 else "float16"
    xq = ko.round_to(x, dt)
    cq = ko.round_to(c0, dt)
    o_new, _, o_ids = ko.lloyd_iter(xq, ko.row_sqnorm(xq, dt), cq, dt, exact_order=False)
    assert_labels(xq, cq, lab.cpu().numpy(), o_ids, dt, "batched largeN")
    touched = clusters_touched(lab.cpu().numpy(), o_ids, K)
    assert_centroids(_np(cent), o_new, "batched largeN", skip=touched)
    # assign-only pipeline, batched
    lab2 = fk.kmeans_largeN_assign(xt, cent, BLOCK_N=25_000, device="cuda:0", dtype=dtype)
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign
    xd = xt.cuda().to(dtype)
    assert torch.equal(lab2, euclid_assign(xd, cent, _ops.row_sqnorm(xd)))


def test_flashkmeans_batched_cpu_largeN(fk):
    """Batched host data above chunk_size_data_cpu (the reference asserts it
    unsupported) goes through batched kmeans_largeN and batched predict."""
    x, _ = _batched_case(B=2, N=70_000, D=32, K=16, seed=3)
    data = torch.from_numpy(x)
    km = fk.FlashKMeans(d=32, k=16, niter=4, tol=-1, seed=7, chunk_size_data_cpu=30_000)
    lab = km.fit_predict(data)
    assert lab.shape == (2, 70_000) and km.centroids_b.shape == (2, 16, 32)
    pred = km.predict(data)
    direct = fk.kmeans_largeN_assign(data, km.centroids_b, BLOCK_N=30_000)
    assert torch.equal(pred.cpu(), direct.cpu())
    # a converging run: one more assignment barely moves the training labels
    assert (pred.cpu() == lab.cpu()).double().mean().item() > 0.95


def test_kmeans_largeN_device_centroids_from_side_stream(fk):
    """init_centroids produced by work on the caller's current stream (here a
    side stream) are copied only after that work: every lane's compute stream
    waits on the caller's stream first."""
    rng = np.random.default_rng(21)
    x = ko.gmm_points(rng, 1, 120_000, 16, 12, 6.0)[0]
    c0 = x[rng.integers(0, len(x), 12)]
    xt = torch.from_numpy(x).pin_memory()
    ref_lab, ref_cent = fk.kmeans_largeN(xt, 12, max_iters=2, tol=-1, BLOCK_N=40_000,
                                         init_centroids=torch.from_numpy(c0), device="cuda:0")
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        # a long kernel ahead of the values the run must start from
        junk = torch.randn(4096, 4096, device="cuda")
        for _ in range(8):
            junk = junk @ junk
            junk = junk / junk.norm()
        cd = torch.zeros(12, 16, device="cuda")
        cd.copy_(torch.from_numpy(c0).cuda(non_blocking=True))
        lab, cent = fk.kmeans_largeN(xt, 12, max_iters=2, tol=-1, BLOCK_N=40_000,
                                     init_centroids=cd, device="cuda:0")
    torch.cuda.synchronize()
    assert (lab.cpu() == ref_lab.cpu()).double().mean().item() >= 0.999
    assert_centroids(_np(cent)[None], _np(ref_cent)[None], "side-stream init")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kmeans_largeN_two_devices_equals_one(fk):
    """device=None on 2 GPUs: contiguous partition, NCCL all-reduce; one pass
    from the same centroids gives the 1-GPU labels bit for bit and its
    centroids to float-atomic rounding."""
    rng = np.random.default_rng(31)
    N, K, D = 400_000, 64, 32
    x = rng.standard_normal((N, D), dtype=np.float32)
    c0 = torch.from_numpy(x[rng.integers(0, N, K)])
    xt = torch.from_numpy(x).pin_memory()
    l1, c1 = fk.kmeans_largeN(xt, K, max_iters=1, tol=-1, BLOCK_N=65_536,
                              init_centroids=c0, device="cuda:0")
    l2, c2 = fk.kmeans_largeN(xt, K, max_iters=1, tol=-1, BLOCK_N=65_536, init_centroids=c0,
                              device=None)
    assert not l2.is_cuda and l2.shape == (N,)
    assert torch.equal(l1.cpu(), l2)
    assert_centroids(_np(c2)[None], _np(c1)[None], "2 GPUs vs 1", rtol=1e-5)
    o_new, _, o_ids = ko.lloyd_iter(x[None], ko.row_sqnorm(x[None], "float32"), c0.numpy()[None],
                                    "float32", exact_order=False)
    assert_labels(x[None], c0.numpy()[None], l2.numpy()[None], o_ids, "float32", "2 GPUs")


_PG_WORKER = r"""
import os, sys
sys.path[:0] = [{root!r}, os.path.join({root!r}, "flash-kmeans_b200")]
import numpy as np, torch, torch.distributed as dist
from datetime import timedelta
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
import flash_kmeans as fk
from flash_kmeans.kmeans_large import partition_blocks
rng = np.random.default_rng(31)
N, K, D, BLOCK = 400_000, 64, 32, 65_536
x = rng.standard_normal((N, D), dtype=np.float32)
c0 = torch.from_numpy(x[rng.integers(0, N, K)])
_, ps, pe = partition_blocks(N, BLOCK, world)
shard = torch.from_numpy(x[ps[rank]:pe[rank]]).pin_memory()
lab, cent = fk.kmeans_largeN(shard, K, max_iters=2, tol=-1, BLOCK_N=BLOCK, init_centroids=c0,
                             process_group=dist.group.WORLD, device=f"cuda:{{rank}}")
torch.cuda.synchronize()
labs = [torch.empty(pe[r] - ps[r], dtype=torch.int32, device="cuda") for r in range(world)]
dist.all_gather(labs, lab)
cents = [torch.empty_like(cent) for _ in range(world)]
dist.all_gather(cents, cent)
if rank == 0:
    np.save({out!r} + "_labels.npy", torch.cat(labs).cpu().numpy())
    np.save({out!r} + "_cent.npy", torch.stack(cents).float().cpu().numpy())
dist.barrier()
dist.destroy_process_group()
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kmeans_largeN_process_group_two_ranks(fk, tmp_path):
    """One process per GPU over torch.distributed NCCL: every rank ends with the
    same centroids, equal (to float-atomic rounding) to the single-process run;
    the gathered shard labels equal the single-process labels."""
    out = str(tmp_path / "pg")
    script = tmp_path / "worker.py"
    script.write_text(_PG_WORKER.format(root=ROOT, out=out))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29533", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    lab = np.load(out + "_labels.npy")
    cents = np.load(out + "_cent.npy")
    np.testing.assert_array_equal(cents[0], cents[1])   # replicas identical
    rng = np.random.default_rng(31)
    N, K, D = 400_000, 64, 32
    x = rng.standard_normal((N, D), dtype=np.float32)
    c0 = torch.from_numpy(x[rng.integers(0, N, K)])
    l1, c1 = fk.kmeans_largeN(torch.from_numpy(x).pin_memory(), K, max_iters=2, tol=-1,
                              BLOCK_N=65_536, init_centroids=c0, device="cuda:0")
    assert (lab == l1.cpu().numpy()).mean() >= 0.999
    assert_centroids(cents[0][None], _np(c1)[None], "process group vs single process")
