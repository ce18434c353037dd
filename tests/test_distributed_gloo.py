"""Multi-process decomposition of the out-of-core path, on CPU with gloo.

Two ranks each own a contiguous shard (the reference's block partition), compute
partial float32 sums and int32 counts for their shard, and exchange them with
the package's own reduce_partials / broadcast_centroids -- the only collective
of the iteration.  The per-shard arithmetic comes from the CPU oracle (the CUDA
kernels need a GPU); the result must equal the single-process oracle update.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, port, N, K, D, BLOCK_N, iters, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "flash-kmeans_b200")]
    from datetime import timedelta
    from flash_kmeans import kmeans_large
    from oracle import kmeans_oracle as ko

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        rng = np.random.default_rng(123)
        x = ko.gmm_points(rng, 1, N, D, 8, 3.0)[0]
        bpg, ps, pe = kmeans_large.partition_blocks(N, BLOCK_N, WORLD)
        shard = x[ps[rank]:pe[rank]]
        # rank 0's sample wins the broadcast
        c0 = torch.from_numpy(shard[np.random.default_rng(rank).integers(0, len(shard), K)].copy())
        c0 = kmeans_large.broadcast_centroids(c0, dist.group.WORLD)
        c = c0.numpy()
        for _ in range(iters):
            ids = ko.assign(shard[None], c[None], ko.row_sqnorm(shard[None], "float32"), "float32")
            s, n = ko.centroid_sums(shard[None], ids, K)
            st = torch.from_numpy(s[0].copy())
            ct = torch.from_numpy(n[0].astype(np.int32))
            kmeans_large.reduce_partials(st, ct, dist.group.WORLD)
            c = ko.finalize(st.numpy()[None], ct.numpy()[None].astype(np.float32), c[None],
                            "float32")[0]
        q.put((rank, c0.numpy(), c))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_matches_single_process():
    N, K, D, BLOCK_N, iters = 4000, 8, 16, 700, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, N, K, D, BLOCK_N, iters, q))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(WORLD):
        r, c0, c = q.get(timeout=120)
        res[r] = (c0, c)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # both ranks started from rank 0's centroids and ended identical
    np.testing.assert_array_equal(res[0][0], res[1][0])
    np.testing.assert_array_equal(res[0][1], res[1][1])
    # and equal to the single-process computation
    import sys
    from oracle import kmeans_oracle as ko
    rng = np.random.default_rng(123)
    x = ko.gmm_points(rng, 1, N, D, 8, 3.0)
    c = res[0][0][None]
    for _ in range(iters):
        c, _, _ = ko.lloyd_iter(x, ko.row_sqnorm(x, "float32"), c, "float32")
    np.testing.assert_allclose(res[0][1], c[0], rtol=1e-5, atol=1e-5)
