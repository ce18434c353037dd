"""Out-of-core / multi-GPU Lloyd k-means, drop-in for flash_kmeans.kmeans_large.

Contract of the reference (kmeans_large.py:33-421): x (N, D) lives in host
memory (ideally pinned) and is streamed to the GPUs in blocks of ``BLOCK_N``
points; the blocks are partitioned contiguously over the devices
(kmeans_large.py:69-80); every iteration each device assigns its blocks and
accumulates per-cluster float32 sums and int32 counts, the partial sums are
reduced across devices, and the centroids are finalized.  On a tolerance
break the NEW centroids are returned (kmeans_large.py:251-258).  With one
device the labels and centroids stay on that device; with several they are
returned on the host (labels in pinned memory).

B200 design:
* per device a copy stream and a compute stream over two block buffers; the
  copy of block i+1 (and of the next iteration's first blocks) overlaps the
  assignment of block i, ordered by events only (no host waits);
* when a device's slice of x fits in half of its free HBM (a B200 holds
  180 GB) and several passes are coming, the blocks are copied once into a
  resident buffer during the first pass and later passes read them from
  HBM: iterations stop being bound by the host link (all GPUs of a node
  share the host's PCIe bandwidth);
* x_sq per block is computed once and kept on the device;
* each block goes through fk_assign_accumulate: labels, counts and per-cluster
  row sums in one call (one kernel for 16-bit data with D <= 128); float32
  blocks of rows up to XSPLIT_MAX_D floats are first split into their tf32
  halves (fk_assign_accumulate_split_x, one HBM pass) so the 3xTF32
  assignment loads them instead of splitting every tile in shared memory;
* reduction: every device ends with identical sums/counts after an NCCL
  all-reduce (single-process communicator over the devices, or the process
  group when one process drives one GPU), then finalizes its own replica, so
  no broadcast is needed;
* batched input (B, N, D) (an extension: the reference asserts it away,
  interface.py:138): the B independent problems share the block pipeline,
  each block carrying the same point range of every batch.
"""
from __future__ import annotations

import time
import warnings
from typing import Optional

import torch

from . import _native as nat
from . import _ops


def _resolve_devices(device):
    """device=None -> all visible GPUs; otherwise exactly that one device
    (kmeans_large.py:18-30)."""
    if device is None:
        G = torch.cuda.device_count()
        if G == 0:
            raise RuntimeError("No CUDA devices available")
        return [torch.device(f"cuda:{i}") for i in range(G)]
    return [torch.device(device)]


def partition_blocks(N: int, BLOCK_N: int, G: int):
    """Contiguous block partition of N points over G devices
    (kmeans_large.py:69-80).  Returns (blocks_per_gpu, point_start, point_end)."""
    num_blocks = (N + BLOCK_N - 1) // BLOCK_N
    blocks_per_gpu = [(num_blocks // G) + (1 if g < (num_blocks % G) else 0) for g in range(G)]
    block_start = [0] * G
    for g in range(1, G):
        block_start[g] = block_start[g - 1] + blocks_per_gpu[g - 1]
    point_start = [block_start[g] * BLOCK_N for g in range(G)]
    point_end = [min(point_start[g] + blocks_per_gpu[g] * BLOCK_N, N) for g in range(G)]
    return blocks_per_gpu, point_start, point_end


def _fits_resident(dev, rows: int, D: int, dtype: torch.dtype) -> bool:
    """Whether `rows` rows of x (padded like the block buffers; all batches'
    rows counted) take at most half of the device's free memory."""
    esize = torch.empty((), dtype=dtype).element_size()
    row_bytes = -(-D * esize // 16) * 16
    free, _ = torch.cuda.mem_get_info(dev)
    return rows * row_bytes <= free // 2


class _DeviceLane:
    """Per-device streaming pipeline for one contiguous slice of x.

    ``x_host`` is (B, N, D); every block holds the same point range of all B
    batches.  ``resident``: copy every block once into one device buffer and
    reuse it on later passes (no per-pass host transfers)."""

    def __init__(self, dev, x_host, p0, p1, BLOCK_N, K, D, dtype, resident: bool = False):
        self.dev = dev
        self.x_host = x_host
        self.B = B = x_host.shape[0]
        self.p0, self.p1 = p0, p1
        self.BLOCK_N = BLOCK_N
        self.blocks = [(n0, min(n0 + BLOCK_N, p1)) for n0 in range(p0, p1, BLOCK_N)]
        self.K, self.D, self.dtype = K, D, dtype
        self.resident = resident
        with torch.cuda.device(dev):
            self.copy_stream = torch.cuda.Stream(device=dev)
            self.compute_stream = torch.cuda.Stream(device=dev)
            nb = min(BLOCK_N, p1 - p0)
            if resident:
                # one buffer for the whole slice; block i is rows n0-p0 .. n1-p0
                self.xres = _ops.empty_rows(B, p1 - p0, D, dtype, dev)
                self.res_loaded = [torch.cuda.Event() for _ in self.blocks]
                self.res_issued = False
            self.xbuf = [_ops.empty_rows(B, nb, D, dtype, dev) for _ in range(1 if resident else 2)]
            self.stage = None
            if x_host.dtype != dtype or not (x_host[0].is_contiguous() and
                                             self.xbuf[0].is_contiguous()):
                # host rows land here, then one device kernel converts / pads them
                self.stage = [torch.empty((B, nb, D), dtype=x_host.dtype, device=dev)
                              for _ in range(2)]
            self.loaded = [torch.cuda.Event() for _ in range(2)]
            self.free = [torch.cuda.Event() for _ in range(2)]
            self.labels = torch.empty((B, p1 - p0), dtype=torch.int32, device=dev)
            self.xsq = [None] * len(self.blocks)
            self.c_cur = _ops.empty_rows(B, K, D, dtype, dev)
            self.c_nxt = _ops.empty_rows(B, K, D, dtype, dev)
            self.csq = torch.empty((B, K), dtype=torch.float32, device=dev)
            self.sums = torch.empty((B, K, D), dtype=torch.float32, device=dev)
            self.cnt = torch.empty((B, K), dtype=torch.int32, device=dev)
            self.stat = torch.zeros(4, dtype=torch.int32, device=dev)
            self.stat_host = torch.empty(4, dtype=torch.int32, pin_memory=True)
            self.csq_valid = False
            lib = nat.load()
            # float32 blocks with rows of at most XSPLIT_MAX_D: x's tf32 halves
            # are split once per block and pass into the workspace
            # (FK_F32_XSPLIT) instead of in every assignment tile, when the
            # halves take at most a quarter of the free memory
            free = torch.cuda.mem_get_info(dev)[0] if dtype == torch.float32 else 0
            self.xcode, ws_bytes = nat.accumulate_x_code(lib, dtype, B, nb, K, D, free, 0.25)
            self.ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        # Copies form one sequence over passes: element s streams block s % nb
        # into buffer slot s % 2, so consecutive copies always alternate slots.
        self._issued = 0
        self._ahead = []   # (block, slot) copied or in flight, not yet computed
        self._pass = 0

    # ---------------------------------------------------------------- loads
    def _copy_block(self, dst, stage, n0: int, n1: int) -> None:
        """H2D copy of rows n0:n1 of every batch into dst (B, n1-n0, D) on
        the current stream: one copy per batch (each a contiguous host range),
        through `stage` when the rows need a dtype conversion or padding."""
        nb = n1 - n0
        for b in range(self.B):
            src = self.x_host[b, n0:n1]
            if stage is None:
                dst[b].copy_(src, non_blocking=True)
            else:
                stage[b, :nb].copy_(src, non_blocking=True)
        if stage is not None:
            dst.copy_(stage[:, :nb])

    def _issue_load(self, blk: int, slot: int) -> None:
        n0, n1 = self.blocks[blk]
        nb = n1 - n0
        cs = self.copy_stream
        with torch.cuda.device(self.dev), torch.cuda.stream(cs):
            cs.wait_event(self.free[slot])
            self._copy_block(self.xbuf[slot][:, :nb],
                             None if self.stage is None else self.stage[slot], n0, n1)
            self.loaded[slot].record(cs)

    def _prefetch_one(self) -> None:
        nblk = len(self.blocks)
        blk, slot = self._issued % nblk, self._issued % 2
        self._issue_load(blk, slot)
        self._ahead.append((blk, slot))
        self._issued += 1

    def _refill(self, wrap: bool) -> None:
        """Keep two copies in flight; cross into the next pass only if `wrap`."""
        nblk = len(self.blocks)
        limit = (self._pass + (2 if wrap else 1)) * nblk
        while len(self._ahead) < 2 and self._issued < limit:
            self._prefetch_one()

    def _load_resident(self) -> None:
        """First pass of a resident lane: queue every block's copy into its
        own rows of the resident buffer (no slot reuse, so no waits)."""
        if self.res_issued:
            return
        self.res_issued = True
        cs = self.copy_stream
        with torch.cuda.device(self.dev), torch.cuda.stream(cs):
            for i, (n0, n1) in enumerate(self.blocks):
                self._copy_block(self.xres[:, n0 - self.p0:n1 - self.p0],
                                 None if self.stage is None else self.stage[0], n0, n1)
                self.res_loaded[i].record(cs)

    # -------------------------------------------------------------- compute
    def run_pass(self, assign_only: bool = False, wrap: bool = False) -> None:
        """Assign (and accumulate) every block of this lane once.  With `wrap`
        the first copies of the next pass are queued as buffers free up."""
        lib = nat.load()
        ks = self.compute_stream
        B, K, D = self.B, self.K, self.D
        with torch.cuda.device(self.dev), torch.cuda.stream(ks):
            if not assign_only:
                self.sums.zero_()
                self.cnt.zero_()
            s = nat.stream_handle(self.dev)
            status = nat.ptr(self.stat[1:2])
            if self.resident:
                self._load_resident()
            else:
                self._refill(wrap)
            for i, (n0, n1) in enumerate(self.blocks):
                nb = n1 - n0
                if self.resident:
                    slot = None
                    if self._pass == 0:
                        ks.wait_event(self.res_loaded[i])
                    xb = self.xres[:, n0 - self.p0:n1 - self.p0]
                else:
                    blk, slot = self._ahead.pop(0)
                    assert blk == i, (blk, i)
                    ks.wait_event(self.loaded[slot])
                    xb = self.xbuf[slot][:, :nb]
                if self.xsq[i] is None:
                    self.xsq[i] = _ops.row_sqnorm(xb)
                xsq = self.xsq[i]
                lo, hi = n0 - self.p0, n1 - self.p0
                out = self.labels[:, lo:hi]
                c_sq = self.csq if self.csq_valid else None
                args = (nat.ptr(xb), nat.ptr(self.c_cur), nat.ptr(xsq), nat.ptr(c_sq), nat.ptr(out))
                tail = (nat.dtype_code(xsq.dtype), nat.FK_F32, B, nb, K, D, nat.strides(xb, 3),
                        nat.strides(self.c_cur, 3), nat.strides(xsq, 2), nat.strides(self.csq, 2),
                        nat.strides(out, 2), nat.ptr(self.ws), self.ws.numel(), status, s)
                if assign_only:
                    nat.check(lib.fk_assign(*args, None, nat.dtype_code(xb.dtype), *tail),
                              "fk_assign")
                else:  # labels, counts and row sums of this block in one pass
                    if self.xcode == nat.FK_F32_XSPLIT:
                        nat.check(lib.fk_assign_accumulate_split_x(
                            nat.ptr(xb), B, nb, K, D, nat.strides(xb, 3), nat.ptr(self.ws),
                            self.ws.numel(), s), "fk_assign_accumulate_split_x")
                    nat.check(lib.fk_assign_accumulate(*args, nat.ptr(self.cnt), nat.ptr(self.sums),
                                                       self.xcode, *tail),
                              "fk_assign_accumulate")
                if not self.resident:
                    self.free[slot].record(ks)
                    self._refill(wrap)
            self._pass += 1

    def finalize(self) -> None:
        lib = nat.load()
        with torch.cuda.device(self.dev), torch.cuda.stream(self.compute_stream):
            nat.check(lib.fk_centroid_finalize(
                nat.ptr(self.sums), nat.ptr(self.cnt), nat.ptr(self.c_cur), nat.ptr(self.c_nxt),
                nat.dtype_code(self.dtype), self.B, self.K, self.D, nat.strides(self.c_cur, 3),
                nat.strides(self.c_nxt, 3), nat.ptr(self.csq), nat.ptr(self.stat[0:1]), 0,
                nat.stream_handle(self.dev)), "fk_centroid_finalize")
            self.csq_valid = True

    def advance(self) -> None:
        self.c_cur, self.c_nxt = self.c_nxt, self.c_cur

    def read_stat(self):
        """(shift, device status) after the work queued on the compute stream."""
        host = self.stat_host
        with torch.cuda.device(self.dev), torch.cuda.stream(self.compute_stream):
            host.copy_(self.stat, non_blocking=True)
        self.compute_stream.synchronize()
        return host[0:1].view(torch.float32).item(), int(host[1].item())

    def set_centroids(self, c0: torch.Tensor) -> None:
        """Copy c0 (B, K, D), host or any device, into c_cur on the compute
        stream, after whatever the caller's current streams have queued that
        produces c0 (an init broadcast, a caller's kernel)."""
        ks = self.compute_stream
        with torch.cuda.device(self.dev):
            ks.wait_stream(torch.cuda.current_stream(self.dev))
            if c0.is_cuda and c0.device != self.dev:
                ks.wait_stream(torch.cuda.current_stream(c0.device))
            with torch.cuda.stream(ks):
                self.c_cur.copy_(c0.to(self.dev, dtype=self.dtype, non_blocking=True))
                self.stat.zero_()


def reduce_partials(sums: torch.Tensor, counts: torch.Tensor, process_group) -> None:
    """In-place all-reduce (sum) of one process's partial sums and counts.

    This is the iteration's only exchange: K*D float32 sums plus K int32
    counts.  Works with any torch.distributed backend (NCCL on GPUs, gloo for
    host tensors)."""
    import torch.distributed as dist
    dist.all_reduce(sums, group=process_group)
    dist.all_reduce(counts, group=process_group)


def broadcast_centroids(c0: torch.Tensor, process_group) -> torch.Tensor:
    """Make every process start from group rank 0's initial centroids."""
    import torch.distributed as dist
    src = dist.get_global_rank(process_group, 0) if process_group is not None else 0
    dist.broadcast(c0, src=src, group=process_group)
    return c0


def _allreduce(lanes, process_group=None) -> None:
    """Sum sums/counts over all lanes so every lane holds the total."""
    if process_group is not None:
        ln = lanes[0]
        with torch.cuda.device(ln.dev), torch.cuda.stream(ln.compute_stream):
            reduce_partials(ln.sums, ln.cnt, process_group)
        return
    if len(lanes) == 1:
        return
    import torch.cuda.nccl as nccl
    streams = [ln.compute_stream for ln in lanes]
    nccl.all_reduce([ln.sums for ln in lanes], streams=streams)
    nccl.all_reduce([ln.cnt for ln in lanes], streams=streams)


def _check_status(code: int) -> None:
    if code:
        raise RuntimeError(f"flash_kmeans device error {code}: {nat.device_status_message(code)}")


def _as_host_batched(x: torch.Tensor):
    """(N, D) -> (1, N, D) view, batched=False; (B, N, D) -> itself, batched=True."""
    if x.dim() == 2:
        return x.unsqueeze(0), False
    if x.dim() == 3:
        return x, True
    raise ValueError("x must be (N, D) or (B, N, D)")


def _gather_labels(lanes, B: int, N: int) -> torch.Tensor:
    """Labels of all lanes into one pinned host tensor (B, N)."""
    labels = torch.empty((B, N), dtype=torch.int32, pin_memory=True)
    for ln in lanes:
        labels[:, ln.p0:ln.p1].copy_(ln.labels)
    return labels


def kmeans_largeN(
    x: torch.Tensor,
    n_clusters: int,
    max_iters: int = 100,
    tol: float = 0.0,
    verbose: bool = False,
    BLOCK_N=1048576,
    init_centroids: Optional[torch.Tensor] = None,
    device: Optional[torch.device] = None,
    dtype: Optional[torch.dtype] = None,
    *,
    process_group=None,
    resident: Optional[bool] = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Lloyd k-means for x (N, D) in host memory, streamed in blocks of BLOCK_N.

    ``device=None`` uses every visible GPU (one host thread drives them);
    a device pins the run to that GPU.  ``process_group`` (extension): x is
    this process's contiguous shard, the process drives one GPU (``device``
    or the current one) and partial sums are all-reduced over the group;
    labels of the shard are returned on the device.  ``resident``
    (extension): None keeps a device's slice of x in HBM after the first pass
    when it takes at most half of the free device memory and ``max_iters`` >
    1; False streams every pass like the reference; True keeps it resident
    regardless (the allocation must succeed).  Batched x (B, N, D)
    (extension; the reference supports (N, D) only) clusters the B problems
    independently with the same pipeline; ``init_centroids`` is then
    (B, K, D).

    Returns (cluster_ids int32 (N,), centroids (K, D)), or (B, N) and
    (B, K, D) for batched x.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("kmeans_largeN needs CUDA (this build has no CPU fallback)")
    if max_iters < 1:
        raise ValueError("max_iters must be >= 1")
    distributed = process_group is not None
    if distributed:
        devices = [torch.device(device) if device is not None
                   else torch.device("cuda", torch.cuda.current_device())]
    else:
        devices = _resolve_devices(device)
    G = len(devices)
    dtype = dtype or x.dtype

    if not x.is_pinned() and G > 1:
        warnings.warn(
            "x is not in pinned memory. H2D transfers will not overlap with compute. "
            "Use x = x.pin_memory() for best multi-GPU performance.",
            stacklevel=2,
        )

    xb, batched = _as_host_batched(x)
    B, N, D = xb.shape
    K = int(n_clusters)
    blocks_per_gpu, point_start, point_end = partition_blocks(N, BLOCK_N, G)
    active = [g for g in range(G) if blocks_per_gpu[g] > 0]

    def keep(g):
        if resident is not None:
            return bool(resident)
        return max_iters > 1 and _fits_resident(devices[g], B * (point_end[g] - point_start[g]),
                                                D, dtype)

    lanes = [_DeviceLane(devices[g], xb, point_start[g], point_end[g], BLOCK_N, K, D, dtype,
                         resident=keep(g))
             for g in active]
    primary = lanes[0]

    # ---- initial centroids (replicated)
    if init_centroids is not None:
        c0 = init_centroids.reshape(B, K, D)
    else:
        # random points, sampled on the host like the reference (kmeans_large.py:106-108)
        if batched:
            idx = torch.randint(0, N, (B, K), device="cpu")
            c0 = torch.gather(xb, 1, idx[..., None].expand(-1, -1, D))
        else:
            c0 = x[torch.randint(0, N, (K,), device="cpu", dtype=torch.int32)].unsqueeze(0)
        if distributed:
            # x is this process's shard: every rank sampled, rank 0's sample wins
            c0 = broadcast_centroids(c0.to(primary.dev, dtype=dtype).contiguous(), process_group)
    for ln in lanes:
        ln.set_centroids(c0)

    need_sync = tol > 0 or verbose
    tol_r = float(torch.tensor(float(tol), dtype=dtype))
    for it in range(max_iters):
        t0 = time.time()
        # with wrap, the next pass's first copies are queued during this pass
        # and overlap the reduction below
        for ln in lanes:
            ln.run_pass(wrap=it + 1 < max_iters)
        _allreduce(lanes, process_group)
        for ln in lanes:
            ln.finalize()
        if need_sync:
            shift, code = primary.read_stat()
            _check_status(code)
            if verbose:
                print(f"Iter {it}, center shift: {shift:.6f}, time: {time.time() - t0:.2f}s")
            if shift < tol_r:
                for ln in lanes:
                    ln.advance()
                break
        for ln in lanes:
            ln.advance()

    # drain any prefetched copies before buffers can be reused or freed
    for ln in lanes:
        with torch.cuda.device(ln.dev):
            ln.copy_stream.synchronize()
            ln.compute_stream.synchronize()
        _, code = ln.read_stat()
        _check_status(code)

    centroids = primary.c_cur
    centroids = centroids if centroids.is_contiguous() else centroids.contiguous()
    if G == 1 or distributed:
        labels = primary.labels
    else:
        labels = _gather_labels(lanes, B, N)
        centroids = centroids.cpu()
    if not batched:
        return labels[0], centroids[0]
    return labels, centroids


def kmeans_largeN_assign(
    x: torch.Tensor,
    centroids: torch.Tensor,
    BLOCK_N=1048576,
    device: Optional[torch.device] = None,
    dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """Labels for x (N, D) in host memory against centroids (K, D)
    (kmeans_large.py:288-421).  One device -> labels on it; several -> pinned
    host.  Batched x (B, N, D) with centroids (B, K, D) gives (B, N)."""
    if not torch.cuda.is_available():
        raise RuntimeError("kmeans_largeN_assign needs CUDA (this build has no CPU fallback)")
    devices = _resolve_devices(device)
    G = len(devices)
    dtype = dtype or x.dtype
    xb, batched = _as_host_batched(x)
    B, N, D = xb.shape
    assert centroids.shape[-1] == D, "centroids and x must have the same feature dimension"
    K = centroids.shape[-2]
    blocks_per_gpu, point_start, point_end = partition_blocks(N, BLOCK_N, G)
    active = [g for g in range(G) if blocks_per_gpu[g] > 0]
    lanes = [_DeviceLane(devices[g], xb, point_start[g], point_end[g], BLOCK_N, K, D, dtype)
             for g in active]
    for ln in lanes:
        ln.set_centroids(centroids.reshape(B, K, D))
    for ln in lanes:
        ln.run_pass(assign_only=True)
    for ln in lanes:
        with torch.cuda.device(ln.dev):
            ln.compute_stream.synchronize()
        _, code = ln.read_stat()
        _check_status(code)
    labels = lanes[0].labels if G == 1 else _gather_labels(lanes, B, N)
    return labels if batched else labels[0]
