"""Batched Lloyd k-means driver, drop-in for flash_kmeans.kmeans_triton_impl.

``batch_kmeans_Euclid`` keeps the reference's contract
(kmeans_triton_impl.py:55-115): random-point init with replacement from the
CUDA RNG when no centroids are given, x_sq precomputed once in x's dtype, one
assignment + update + shift per iteration, ``break`` when the shift drops
below ``tol`` (returning the centroids that produced the last labels), and the
result ``(cluster_ids int32 (B,N), centroids (B,K,D) x.dtype, n_iters)``.

Per iteration the B200 build launches fk_assign_accumulate (the centroid
operand and c_sq staged by one small kernel, then labels with the points' rows
and counts added to the per-cluster sums in the same pass over x whenever x is
16-bit with D <= 128) and fk_centroid_finalize (means, next ||c||^2, shift),
whose two stream-ordered memsets zero the accumulators for the next
iteration.  The host reads the 8-byte (shift, status) record only when
``tol > 0`` or ``verbose`` needs it, and then only after the next iteration
is queued (``LloydEngine.run``); with ``tol <= 0`` the shift can never be
below tol, so iterations are queued back to back with no host
synchronisation.
"""
from __future__ import annotations

import torch

from . import _native as nat
from . import _ops


def _round_tol(tol: float, dtype: torch.dtype) -> float:
    # `center_shift < tol` on a 0-dim tensor of x.dtype compares in that dtype
    return float(torch.tensor(float(tol), dtype=dtype))


# Runs of at least this many iterations replay their steps from CUDA graphs:
# capture costs about as much host time as 50-75 eager steps save.
_GRAPH_MIN_ITERS = 64


class LloydEngine:
    """Buffers and launches for batched Lloyd iterations on one device.

    Reusable across fits of the same shape: ``load(x, centroids)`` then
    ``step()`` per iteration and ``advance()`` to adopt its centroids.
    Iteration k reads centroid buffer k % 3, writes buffer (k+1) % 3 and label
    buffer k % 3, and copies its (shift, status) record to pinned host slot
    k % 2, so iteration k+1 can run while the host checks iteration k's shift
    without touching the labels or centroids iteration k would return
    (``run``).  ``c_cur`` / ``c_nxt`` / ``ids`` are the current iteration's
    buffers.
    """

    def __init__(self, B: int, N: int, K: int, D: int, dtype: torch.dtype, device,
                 metric: str = "euclid", use_graphs: bool = True):
        """``metric``: "euclid" (nearest centroid, mean update) or "dot"
        (largest dot product, L2-normalised mean update: the cosine and
        dot-product k-means of the reference).  ``use_graphs``: replay the
        steady-state step as CUDA graphs (see ``step``); capturing the three
        pairs (one per centroid buffer) costs a few ms of host time, so it pays
        for long runs only."""
        if metric not in ("euclid", "dot"):
            raise ValueError(f"unknown metric {metric!r}")
        self.metric = metric
        self.B, self.N, self.K, self.D, self.dtype = B, N, K, D, dtype
        self.device = torch.device(device)
        dev = self.device
        self._cbuf = [_ops.empty_rows(B, K, D, dtype, dev) for _ in range(3)]
        self._ibuf = [torch.empty((B, N), dtype=torch.int32, device=dev) for _ in range(3)]
        self._k = 0   # current iteration: reads _cbuf[k % 3]
        self.sums = torch.empty((B, K, D), dtype=torch.float32, device=dev)
        self.hist = torch.empty((B, K), dtype=torch.int32, device=dev)
        self.csq = torch.empty((B, K), dtype=torch.float32, device=dev)
        # [0] shift (float32 bits), [1] device status, [2..3] spare; each step
        # copies it to pinned slot k % 2 and records that slot's event
        self.stat = torch.zeros(4, dtype=torch.int32, device=dev)
        self.stat_host = torch.zeros((2, 4), dtype=torch.int32, pin_memory=True)
        self._stat_ev = [torch.cuda.Event(), torch.cuda.Event()]
        self._stat_k = [-1, -1]   # iteration whose record each slot holds
        self.csq_valid = False
        lib = nat.load()
        # float32 x with rows of at most XSPLIT_MAX_D: its tf32 halves are
        # split once per load() into the workspace (twice x's bytes) when the
        # device has room, instead of in every assignment tile
        free = torch.cuda.mem_get_info(dev)[0] if dtype == torch.float32 else 0
        self.xcode, ws_bytes = nat.accumulate_x_code(lib, dtype, B, N, K, D, free, 0.5)
        self.ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        self.x = None
        self.x_sq = None
        self.use_graphs = use_graphs
        self._graphs = {}
        self._arg_cache = {}
        self._capture_stream = None
        self._steps = 0

    @property
    def kernels_per_step(self) -> int:
        """Kernel launches of one ``step()``, following fk_assign_accumulate's
        method: privatised -> c_sq staging, assignment, privatised sum,
        finalize; fused -> c_sq staging, assignment with fused accumulation,
        finalize; sorted -> c_sq staging, assignment, scan, scatter, segmented
        sum, finalize."""
        method = nat.load().fk_assign_accumulate_method(self.K, self.D, nat.dtype_code(self.dtype))
        if self.metric == "dot":  # as below, without the c_sq staging
            return {nat.FK_ACC_PRIVATISED: 3, nat.FK_ACC_FUSED: 2}.get(method, 5)
        return {nat.FK_ACC_PRIVATISED: 4, nat.FK_ACC_FUSED: 3}.get(method, 6)

    # ------------------------------------------------------------ buffers
    @property
    def c_cur(self) -> torch.Tensor:
        """Centroids the current iteration assigns with."""
        return self._cbuf[self._k % 3]

    @property
    def c_nxt(self) -> torch.Tensor:
        """Centroids the current iteration's update writes."""
        return self._cbuf[(self._k + 1) % 3]

    @property
    def ids(self) -> torch.Tensor:
        """Labels of the current iteration."""
        return self._ibuf[self._k % 3]

    @property
    def iteration(self) -> int:
        """Index of the current iteration since ``load``."""
        return self._k

    # ---------------------------------------------------------------- set-up
    def load(self, x: torch.Tensor, centroids: torch.Tensor, x_sq: torch.Tensor | None = None):
        self.x = _ops.ensure_tma(x)
        if self.metric == "euclid":
            self.x_sq = x_sq if x_sq is not None else _ops.row_sqnorm(self.x)
        if self.xcode == nat.FK_F32_XSPLIT:
            with torch.cuda.device(self.device):
                nat.check(nat.load().fk_assign_accumulate_split_x(
                    nat.ptr(self.x), self.B, self.N, self.K, self.D, nat.strides(self.x, 3),
                    nat.ptr(self.ws), self.ws.numel(), nat.stream_handle(self.device)),
                    "fk_assign_accumulate_split_x")
        self._k = 0
        self._stat_k = [-1, -1]
        self.c_cur.copy_(centroids.view(self.B, self.K, self.D))
        self.csq_valid = False
        self._graphs.clear()   # captured with the previous x
        self._arg_cache.clear()
        self._steps = 0
        self.stat.zero_()
        self.hist.zero_()
        self.sums.zero_()

    # ------------------------------------------------------------- iteration
    def step(self, ev_assign=None) -> None:
        """One Lloyd iteration: ids <- assign(centroids); c_nxt <- update; shift.

        ``ev_assign``: optional (start, end) CUDA events recorded around the
        assignment (with its accumulation) on the current stream.

        From the second step on (the first one stages c_sq from the centroids
        and sets the kernels' shared-memory attributes) the two launches of a
        step replay as CUDA graphs, one pair per centroid buffer, so a step
        costs two graph launches on the host instead of argument marshalling,
        tensor-map encoding and three to six kernel launches.  Every step then
        copies its (shift, status) record to pinned slot k % 2."""
        # a caller that overwrote c_cur clears csq_valid: the Euclidean graph
        # would pass the stale c_sq, so that step runs eagerly
        if self.use_graphs and self._steps > 0 and (self.metric == "dot" or self.csq_valid):
            pair = self._graph_pair()
            if pair is not None:
                if ev_assign is not None:
                    ev_assign[0].record()
                pair[0].replay()
                if ev_assign is not None:
                    ev_assign[1].record()
                pair[1].replay()
                self._steps += 1
                self._post_stat()
                return
        if ev_assign is not None:
            ev_assign[0].record()
        self._launch_assign()
        if ev_assign is not None:
            ev_assign[1].record()
        self._launch_finalize()
        self.csq_valid = True
        self._steps += 1
        self._post_stat()

    def _post_stat(self) -> None:
        slot = self._k % 2
        self.stat_host[slot].copy_(self.stat, non_blocking=True)
        self._stat_ev[slot].record()
        self._stat_k[slot] = self._k

    def _launch_assign(self) -> None:
        """Assignment with the per-cluster sums and counts, on the current stream."""
        lib = nat.load()
        s = nat.stream_handle(self.device)
        if self.metric == "dot":
            nat.check(lib.fk_assign_dot_accumulate(*self._args("assign"), s),
                      "fk_assign_dot_accumulate")
        else:
            nat.check(lib.fk_assign_accumulate(*self._args("assign"), s), "fk_assign_accumulate")

    def _launch_finalize(self) -> None:
        """New centroids, shift (and the next c_sq), accumulators reset."""
        lib = nat.load()
        s = nat.stream_handle(self.device)
        if self.metric == "dot":
            nat.check(lib.fk_centroid_finalize_normalized(*self._args("finalize"), s),
                      "fk_centroid_finalize_normalized")
        else:
            nat.check(lib.fk_centroid_finalize(*self._args("finalize"), s), "fk_centroid_finalize")

    def _args(self, which: str) -> tuple:
        """ctypes arguments (all but the stream) of this step's calls, built
        once per centroid buffer and c_sq state: marshalling them costs more
        host time than the launches themselves."""
        c_sq_on = self.metric == "euclid" and self.csq_valid
        key = (which, self.c_cur.data_ptr(), c_sq_on)
        a = self._arg_cache.get(key)
        if a is not None:
            return a
        B, N, K, D = self.B, self.N, self.K, self.D
        x = self.x
        status = nat.ptr(self.stat[1:2])
        if which == "assign" and self.metric == "dot":
            a = (nat.ptr(x), nat.ptr(self.c_cur), nat.ptr(self.ids), nat.ptr(self.hist),
                 nat.ptr(self.sums), self.xcode, B, N, K, D, nat.strides(x, 3),
                 nat.strides(self.c_cur, 3), nat.strides(self.ids, 2), nat.ptr(self.ws),
                 self.ws.numel(), status)
        elif which == "assign":
            a = (nat.ptr(x), nat.ptr(self.c_cur), nat.ptr(self.x_sq),
                 nat.ptr(self.csq if c_sq_on else None), nat.ptr(self.ids), nat.ptr(self.hist),
                 nat.ptr(self.sums), self.xcode, nat.dtype_code(self.x_sq.dtype),
                 nat.FK_F32, B, N, K, D, nat.strides(x, 3), nat.strides(self.c_cur, 3),
                 nat.strides(self.x_sq, 2), nat.strides(self.csq, 2), nat.strides(self.ids, 2),
                 nat.ptr(self.ws), self.ws.numel(), status)
        elif self.metric == "dot":
            a = (nat.ptr(self.sums), nat.ptr(self.hist), nat.ptr(self.c_cur), nat.ptr(self.c_nxt),
                 nat.dtype_code(self.dtype), B, K, D, nat.strides(self.c_cur, 3),
                 nat.strides(self.c_nxt, 3), nat.ptr(self.stat[0:1]), 1)
        else:
            a = (nat.ptr(self.sums), nat.ptr(self.hist), nat.ptr(self.c_cur), nat.ptr(self.c_nxt),
                 nat.dtype_code(self.dtype), B, K, D, nat.strides(self.c_cur, 3),
                 nat.strides(self.c_nxt, 3), nat.ptr(self.csq), nat.ptr(self.stat[0:1]), 1)
        self._arg_cache[key] = a
        return a

    def _graph_pair(self):
        """(assignment, finalize) graphs for the current centroid buffer,
        captured on first use; None (eager from then on) if capture fails."""
        key = self.c_cur.data_ptr()
        pair = self._graphs.get(key)
        if pair is not None:
            return pair
        cur = torch.cuda.current_stream(self.device)
        side = self._capture_stream
        if side is None:
            side = self._capture_stream = torch.cuda.Stream(self.device)
        side.wait_stream(cur)
        try:
            pair = []
            with torch.cuda.stream(side):
                for launch in (self._launch_assign, self._launch_finalize):
                    g = torch.cuda.CUDAGraph()
                    # thread-local: the capture restricts only this thread's
                    # CUDA calls (kernel launches and memsets here), not those
                    # of other threads such as a communicator's
                    g.capture_begin(capture_error_mode="thread_local")
                    try:
                        launch()
                    finally:
                        g.capture_end()
                    pair.append(g)
        except RuntimeError:
            self.use_graphs = False
            self._graphs.clear()
            cur.wait_stream(side)
            return None
        cur.wait_stream(side)
        self._graphs[key] = pair
        return pair

    def advance(self) -> None:
        """Adopt the updated centroids for the next iteration."""
        self._k += 1

    def read_stat(self):
        """(shift, device status) of the last step; waits for that step."""
        return self.read_stat_of(self._k)

    def read_stat_of(self, k: int):
        """(shift, device status) of iteration k, one of the last two
        iterations stepped; waits until its record has reached the host."""
        slot = k % 2
        if self._stat_k[slot] != k:
            raise RuntimeError(f"no (shift, status) record of iteration {k}")
        self._stat_ev[slot].synchronize()
        row = self.stat_host[slot]
        return row[0:1].view(torch.float32).item(), int(row[1].item())

    def run(self, max_iters: int, tol: float, need_sync: bool, verbose_fmt: str | None = None):
        """Lloyd iterations from the loaded centroids until ``max_iters`` or a
        shift below ``tol`` (read only when ``need_sync``); returns (labels,
        centroids, iterations) with the reference's break semantics: on a
        break the labels of that iteration and the centroids that produced
        them, else the last labels and the last update's centroids.

        Iteration it+1 is queued before iteration it's shift is read: it
        writes the other ring buffers, so the device does not wait on the
        host's check, and a break discards it (one speculative iteration of
        device work at convergence)."""
        self.step()
        for it in range(max_iters):
            if it + 1 < max_iters:
                self.advance()
                self.step()
            if need_sync:
                shift, code = self.read_stat_of(it)
                self.raise_on_status(code)
                if verbose_fmt is not None:
                    print(verbose_fmt.format(it=it, shift=shift))
                if shift < tol:
                    return self._ibuf[it % 3], self._contiguous(self._cbuf[it % 3]), it + 1
        last = max_iters - 1
        if not need_sync:
            _, code = self.read_stat_of(last)
            self.raise_on_status(code)
        return self._ibuf[last % 3], self._contiguous(self._cbuf[(last + 1) % 3]), max_iters

    def raise_on_status(self, code: int) -> None:
        if code:
            raise RuntimeError(f"flash_kmeans device error {code}: {nat.device_status_message(code)}")

    def result_centroids(self) -> torch.Tensor:
        return self._contiguous(self.c_cur)

    @staticmethod
    def _contiguous(c: torch.Tensor) -> torch.Tensor:
        return c if c.is_contiguous() else c.contiguous()


def batch_kmeans_Euclid(
    x,
    n_clusters,
    max_iters=100,
    tol=0.0,
    init_centroids=None,
    verbose=False,
    *,
    use_heuristic=True,
):
    """Batched k-means (Euclidean) on CUDA; reference kmeans_triton_impl.py:55-115.

    Args:
        x: (B, N, D) float16 / bfloat16 / float32 CUDA tensor.
        n_clusters: K.
        max_iters: maximum number of Lloyd iterations (>= 1).
        tol: stop when the max centroid shift is below tol.
        init_centroids: optional (B, K, D) initial centroids.
        verbose: print the shift per iteration.
        use_heuristic: accepted for compatibility, ignored.
    Returns:
        cluster_ids (B, N) int32, centroids (B, K, D) x.dtype, number of iterations.
    """
    if not torch.cuda.is_available() or not x.is_cuda:
        raise RuntimeError("batch_kmeans_Euclid needs a CUDA tensor (this build has no CPU fallback)")
    if max_iters < 1:
        raise ValueError("max_iters must be >= 1")
    B, N, D = x.shape
    K = int(n_clusters)
    if init_centroids is None:
        indices = torch.randint(0, N, (B, K), device=x.device)
        centroids = torch.gather(x, dim=1, index=indices[..., None].expand(-1, -1, D))
    else:
        centroids = init_centroids
    centroids = centroids.view(B, K, D)

    with torch.cuda.device(x.device):
        eng = LloydEngine(B, N, K, D, x.dtype, x.device, use_graphs=max_iters >= _GRAPH_MIN_ITERS)
        eng.load(x, centroids)
        return eng.run(max_iters, _round_tol(tol, x.dtype), tol > 0 or verbose,
                       "Iter {it}, center shift: {shift:.6f}" if verbose else None)


def _batch_kmeans_similarity(x, n_clusters, max_iters, tol, init_centroids, verbose, cosine):
    name = "batch_kmeans_Cosine" if cosine else "batch_kmeans_Dot"
    if not torch.cuda.is_available() or not x.is_cuda:
        raise RuntimeError(f"{name} needs a CUDA tensor (this build has no CPU fallback)")
    if max_iters < 1:
        raise ValueError("max_iters must be >= 1")
    B, N, D = x.shape
    K = int(n_clusters)
    with torch.cuda.device(x.device):
        xs = _ops.row_normalize(x) if cosine else x
        if init_centroids is None:
            indices = torch.randint(0, N, (B, K), device=x.device)
            centroids = torch.gather(xs, dim=1, index=indices[..., None].expand(-1, -1, D))
        else:
            centroids = init_centroids
        centroids = centroids.view(B, K, D)
        if cosine:
            centroids = _ops.row_normalize(centroids)
        eng = LloydEngine(B, N, K, D, x.dtype, x.device, metric="dot",
                          use_graphs=max_iters >= _GRAPH_MIN_ITERS)
        eng.load(xs, centroids)
        tag = "" if cosine else " (dot)"
        return eng.run(max_iters, _round_tol(tol, x.dtype), tol > 0 or verbose,
                       f"Iter {{it}}{tag}, center shift: {{shift:.6f}}" if verbose else None)


def batch_kmeans_Cosine(x, n_clusters, max_iters=100, tol=0.0, init_centroids=None, verbose=False):
    """Batched k-means by cosine similarity; reference kmeans_triton_impl.py:118-158.

    x (B, N, D) is L2-normalised in its dtype, centroids start from normalised
    random points (or ``init_centroids``, normalised), each iteration assigns
    by the largest dot product and replaces each centroid by its cluster's
    normalised mean.  On a tolerance break the centroids of the last
    assignment are returned, as in the reference.
    Returns cluster_ids (B, N) int32, centroids (B, K, D) x.dtype, iterations.
    """
    return _batch_kmeans_similarity(x, n_clusters, max_iters, tol, init_centroids, verbose, True)


def batch_kmeans_Dot(x, n_clusters, max_iters=100, tol=0.0, init_centroids=None, verbose=False):
    """Batched k-means by raw dot product; reference kmeans_triton_impl.py:161-188.

    Like batch_kmeans_Cosine without normalising x or the initial centroids;
    the update still normalises the cluster means (the reference's
    _dot_iter uses the cosine update).
    """
    return _batch_kmeans_similarity(x, n_clusters, max_iters, tol, init_centroids, verbose, False)
