"""Benchmark of the Lloyd-iteration hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload cfg2|cfg1|cfg3|cfg4|cfg5] [--op lloyd|assign] [--stream]
                    [--metric euclid|cosine|dot] [--no-large-n] [--no-cpu-baseline]

A step is one Lloyd iteration (assign + update + shift check) over the whole
batch of the workload.  Default workload: BASELINE config 2 (B=32, N=75600,
D=128, K=1000, fp16, x ~ N(0,1)), which fits one GPU.  With N>1 ranks
(torchrun, NCCL) the batches are split between the ranks (strong scaling:
rank r clusters batches [r*B/N, (r+1)*B/N) of the same data; the batched path
has no exchange step), and `value` is the whole workload's rate.

`value`: assign-equivalent TFLOP/s = 2*B*N*K*D per iteration / time per
iteration (max over ranks), whole job.  `e2e`: the same metric through the
public API (`batch_kmeans_Euclid`, 20 iterations, tol 1e-4) with each rank's
x copied from pinned host memory and the labels/centroids copied back inside
each timed step.  `roofline`: the assignment kernel's own CUDA-event time
against the measured dense bf16 peak.  `cpu_baseline` / `--impl reference`:
the reference's own CPU path (`torch_fallback._euclid_iter_torch_naive`,
imported from the reference installed under baseline/_ref) with every host
thread, on a bounded sample of the workload's batches; when that install is
absent, the numpy restatement in oracle/ (kind "port").
`large_n` (default workload, every N): config 5 through kmeans_largeN's
engine (N=2^26, D=128, K=8192, fp32, x in pinned host memory, partitioned
over the ranks): ms per iteration streamed from host every pass and resident
in HBM, per-rank H2D GB/s, NCCL all-reduce time, the concurrent pinned-H2D
ceiling of the ranks, and a parity check of the multi-GPU reduction; with 4
or more ranks and the host memory for it, also the 2^28-point scaling point.
`--op assign`: the assignment alone (`euclid_assign_triton`, labels only, the
predict path) per step, instead of a Lloyd iteration.
`--workload cfg5`: config 5 alone as the headline (N partitioned over the
ranks, NCCL all-reduce of the partial sums); each rank's shard stays resident
in HBM after the first pass when it fits, `--stream` re-streams it.
`--metric cosine|dot`: the same step for batch_kmeans_Cosine / batch_kmeans_Dot
(dot-product argmax assignment, normalised-mean update; x row-normalised
once, outside the timed region, for cosine); the CPU leg is skipped.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "flash-kmeans_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "ms/Lloyd iter and assign TFLOP/s (% of peak) at 1/2/4/8 B200 vs host CPU"
UNIT = "TFLOP/s"

WORKLOADS = {
    "cfg1": dict(B=2, N=16384, D=128, K=256, dtype="float32", gen="gmm", comps=256, mean_std=2.0),
    "cfg2": dict(B=32, N=75600, D=128, K=1000, dtype="float16", gen="randn"),
    "cfg3": dict(B=1, N=1 << 22, D=128, K=128, dtype="float16", gen="gmm", comps=128,
                 mean_std=3.0, dirichlet=True, cpu_n=1 << 20),
    "cfg4": dict(B=1, N=262144, D=2048, K=1024, dtype="float32", gen="randn", cpu_n=65536),
    # out-of-core kmeans_largeN: x in pinned host memory, streamed in BLOCK_N blocks,
    # N partitioned contiguously over the ranks (one process per GPU)
    "cfg5": dict(B=1, N=1 << 26, D=128, K=8192, dtype="float32", gen="randn", large=True,
                 block=1 << 20, cpu_n=1 << 16),
}


def _flops(w):
    return 2.0 * w["B"] * w["N"] * w["K"] * w["D"]


def _describe(name, w):
    return (f"{name}: B={w['B']} N={w['N']} D={w['D']} K={w['K']} {w['dtype']}, "
            + ("x~N(0,1)" if w["gen"] == "randn" else f"GMM({w['comps']} comps)"))


# ------------------------------------------------------------ CPU baselines
REF_FALLBACK = os.path.join(ROOT, "baseline", "_ref", "flash_kmeans", "torch_fallback.py")


def _load_reference_fallback():
    """The reference's own CPU path (flash_kmeans/torch_fallback.py of the
    reference installed under baseline/_ref), loaded under a private name so
    it cannot shadow this repository's flash_kmeans package; None if absent."""
    if not os.path.exists(REF_FALLBACK):
        return None
    import importlib.util
    spec = importlib.util.spec_from_file_location("_reference_torch_fallback", REF_FALLBACK)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


class CpuReference:
    """One Lloyd iteration of the reference's torch CPU path
    (``_euclid_iter_torch_naive``, torch_fallback.py:111-135) per step on a
    sample of the workload's batches (``cpu_n`` points each), all host
    threads.  The number of batches is sized from the first (untimed) step so
    that a step takes about two seconds."""

    kind = "reference"

    def __init__(self, w, mod):
        import torch
        self.w, self.mod = w, mod
        self.cores = os.cpu_count() or 1
        torch.set_num_threads(self.cores)
        self.n = w.get("cpu_n", w["N"])
        self.batches = 1
        self._sized = False

    def _inputs(self, seed):
        import torch
        w = self.w
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((self.batches, self.n, w["D"]), generator=g).to(getattr(torch, w["dtype"]))
        idx = torch.randint(0, self.n, (self.batches, w["K"]), generator=g)
        c = torch.gather(x, 1, idx[..., None].expand(-1, -1, w["D"]))
        return x, (x ** 2).sum(dim=-1), c          # x_sq as batch_kmeans_Euclid_torch_native

    def step(self, seed=0):
        x, x_sq, c = self._inputs(seed)
        t0 = time.perf_counter()
        self.mod._euclid_iter_torch_naive(x, x_sq, c)
        secs = time.perf_counter() - t0
        if not self._sized:   # the first step sizes the sample
            self._sized = True
            self.batches = max(1, min(self.w["B"], int(2.0 / max(secs, 1e-3))))
        return secs

    def tflops(self, seconds):
        return 2.0 * self.n * self.w["K"] * self.w["D"] * self.batches / seconds / 1e12

    def sample(self):
        part = "" if self.n == self.w["N"] else f" ({self.n} of their {self.w['N']} points)"
        return (f"{self.batches} of {self.w['B']} batches of the workload{part}, one Lloyd "
                f"iteration per step (reference torch_fallback._euclid_iter_torch_naive, "
                f"{self.cores} threads, {_cpu_model()})")

    def close(self):
        pass


def _oracle_batch_iter(args):
    """One Lloyd iteration of the numpy oracle on one batch (runs in a worker)."""
    seed, N, K, D, dtype = args
    import numpy as np
    from oracle import kmeans_oracle as ko
    rng = np.random.default_rng(seed)
    x = ko.round_to(rng.standard_normal((1, N, D), dtype=np.float32), dtype)
    c = ko.init_from_points(rng, x, K, replace=True)
    t0 = time.perf_counter()
    x_sq = ko.row_sqnorm(x, dtype)
    ko.lloyd_iter(x, x_sq, c, dtype, exact_order=False)
    return time.perf_counter() - t0


class CpuOracle:
    """The numpy restatement of the reference's CPU path (used when the
    reference install is absent): a spawned pool, one process per core, each
    step one Lloyd iteration on one batch per process."""

    kind = "port"

    def __init__(self, w):
        import multiprocessing as mp
        os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
        os.environ.setdefault("OMP_NUM_THREADS", "1")
        self.w = w
        self.cores = max(1, min(os.cpu_count() or 1, w["B"]))
        self.pool = mp.get_context("spawn").Pool(self.cores)

    def step(self, seed=0):
        w = self.w
        jobs = [(seed * 1000 + i, w.get("cpu_n", w["N"]), w["K"], w["D"], w["dtype"])
                for i in range(self.cores)]
        t0 = time.perf_counter()
        self.pool.map(_oracle_batch_iter, jobs)
        return time.perf_counter() - t0

    def tflops(self, seconds):
        n = self.w.get("cpu_n", self.w["N"])
        return 2.0 * n * self.w["K"] * self.w["D"] * self.cores / seconds / 1e12

    def sample(self):
        n = self.w.get("cpu_n", self.w["N"])
        part = "" if n == self.w["N"] else f" ({n} of their {self.w['N']} points)"
        return (f"{self.cores} of {self.w['B']} batches of the workload{part}, one Lloyd "
                f"iteration per step (numpy oracle, one process per core, {_cpu_model()})")

    def close(self):
        self.pool.close()
        self.pool.join()


def cpu_baseline_runner(w):
    """The reference's CPU path when installed, else the numpy restatement."""
    mod = _load_reference_fallback()
    return CpuReference(w, mod) if mod is not None else CpuOracle(w)


# -------------------------------------------------------------- clock sampler
class ClockSampler:
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting"}

    def __init__(self, torch_device, period_s=0.001):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self.power_w = []
        self.period = period_s
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            import torch
            uuid = str(torch.cuda.get_device_properties(torch_device).uuid)
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # sampling is best effort; the JSON says so
            self.error = repr(e)
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self, power):
        nv = self._nv
        try:
            self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
            self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            if power:
                self.power_w.append(nv.nvmlDeviceGetPowerUsage(self._h) / 1000.0)
        except Exception:
            pass

    def _run(self):
        # clock and throttle reasons on every pass, power on every 8th: each
        # NVML query takes a while, and the timed regions are short
        i = 0
        while not self._stop.is_set():
            self._sample(i % 8 == 0)
            i += 1
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._h is not None:
            self._t.join()
            self._sample(True)   # the end of the timed region, with the device still warm

    def summary(self):
        if self._h is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": "NVML unavailable"}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz,
                "reasons": [n for b, n in self.REASONS.items() if self.reasons & b],
                "samples": len(self.samples),
                "power_w_max": max(self.power_w) if self.power_w else None}


# ----------------------------------------------------------------- our arm
def _make_inputs(w, device, seed=0):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    B, N, D, K = w["B"], w["N"], w["D"], w["K"]
    dt = getattr(torch, w["dtype"])
    if w["gen"] == "randn":
        x = torch.randn((B, N, D), device=device, generator=g, dtype=torch.float32)
    else:
        means = torch.randn((B, w["comps"], D), device=device, generator=g) * w["mean_std"]
        if w.get("dirichlet"):
            wts = torch.distributions.Dirichlet(torch.ones(w["comps"])).sample((B,)).to(device)
        else:
            wts = torch.full((B, w["comps"]), 1.0 / w["comps"], device=device)
        comp = torch.multinomial(wts, N, replacement=True, generator=g)
        x = torch.gather(means, 1, comp[..., None].expand(-1, -1, D))
        x += torch.randn((B, N, D), device=device, generator=g)
    x = x.to(dt)
    idx = torch.randint(0, N, (B, K), device=device, generator=g)
    c0 = torch.gather(x, 1, idx[..., None].expand(-1, -1, D)).contiguous()
    return x, c0


def _load_traffic(name):
    path = os.path.join(ROOT, "profiles", f"assign_{name}_ncu.json")
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except Exception:
        return None


def _hbm_bound(alg_bytes, flops, burst_tflops, hbm_gbs):
    """True when a launch's algorithmic bytes at the measured copy bandwidth take
    longer than its FLOPs at the measured dense bf16 peak."""
    return alg_bytes / (hbm_gbs * 1e9) > flops / (burst_tflops * 1e12)


def _roofline(hbm_bound, tflops, alg_bytes, ms, burst, sustained, hbm, src, traffic):
    """The binding roofline of the assignment launch: the tensor pipe when its
    FLOPs take longer at the measured GEMM peak than its algorithmic bytes at the
    measured copy bandwidth (configs 2 and 4), else HBM (config 3: K=128 gives
    128 FLOPs per byte of x, below the ridge)."""
    if hbm_bound:
        gbs = alg_bytes / (ms * 1e-3) / 1e9
        return {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(gbs / hbm, 4), "peak_source": f"{src} copy bandwidth, per GPU",
                "algorithmic_bytes": int(alg_bytes), "tensor_tflops": round(tflops, 2),
                "traffic": traffic}
    return {"bound": "tensor", "achieved": round(tflops, 2), "peak": burst, "unit": "TFLOP/s",
            "frac": round(tflops / burst, 4), "peak_source": f"{src} dense bf16 (burst), per GPU",
            "frac_of_sustained": round(tflops / sustained, 4) if sustained else None,
            "algorithmic_bytes": int(alg_bytes), "traffic": traffic}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p.get("bf16_tflops_sustained"), p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def _batch_range(B, rank, world):
    """Contiguous batches [b0, b1) of rank `rank` out of `world`."""
    return rank * B // world, (rank + 1) * B // world


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import flash_kmeans
    from flash_kmeans import _ops
    from flash_kmeans.kmeans_triton_impl import LloydEngine

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, N, D, K = w["B"], w["N"], w["D"], w["K"]
    if world > B:
        raise SystemExit(f"{world} ranks but only {B} batches to split")
    sim = args.metric != "euclid"
    driver = {"euclid": flash_kmeans.batch_kmeans_Euclid, "cosine": flash_kmeans.batch_kmeans_Cosine,
              "dot": flash_kmeans.batch_kmeans_Dot}[args.metric]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not sim:
        cpu = cpu_baseline_runner(w)  # a spawned pool, if any, starts before heavy GPU work

    # every rank builds the same data and keeps its own batches: the workload is
    # identical at every rank count (strong scaling of the batch axis)
    b0, b1 = _batch_range(B, rank, world)
    x_all, c_all = _make_inputs(w, dev, seed=1234)
    x, c0 = x_all[b0:b1].contiguous(), c_all[b0:b1].contiguous()
    del x_all, c_all
    torch.cuda.empty_cache()
    Bl = b1 - b0
    eng = LloydEngine(Bl, N, K, D, x.dtype, dev, metric="dot" if sim else "euclid")
    if args.metric == "cosine":
        eng.load(_ops.row_normalize(x), _ops.row_normalize(c0))
    else:
        eng.load(x, c0)
    torch.cuda.synchronize()

    steps, warm = args.steps, args.warmup
    a0 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    a1 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]

    def iterations(n, timed):
        """n Lloyd iterations as the drivers run them (LloydEngine.run): each
        iteration's (shift, status) is read back on the host - the reference's
        per-iteration `shift < tol` check - after the next one is queued."""
        k0 = eng.iteration
        eng.step(ev_assign=(a0[0], a1[0]) if timed else None)
        for i in range(n):
            if i + 1 < n:
                eng.advance()
                eng.step(ev_assign=(a0[i + 1], a1[i + 1]) if timed else None)
            shift, code = eng.read_stat_of(k0 + i)
            if code:
                raise RuntimeError(f"device status {code}")
        eng.advance()

    iterations(warm, False)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        iterations(steps, True)
        e1.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / steps
    assign_ms = sum(a0[i].elapsed_time(a1[i]) for i in range(steps)) / steps
    t = torch.tensor([ms, assign_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, assign_ms = float(t[0]), float(t[1])

    flops = _flops(w)                     # the whole workload, all ranks
    flops_rank = flops * Bl / B           # this rank's share (equal shares when world | B)
    value = flops / (ms * 1e-3) / 1e12
    burst, sustained, hbm, src = _peaks()
    achieved = flops_rank / (assign_ms * 1e-3) / 1e12
    # algorithmic DRAM bytes of one assignment launch on this rank: x, x_sq and
    # the centroids read once, labels and float32 sums written once
    alg_bytes = sum(t.numel() * t.element_size() for t in (eng.x, eng.x_sq, eng.c_cur, eng.ids)
                    if t is not None) + eng.sums.numel() * 4
    hbm_bound = _hbm_bound(alg_bytes, flops_rank, burst, hbm)

    # ---- the labels-only assignment (`--op assign`'s kernel, the predict path)
    # on the same resident data, so both assignment numbers come from one run
    labels_only = None
    if not sim:
        from flash_kmeans.assign_euclid_triton import euclid_assign_triton
        out_l = torch.empty((Bl, N), dtype=torch.int32, device=dev)
        for _ in range(3):
            euclid_assign_triton(eng.x, eng.c_cur, eng.x_sq, out=out_l)
        n_l = max(steps, 5)
        l0 = torch.cuda.Event(enable_timing=True)
        l1 = torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        l0.record()
        for _ in range(n_l):
            euclid_assign_triton(eng.x, eng.c_cur, eng.x_sq, out=out_l)
        l1.record()
        torch.cuda.synchronize()
        tl = torch.tensor([l0.elapsed_time(l1) / n_l], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tl, op=dist.ReduceOp.MAX)
        lms = float(tl[0])
        labels_only = {"ms": round(lms, 4),
                       "tflops": round(flops_rank / (lms * 1e-3) / 1e12, 2),
                       "frac_of_burst": round(flops_rank / (lms * 1e-3) / 1e12 / burst, 4),
                       "calls": n_l,
                       "call": "euclid_assign_triton(x, c, x_sq, out=...) on the engine's resident "
                               "tensors, labels only (no sums), back to back"}
        del out_l

    # ---- e2e through the public API with host buffers (each rank its batches)
    e2e = None
    if args.e2e_steps > 0:
        x_h = x.cpu().pin_memory()
        c_h = c0.cpu().pin_memory()
        # the results come back into pinned host buffers, as the inputs go out of them
        ids_h = torch.empty((Bl, N), dtype=torch.int32, pin_memory=True)
        cent_h = torch.empty((Bl, K, D), dtype=x.dtype, pin_memory=True)
        del x, eng
        torch.cuda.empty_cache()
        iters_total, t_total = 0, 0.0
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        for s_ in range(args.e2e_steps + 1):
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            f0.record()
            xd = x_h.to(dev, non_blocking=True)
            cd = c_h.to(dev, non_blocking=True)
            ids, cent, n_it = driver(xd, K, max_iters=20, tol=1e-4, init_centroids=cd)
            ids_h.copy_(ids, non_blocking=True)
            cent_h.copy_(cent, non_blocking=True)
            f1.record()
            torch.cuda.synchronize()
            if s_ > 0:  # first run is warm-up
                iters_total += n_it
                t_total += f0.elapsed_time(f1) * 1e-3
            del xd, cd, ids, cent
        tt = torch.tensor([t_total, iters_total], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        per_step = float(tt[0]) / args.e2e_steps
        # each rank ran its own batches for its own iteration count; the rate
        # counts every rank's work over the slowest rank's time
        work = torch.tensor([flops_rank * iters_total / args.e2e_steps], device=dev,
                            dtype=torch.float64)
        if world > 1:
            dist.all_reduce(work)
        e2e = {"value": round(float(work[0]) / per_step / 1e12, 3),
               "unit": UNIT,
               "h2d_bytes_per_step": int(x_h.numel() * x_h.element_size()
                                         + c_h.numel() * c_h.element_size()),
               "d2h_bytes_per_step": int(ids_h.numel() * 4 + cent_h.numel() * cent_h.element_size()),
               "step": f"{driver.__name__}(max_iters=20, tol=1e-4) on each rank's batches copied "
                       "from pinned host, labels+centroids copied back (bytes per rank)",
               "iters_per_step": iters_total / args.e2e_steps}
    else:
        del x, eng
        torch.cuda.empty_cache()

    large_n = None
    if args.workload == "cfg2" and args.metric == "euclid" and not args.no_large_n:
        large_n = large_n_record(rank, world, dev)

    cpu_baseline = None
    if cpu is not None:
        cpu.step(seed=99)                      # warm-up (sizes the reference's sample)
        secs = cpu.step(seed=7)
        cpu_baseline = {"value": round(cpu.tflops(secs), 5), "unit": UNIT, "cores": cpu.cores,
                        "kind": cpu.kind, "sample": cpu.sample()}
        cpu.close()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16" if w["dtype"] == "float16" else ("bf16" if w["dtype"] == "bfloat16" else "f32(3xTF32)"),
            "data": "synthetic (seeded torch generator; shapes/distribution of the BASELINE config)",
            "config": {"workload": _describe(args.workload, w),
                       "metric": args.metric,
                       "parallelism": (f"batches split over {world} ranks ({B // world} or "
                                       f"{-(-B // world)} each), no exchange step"
                                       if world > 1 else "single GPU"),
                       "l2": "inputs exceed the 126 MB L2 (x is %d MB); no flush" %
                             (B * N * D * (2 if w["dtype"] != "float32" else 4) // 2 ** 20),
                       "step": "one Lloyd iteration incl. the per-iteration shift readback"},
            "ms_per_iter": round(ms, 4),
            "assign_ms": round(assign_ms, 4),
            "assign_labels_only": labels_only,
            "roofline": _roofline(hbm_bound, achieved, alg_bytes, assign_ms, burst, sustained, hbm,
                                  src, None if sim else _load_traffic(args.workload)),
            "e2e": e2e,
            "cpu_baseline": cpu_baseline,
            "large_n": large_n,
            "gpu_launches": LloydEngine(1, 1, K, D, getattr(torch, w["dtype"]), dev,
                                        metric="dot" if sim else "euclid").kernels_per_step * steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)


# --------------------------------------------------- out-of-core record (cfg5)
LARGE_N = dict(N=1 << 26, D=128, K=8192, block=1 << 20)
LARGE_N_BIG = dict(N=1 << 28, D=128, K=16384, block=1 << 20)  # its scaling point


def _fill_host_blocks(x_h, p0, block, seed, dev):
    """Rows p0.. of the global point set (x ~ N(0,1), float32), generated
    block by block on the GPU from seed + global block index, so the data is
    the same for any partition into block-aligned shards."""
    import torch
    n, D = x_h.shape
    for a in range(0, n, block):
        rows = min(block, n - a)
        g = torch.Generator(device=dev).manual_seed(seed + (p0 + a) // block)
        x_h[a:a + rows].copy_(torch.randn((rows, D), device=dev, generator=g))
    torch.cuda.synchronize(dev)


def _largeN_iters(lane, pg, warm, steps):
    """ms per Lloyd iteration of one lane (max over ranks) and the mean NCCL
    all-reduce time per iteration, CUDA events on the lane's compute stream."""
    import torch
    import torch.distributed as dist
    from flash_kmeans import kmeans_large as kl
    ar = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]

    def one(i, wrap):
        lane.run_pass(wrap=wrap)
        if i is not None:
            ar[i][0].record(lane.compute_stream)
        kl._allreduce([lane], pg)
        if i is not None:
            ar[i][1].record(lane.compute_stream)
        lane.finalize()
        _, code = lane.read_stat()        # the reference's per-iteration shift readback
        if code:
            raise RuntimeError(f"device status {code}")
        lane.advance()

    for _ in range(warm):
        one(None, True)
    if pg is not None:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(lane.compute_stream)
    for i in range(steps):
        one(i, i + 1 < steps)
    e1.record(lane.compute_stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps,
                      sum(a.elapsed_time(b) for a, b in ar) / steps],
                     device=lane.dev, dtype=torch.float64)
    if pg is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    with torch.cuda.device(lane.dev):
        lane.copy_stream.synchronize()
        lane.compute_stream.synchronize()
    return float(t[0]), float(t[1])


def _largeN_point(cfg, rank, world, dev, pg, warm=2, steps=3, seed=4321):
    """Streamed and resident ms/iteration of kmeans_largeN's engine on the
    config (N partitioned over the ranks like kmeans_large.py:69-80)."""
    import torch
    import torch.distributed as dist
    from flash_kmeans import kmeans_large as kl
    N, D, K, BLOCK = cfg["N"], cfg["D"], cfg["K"], cfg["block"]
    _, ps, pe = kl.partition_blocks(N, BLOCK, world)
    p0, p1 = ps[rank], pe[rank]
    n = p1 - p0
    t0 = time.perf_counter()
    x_h = torch.empty((n, D), dtype=torch.float32, pin_memory=True)
    _fill_host_blocks(x_h, p0, BLOCK, seed, dev)
    c0 = torch.randn((1, K, D), generator=torch.Generator().manual_seed(seed + 7))
    setup_s = time.perf_counter() - t0
    flops = 2.0 * N * K * D
    out = {"workload": f"kmeans_largeN N={N} D={D} K={K} float32 BLOCK_N={BLOCK}",
           "points_per_rank": n, "host_setup_s": round(setup_s, 1)}

    # concurrent pinned H2D ceiling: every rank copies 1 GiB of its shard at once
    rows = min(n, (1 << 30) // (D * 4))
    dst = torch.empty((rows, D), dtype=torch.float32, device=dev)
    if pg is not None:
        dist.barrier()
    torch.cuda.synchronize()
    h0, h1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0.record()
    for _ in range(3):
        dst.copy_(x_h[:rows], non_blocking=True)
    h1.record()
    torch.cuda.synchronize()
    th = torch.tensor([h0.elapsed_time(h1) / 3], device=dev, dtype=torch.float64)
    if pg is not None:
        dist.all_reduce(th, op=dist.ReduceOp.MAX)
    del dst
    h2d_rank = rows * D * 4 / (float(th[0]) * 1e-3) / 1e9
    out["h2d_ceiling_gbs_per_rank"] = round(h2d_rank, 1)
    out["h2d_ceiling_gbs_total"] = round(h2d_rank * world, 1)

    for mode in ("streamed", "resident"):
        resident = mode == "resident"
        ok = torch.tensor([1.0 if (not resident or kl._fits_resident(dev, n, D, torch.float32))
                           else 0.0], device=dev)
        if pg is not None:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if float(ok[0]) == 0.0:
            out[mode] = {"skipped": "a rank's shard does not fit in half of its free HBM"}
            continue
        lane = kl._DeviceLane(dev, x_h[None], 0, n, BLOCK, K, D, torch.float32,
                              resident=resident)
        lane.set_centroids(c0)
        ms, ar_ms = _largeN_iters(lane, pg, warm, steps)
        rec = {"ms_per_iter": round(ms, 2), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
               "allreduce_ms_per_iter": round(ar_ms, 3) if world > 1 else 0.0}
        if not resident:
            rec["h2d_gbs_per_rank"] = round(n * D * 4 / (ms * 1e-3) / 1e9, 1)
            rec["frac_of_h2d_ceiling"] = round(n * D * 4 / (ms * 1e-3) / 1e9 / h2d_rank, 3)
        out[mode] = rec
        del lane
        torch.cuda.empty_cache()
    del x_h
    return out


def _largeN_parity(rank, world, dev, pg):
    """One kmeans_largeN iteration from the same centroids on 2^21 points:
    with several ranks (process group, NCCL all-reduce) against rank 0's
    single-GPU run of the whole set; on one GPU, streamed against resident.
    Labels must agree bit for bit; centroids to float-atomic rounding."""
    import torch
    import torch.distributed as dist
    from flash_kmeans import kmeans_large as kl
    P, Kp, D, Bp = 1 << 21, 1024, 128, 1 << 17
    cp = torch.randn((Kp, D), generator=torch.Generator().manual_seed(55))
    full = None
    if rank == 0:
        full = torch.empty((P, D), dtype=torch.float32, pin_memory=True)
        _fill_host_blocks(full, 0, Bp, 777, dev)
        lab1, cent1 = kl.kmeans_largeN(full, Kp, max_iters=1, tol=-1, BLOCK_N=Bp,
                                       init_centroids=cp, device=dev, resident=False)
    else:
        lab1 = torch.empty((P,), dtype=torch.int32, device=dev)
        cent1 = torch.empty((Kp, D), dtype=torch.float32, device=dev)
    if world > 1:
        _, ps, pe = kl.partition_blocks(P, Bp, world)
        shard = torch.empty((pe[rank] - ps[rank], D), dtype=torch.float32, pin_memory=True)
        _fill_host_blocks(shard, ps[rank], Bp, 777, dev)
        lab, cent = kl.kmeans_largeN(shard, Kp, max_iters=1, tol=-1, BLOCK_N=Bp,
                                     init_centroids=cp, process_group=pg, device=dev)
        dist.broadcast(lab1, 0)
        dist.broadcast(cent1, 0)
        ref = lab1[ps[rank]:pe[rank]]
        what = f"{world} ranks (process group) vs 1 GPU"
    else:
        lab, cent = kl.kmeans_largeN(full, Kp, max_iters=1, tol=-1, BLOCK_N=Bp,
                                     init_centroids=cp, device=dev, resident=True)
        ref = lab1
        what = "resident vs streamed, 1 GPU"
    mism = (lab != ref).sum().to(torch.float64)
    nrm = cent1.float().norm(dim=-1)
    rel = ((cent.float() - cent1.float()).norm(dim=-1) / torch.clamp(nrm, min=1e-3 * nrm.max())).max()
    t = torch.stack([mism, rel.to(torch.float64)])
    if world > 1:
        dist.all_reduce(t[:1])
        dist.all_reduce(t[1:], op=dist.ReduceOp.MAX)
    return {"check": what, "points": P, "K": Kp, "label_mismatches": int(t[0]),
            "centroid_max_rel_diff": float(t[1]), "ok": int(t[0]) == 0 and float(t[1]) <= 1e-5}


def _bind_to_gpu_cpus(dev):
    """Run this process on the CPUs NVML reports as local to its GPU, so that
    pinned host memory allocated afterwards lands on the GPU's NUMA node
    (first touch).  Returns the number of CPUs bound to, or None."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (os.cpu_count() + 63) // 64)
        cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1}
        cpus &= set(range(os.cpu_count()))
        if cpus:
            os.sched_setaffinity(0, cpus)
            return len(cpus)
    except Exception:
        pass
    return None


def large_n_record(rank, world, dev):
    """The out-of-core record of the default bench line (see the module
    docstring); every rank takes part, rank 0's dict is printed.  With several
    ranks each binds to its GPU's local CPUs first (host-memory placement)."""
    import torch.distributed as dist
    pg = dist.group.WORLD if world > 1 else None
    bound = _bind_to_gpu_cpus(dev) if world > 1 else None
    rec = {"config5": _largeN_point(LARGE_N, rank, world, dev, pg),
           "rank0_cpus_bound": bound}
    rec["parity"] = _largeN_parity(rank, world, dev, pg)
    rec["config5_2e28"] = _largeN_big(rank, world, dev, pg)
    rec["note"] = ("speed-up over 1 GPU = ms_per_iter at N=1 / ms_per_iter here (the N=1 line "
                   "of the same bench carries it)")
    return rec


def _largeN_big(rank, world, dev, pg):
    """The 2^28-point scaling point (K=16384): 128 GiB of float32 host data,
    run when there are at least 4 ranks and the node has the host memory."""
    import torch
    import torch.distributed as dist
    need = LARGE_N_BIG["N"] * LARGE_N_BIG["D"] * 4
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:
        avail = 0
    go = torch.tensor([1.0 if (world >= 4 and avail > 1.25 * need) else 0.0], device=dev)
    if pg is not None:
        dist.broadcast(go, 0)
    if float(go[0]) == 0.0:
        return {"skipped": (f"needs >= 4 GPUs and {1.25 * need / 2**30:.0f} GiB of free host "
                            f"memory; this run: {world} GPU(s), {avail / 2**30:.0f} GiB free")}
    return _largeN_point(LARGE_N_BIG, rank, world, dev, pg, warm=1, steps=2)


def run_assign(args, rank, world, local_rank):
    """`--op assign`: K timed calls of euclid_assign_triton on resident inputs."""
    import torch
    import torch.distributed as dist
    from flash_kmeans import _ops
    from flash_kmeans.assign_euclid_triton import euclid_assign_triton

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    x, c0 = _make_inputs(w, dev, seed=1234 + rank)
    x_sq = _ops.row_sqnorm(x)
    out = torch.empty((w["B"], w["N"]), dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        euclid_assign_triton(x, c0, x_sq, out=out)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record()
        for _ in range(args.steps):
            euclid_assign_triton(x, c0, x_sq, out=out)
        e1.record()
        torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    flops = _flops(w)
    achieved = flops / (ms * 1e-3) / 1e12
    burst, sustained, hbm, src = _peaks()
    alg_bytes = sum(t.numel() * t.element_size() for t in (x, x_sq, c0, out))
    hbm_bound = _hbm_bound(alg_bytes, flops, burst, hbm)
    if rank == 0:
        print(json.dumps({
            "metric": "assign TFLOP/s (euclid_assign_triton, labels only)",
            "value": round(achieved * world, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16" if w["dtype"] == "float16" else w["dtype"],
            "data": "synthetic (seeded torch generator; shapes/distribution of the BASELINE config)",
            "config": {"workload": _describe(args.workload, w),
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "step": "one euclid_assign_triton call (c_sq staging + assignment)"},
            "roofline": _roofline(hbm_bound, achieved, alg_bytes, ms, burst, sustained, hbm, src,
                                  _load_traffic(f"plain_{args.workload}")),
            "gpu_launches": 2 * args.steps,
            "clocks": clk.summary(),
        }), flush=True)


def run_large(args, rank, world, local_rank):
    """cfg5: kmeans_largeN's streaming engine; one step = one Lloyd iteration over all N
    points (every rank streams its contiguous shard from pinned host memory, partial sums
    are all-reduced over NCCL, each rank finalizes its replica)."""
    import torch
    import torch.distributed as dist
    from flash_kmeans import kmeans_large as kl

    w = WORKLOADS[args.workload]
    N, D, K, BLOCK = w["N"], w["D"], w["K"], w["block"]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    pg = dist.group.WORLD if world > 1 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_runner(w)
    _, ps, pe = kl.partition_blocks(N, BLOCK, world)
    p0, p1 = ps[rank], pe[rank]
    n = p1 - p0
    # this rank's shard: x ~ N(0,1) generated on the GPU, kept in pinned host memory
    x_h = torch.empty((n, D), dtype=torch.float32, pin_memory=True)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    for a in range(0, n, BLOCK):
        b = min(n, a + BLOCK)
        x_h[a:b].copy_(torch.randn((b - a, D), device=dev, generator=g))
    torch.cuda.synchronize()
    gc = torch.Generator().manual_seed(99)
    c0 = x_h[torch.randint(0, n, (K,), generator=gc)].to(dev)
    if world > 1:
        kl.broadcast_centroids(c0, None)

    # as kmeans_largeN: keep the shard resident in HBM after the first pass when it fits
    resident = not args.stream and kl._fits_resident(dev, n, D, torch.float32)
    lane = kl._DeviceLane(dev, x_h[None], 0, n, BLOCK, K, D, torch.float32, resident=resident)
    lane.set_centroids(c0[None])

    def one_iter(wrap):
        lane.run_pass(wrap=wrap)
        kl._allreduce([lane], pg)
        lane.finalize()
        _, code = lane.read_stat()  # the reference's per-iteration shift readback
        if code:
            raise RuntimeError(f"device status {code}")
        lane.advance()

    for _ in range(args.warmup):
        one_iter(True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev) as clk:
        e0.record(lane.compute_stream)
        for i in range(args.steps):
            one_iter(i + 1 < args.steps)
        e1.record(lane.compute_stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t[0])
    flops = 2.0 * N * K * D
    value = flops / (ms * 1e-3) / 1e12
    burst, sustained, hbm, src = _peaks()
    with torch.cuda.device(dev):
        lane.copy_stream.synchronize()
        lane.compute_stream.synchronize()
    del lane
    torch.cuda.empty_cache()

    # e2e: the public entry point on the same host shard, labels copied back
    e2e = None
    if args.e2e_steps > 0:
        iters = args.e2e_steps
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        f0 = time.perf_counter()
        kw = dict(process_group=pg, device=dev) if world > 1 else dict(device=dev)
        labels, cent = kl.kmeans_largeN(x_h, K, max_iters=iters, tol=-1, BLOCK_N=BLOCK,
                                        init_centroids=c0.cpu(), **kw)
        labels_h = labels.cpu()
        torch.cuda.synchronize()
        secs = time.perf_counter() - f0
        tt = torch.tensor([secs], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e = {"value": round(flops * iters / float(tt[0]) / 1e12, 3), "unit": UNIT,
               "h2d_bytes_per_step": int(n * D * 4), "d2h_bytes_per_step": int(labels_h.numel() * 4 / iters),
               "step": f"kmeans_largeN(max_iters={iters}) per rank on its pinned host shard, "
                       "labels copied back; wall clock incl. set-up, max over ranks"}

    cpu_baseline = None
    if cpu is not None:
        cpu.step(seed=99)
        secs = cpu.step(seed=7)
        cpu_baseline = {"value": round(cpu.tflops(secs), 5), "unit": UNIT, "cores": cpu.cores,
                        "kind": cpu.kind, "sample": cpu.sample()}
        cpu.close()
    bytes_rank = n * D * 4
    if resident:   # 3xTF32: three tf32 MMAs per useful one, tf32 at half the bf16 rate
        roof = {"bound": "tensor", "achieved": round(value / world, 2),
                "peak": round(burst / 6, 1), "unit": UNIT,
                "frac": round(value / world / (burst / 6), 4),
                "peak_source": f"{src} dense bf16 (burst) / 2 (tf32 rate) / 3 (3xTF32), per GPU",
                "traffic": None}
    else:
        roof = {"bound": "pcie_h2d", "achieved": round(bytes_rank / (ms * 1e-3) / 1e9, 1),
                "peak": None, "unit": "GB/s", "frac": None,
                "peak_source": "no measured H2D peak in MEASURED_PEAKS.json; the default "
                               "bench's large_n record measures the ranks' concurrent ceiling",
                "traffic": None}
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32(3xTF32)", "data": "synthetic (x ~ N(0,1) from a seeded torch generator, "
                                            "pinned host memory)",
            "config": {"workload": f"{args.workload}: kmeans_largeN N={N} D={D} K={K} float32, "
                                   f"BLOCK_N={BLOCK}",
                       "parallelism": f"N partitioned over {world} ranks, NCCL all-reduce of "
                                      "K*D sums + K counts per iteration",
                       "l2": ("x copied from host once, then resident in HBM (GBs per rank, > L2)"
                              if resident else
                              "x streamed from host every iteration (GBs per rank); no flush"),
                       "step": ("one Lloyd iteration from the HBM-resident shard incl. the "
                                "shift readback" if resident else
                                "one Lloyd iteration streamed from pinned host memory incl. the "
                                "shift readback")},
            "roofline": roof,
            "e2e": e2e, "cpu_baseline": cpu_baseline,
            # per block: c_sq staging, assignment, scan, scatter, segmented sum; per
            # iteration: finalize (float32 rows with K*D too large for shared memory)
            "gpu_launches": args.steps * (5 * ((n + BLOCK - 1) // BLOCK) + 1),
            "clocks": clk.summary(),
        }), flush=True)


# ------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """The reference's own CPU implementation of the path on the host cores
    (rank 0 only under torchrun): torch_fallback's Lloyd iteration from the
    reference installed under baseline/_ref, all host threads, on a bounded
    sample of the workload per step; the numpy restatement if not installed."""
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    cpu = cpu_baseline_runner(w)
    for s_ in range(args.warmup):
        cpu.step(seed=s_)
    times = [cpu.step(seed=100 + s_) for s_ in range(args.steps)]
    cpu.close()
    secs = sum(times) / len(times)
    v = round(cpu.tflops(secs), 5)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": v, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs * 1e3, 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": _describe(args.workload, w)},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": cpu.cores, "kind": cpu.kind,
                         "sample": cpu.sample()},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg2")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--op", choices=["lloyd", "assign"], default="lloyd")
    ap.add_argument("--metric", choices=["euclid", "cosine", "dot"], default="euclid")
    ap.add_argument("--no-large-n", action="store_true",
                    help="default workload: skip the out-of-core (config 5) record")
    ap.add_argument("--stream", action="store_true",
                    help="cfg5: stream x from host every iteration even when it fits in HBM")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if WORKLOADS[args.workload].get("large"):
            run_large(args, rank, world, local_rank)
        else:
            (run_assign if args.op == "assign" else run_ours)(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
