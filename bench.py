"""Benchmark of the isotonic-regression hot path on B200: fitted elements/s and HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (one rank per GPU, rows sharded)

A step is one fit of one batch of synthetic input (the configs of the reference's benchmark
grid and calibration example; seeded, generated on the device). The headline workload is the
short-row batch: y float32 [1,000,000, 16] = -0.1 i + N(0, 0.5), unweighted, decreasing,
exact=True, forward only. Batch rows are sharded across ranks with no collective in the data
path (weak scaling: every rank fits its own [1e6, 16]).

value: elements/s of the whole job, the fused fit kernel called through the C ABI on inputs
resident in HBM; input/output sets rotate so that consecutive steps never hit in L2.
e2e: the same metric through the public API torchisotonic_b200.isotonic, with each step's input
copied from pinned host memory and its fitted output read back.

configs (default; --headline-only drops it): every config c1, c2, c2_fast, c3, c4, c5 -
forward, and forward + backward where the config has a gradient, through the C ABI (device
time, with the roofline of the step) and through the public API with autograd; at one GPU also
the reference's own CUDA operators on the same inputs (built from its sources into oracle/_ref
by oracle/ref_cuda.py, driven by the steps of its public API) with the rows whose block
partition equals ours, and the reference's CPU solver on the host (a bounded sample). At N > 1
GPUs c4, one row, is split into N segments instead (`c4_split`, strong scaling).

The reference arm (--impl reference) times the reference's own CPU solver (its pava.h,
compiled into oracle/_ref, all host threads) on the same workload.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "fitted elements/s and HBM GB/s vs peak, fwd and fwd+bwd, at 1/2/4/8 B200"
UNIT = "elements/s"


# ---------------------------------------------------------------------------------------------
# workloads (the reference benchmark's configs; the same recipes as tests/test_fit_gpu.py)

def config(name: str, device: torch.device, seed: int = 0, batch: int | None = None) -> dict:
    """The workload `name`; `batch` (profiling only) overrides its number of rows."""
    g = torch.Generator(device=device).manual_seed(seed)
    if name == "c1":
        y = 0.001 * torch.arange(5000, device=device) + torch.randn(batch or 1000, 5000, generator=g,
                                                                     device=device)
        return dict(name="c1", desc="y float32 [1000, 5000] = 0.001 i + N(0,1), unweighted, "
                    "increasing, exact", y=y, w=None, increasing=True, exact=True,
                    y_min=None, y_max=None, grad=False)
    if name in ("c2", "c2_fast"):
        y = -0.1 * torch.arange(16, device=device) + 0.5 * torch.randn(batch or 1_000_000, 16, generator=g,
                                                                        device=device)
        return dict(name=name, desc="y float32 [1000000, 16] = -0.1 i + N(0,0.5), unweighted, "
                    f"decreasing, exact={name == 'c2'}", y=y, w=None, increasing=False,
                    exact=name == "c2", y_min=None, y_max=None, grad=False)
    if name == "c3":
        n, b = 65536, batch or 4096
        y = torch.sigmoid(torch.linspace(-4, 4, n, dtype=torch.float64, device=device)
                          + torch.randn(b, n, generator=g, dtype=torch.float64, device=device))
        w = torch.empty(b, n, dtype=torch.float64, device=device).exponential_(1.0, generator=g)
        w += 0.1
        rows = (torch.rand(b, generator=g, device=device) < 0.01).nonzero().squeeze(1)
        cols = torch.randint(n, (len(rows),), generator=g, device=device)
        y[rows, cols] = math.nan
        return dict(name="c3", desc="y float64 [4096, 65536] = sigmoid(linspace(-4,4) + N(0,1)), "
                    "w = Exp(1) + 0.1, ~1% NaN rows, clip [0, 1], fwd+bwd", y=y, w=w,
                    increasing=True, exact=True, y_min=0.0, y_max=1.0, grad=True)
    if name == "c4":
        n = 100_000_000
        z = torch.randn(n, generator=g, device=device).sort().values
        w = 1 + torch.poisson(torch.full((n,), 0.5, device=device), generator=g)
        y = torch.binomial(w, torch.sigmoid(3 * z), generator=g) / w
        return dict(name="c4", desc="one row of 1e8 float32 calibration means, w = 1 + "
                    "Poisson(0.5), increasing", y=y[None].float(), w=w[None].float(),
                    increasing=True, exact=True, y_min=None, y_max=None, grad=True)
    if name == "c5":
        b = batch or 65536
        base = (torch.cumsum(0.1 + torch.randn(b, 64, generator=g, device=device), 1)
                + 0.3 * torch.randn(b, 64, generator=g, device=device))
        ragged = torch.rand(b, generator=g, device=device) < 0.1
        lengths = torch.randint(16, 64, (b,), generator=g, device=device)
        pos = torch.arange(64, device=device)[None]
        pad = ragged[:, None] & (pos >= lengths[:, None])
        rowmax = torch.where(pos < lengths[:, None], base,
                             torch.tensor(-math.inf, device=device)).amax(1)
        base = torch.where(pad, (rowmax + 1)[:, None].expand(-1, 64), base)
        w = 0.1 + torch.rand(b, 64, generator=g, device=device)
        return dict(name="c5", desc="y bfloat16 [65536, 64] quantile head, w float32, "
                    "10% ragged rows, fwd+bwd", y=base.bfloat16(), w=w, increasing=True,
                    exact=True, y_min=None, y_max=None, grad=True,
                    lengths=torch.where(ragged, lengths, torch.full_like(lengths, 64)))
    raise ValueError(name)


def fwd_bytes(cfg: dict, with_starts: bool) -> int:
    y, w = cfg["y"], cfg["w"]
    b = y.numel() * y.element_size() * 2  # y in, out written
    if w is not None:
        b += w.numel() * w.element_size()
    if with_starts:
        b += y.numel()
    return b


def bwd_bytes(cfg: dict) -> int:
    """Reads starts, g, [w], [y]; writes grad_y and [grad_w] (the reference's isotonic_grad
    signature; the fit is recomputed from y and w rather than read)."""
    y, w = cfg["y"], cfg["w"]
    b = y.numel() * (1 + 2 * y.element_size())
    if w is not None:
        b += 2 * w.numel() * w.element_size() + y.numel() * y.element_size()
    return b


# ---------------------------------------------------------------------------------------------
# the C ABI call with preallocated buffers (the device-timed value)

class Fitter:
    """tiso_fit through the C ABI on preallocated buffers, `sets` input/output sets in turn."""

    def __init__(self, cfg: dict, with_starts: bool = False, sets: int = 1):
        from torchisotonic_b200 import _ext

        self.ext = _ext
        self.so = _ext.lib()
        y = cfg["y"]
        self.cfg = cfg
        self.dtype = _ext._DTYPES[y.dtype]
        self.flags = (_ext.INCREASING if cfg["increasing"] else 0) | (
            _ext.EXACT if cfg["exact"] else 0)
        self.flags |= (_ext.CLIP_LO if cfg["y_min"] is not None else 0)
        self.flags |= (_ext.CLIP_HI if cfg["y_max"] is not None else 0)
        self.batch, self.n = y.shape
        self.ys = [y] + [y.clone() for _ in range(sets - 1)]
        self.ws = [cfg["w"]] + [None if cfg["w"] is None else cfg["w"].clone()
                                for _ in range(sets - 1)]
        self.outs = [torch.empty_like(y) for _ in range(sets)]
        self.starts = [torch.empty(y.shape, dtype=torch.bool, device=y.device)
                       if with_starts else None for _ in range(sets)]
        size = ctypes.c_size_t()
        self.so.tiso_fit_workspace_size(self.dtype, int(cfg["w"] is not None), self.batch, self.n,
                                        self.flags, ctypes.byref(size))
        self.ws_bytes = size.value
        self.work = (torch.empty(size.value, dtype=torch.uint8, device=y.device)
                     if size.value else None)
        self.stream = torch.cuda.current_stream().cuda_stream

    def __call__(self, k: int = 0) -> None:
        i = k % len(self.ys)
        rc = self.so.tiso_fit(self.dtype, _p(self.ys[i]), _p(self.ws[i]), _p(self.outs[i]),
                              _p(self.starts[i]), self.batch, self.n, self.flags,
                              float(self.cfg["y_min"] or 0.0), float(self.cfg["y_max"] or 0.0),
                              None, _p(self.work), self.ws_bytes, self.stream)
        if rc:
            raise RuntimeError(self.so.tiso_last_error().decode())


class FitGrad:
    """A forward with block starts and the backward (d/dy and, weighted, d/dw of sum(fit * g)),
    both through the C ABI on preallocated buffers: tiso_fit then tiso_grad."""

    def __init__(self, cfg: dict, g: torch.Tensor, sets: int = 1):
        from torchisotonic_b200 import _ext

        self.fit = Fitter(cfg, with_starts=True, sets=sets)
        self.so = self.fit.so
        y, w = cfg["y"], cfg["w"]
        self.gs = [g] + [g.clone() for _ in range(sets - 1)]
        self.gys = [torch.empty_like(y) for _ in range(sets)]
        self.gws = [None if w is None else torch.empty_like(w) for _ in range(sets)]
        self.gflags = (_ext.WANT_GRAD_W if w is not None else 0) | (
            self.fit.flags & (_ext.CLIP_LO | _ext.CLIP_HI))
        self.need_y = w is not None or cfg["y_min"] is not None or cfg["y_max"] is not None
        size = ctypes.c_size_t()
        self.so.tiso_grad_workspace_size(self.fit.dtype, int(w is not None), self.fit.batch,
                                         self.fit.n, self.gflags, ctypes.byref(size))
        self.ws_bytes = size.value
        self.work = (torch.empty(size.value, dtype=torch.uint8, device=y.device)
                     if size.value else None)

    def __call__(self, k: int = 0) -> None:
        f = self.fit
        f(k)
        i = k % len(f.ys)
        rc = self.so.tiso_grad(f.dtype, _p(f.ys[i]) if self.need_y else None, _p(f.ws[i]),
                               _p(f.starts[i]), _p(self.gs[i]), _p(self.gys[i]), _p(self.gws[i]),
                               f.batch, f.n, self.gflags, float(f.cfg["y_min"] or 0.0),
                               float(f.cfg["y_max"] or 0.0), _p(self.work), self.ws_bytes,
                               f.stream)
        if rc:
            raise RuntimeError(self.so.tiso_last_error().decode())


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def fit_kernel_name(n: int, batch: int = 1, weighted: bool = False, f64: bool = False) -> str:
    """What a forward step launches for rows of n elements: one short-row or whole-row kernel,
    or (long rows) the tile, tree-merge and expand kernels, reported together as the step."""
    if n <= 32:
        return "short_rows_kernel" if (weighted or f64) else "short_rows_u_kernel"
    return "fit_tile_kernel" if n <= 512 else "fit_step"


def fit_launches(n: int, batch: int) -> int:
    """Our kernel launches per forward call: one for rows of up to 512 elements (the short-row
    kernel up to 32, the tile kernel's whole-row mode above); longer rows take the tile kernel,
    a kernel for the tree of tile merges (when a row has more than one tile) and the expand
    kernel. Tiles of 2048 for many rows of few tiles, else of 512, as csrc/tiso.cu plan_fit
    decides."""
    if n <= 512:
        return 1
    tiles512 = (n + 511) // 512
    levels = max(0, math.ceil(math.log2(tiles512)))
    few = levels >= 12 or batch * tiles512 <= 65536
    tiles = (n + 2047) // 2048 if (few and batch >= 512) else tiles512
    return 3 if tiles > 1 else 2


def grad_launches(n: int) -> int:
    """Backward launches: one for rows of up to 1024 elements; else the tile kernel twice around
    the scan of tile sums (one launch, or three for rows of more than 1024 tiles)."""
    if n <= 1024:
        return 1
    return 3 if (n + 1023) // 1024 <= 1024 else 5


def time_steps(fn, steps: int, warmup: int) -> tuple[float, list[float]]:
    """Total device seconds of `steps` calls after `warmup`, with per-step event times (CUDA
    events on the current stream, which the C ABI calls launch on)."""
    for k in range(warmup):
        fn(k)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for k in range(steps):
        evs[k][0].record()
        fn(k)
        evs[k][1].record()
    end.record()
    torch.cuda.synchronize()
    per = [a.elapsed_time(b) / 1e3 for a, b in evs]
    return start.elapsed_time(end) / 1e3, per


def timed(fn, steps: int, warmup: int, world: int) -> tuple[float, float]:
    """(max over ranks of the total seconds of `steps` calls, this rank's median step seconds),
    between barriers on every rank."""
    barrier(world)
    total, per = time_steps(fn, steps, warmup)
    barrier(world)
    return max_over_ranks(total, world), statistics.median(per)


API_STEPS = 50  # at least this many steps for the host-bound public-API arms (ours, reference)


def api_ms(fn, steps: int, warmup: int, world: int) -> float:
    """A public-API step in ms: the median of per-step device times over at least API_STEPS
    steps (the same statistic for our API and the reference's; their steps are host-bound, and a
    median over many steps keeps one slow host step from moving the figure)."""
    _, med = timed(fn, max(steps, API_STEPS), warmup, world)
    return 1e3 * med


def rotating_sets(step_bytes: int) -> int:
    """Input/output sets taken in turn so that a step never finds the data of the step before it
    in the 126 MB L2: enough for twice the L2, at most 8 (1 when a step moves more than that)."""
    return max(1, min(8, math.ceil(2 * 126e6 / max(step_bytes, 1))))


# ---------------------------------------------------------------------------------------------
# clocks during the timed region

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        busy = [s for s in sm if s >= 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------------------------


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def traffic_of(kernel: str, workload: str) -> float | None:
    """DRAM bytes per launch of the kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(f"{kernel}:{workload}")


def cpu_reference(cfg: dict, budget_s: float) -> dict | None:
    """The reference's own CPU solver (oracle/_ref, its pava.h) on the workload: elements/s with
    all host threads (rows in parallel, as its ops.cpp:30; a single row runs on one core). A
    bounded sample: whole fits of the workload until budget_s has passed (at least one)."""
    sys.path.insert(0, str(ROOT))
    import oracle

    if oracle.ref_lib() is None:
        return None
    y = cfg["y"].float().cpu().numpy() if cfg["y"].dtype != torch.float64 else cfg["y"].cpu().numpy()
    w = None if cfg["w"] is None else cfg["w"].to(torch.float64 if y.dtype == np.float64
                                                   else torch.float32).cpu().numpy()
    threads = os.cpu_count() or 1
    done, runs, t0 = 0, 0, time.perf_counter()
    while True:
        oracle.ref_fit(y, w, increasing=cfg["increasing"], threads=threads)
        runs += 1
        done += y.size
        if time.perf_counter() - t0 >= budget_s or runs >= 50:
            break
    dt = time.perf_counter() - t0
    used = min(threads, y.shape[0])
    return {"value": done / dt, "unit": UNIT, "cores": used, "kind": "reference",
            "ms_per_fit": 1e3 * dt / runs,
            "sample": f"{runs} full fit(s) of the {cfg['name']} workload ({y.size} elements "
                      f"each) by the reference's pava.h, rows over {used} host thread(s)"}


# ---------------------------------------------------------------------------------------------
# the reference's own CUDA operators (built from its sources by oracle/ref_cuda.py), driven the
# way its public API drives them; for the comparison in the bench line only

def ref_cuda_ops():
    sys.path.insert(0, str(ROOT))
    try:
        from oracle import ref_cuda

        return ref_cuda.load()
    except (OSError, RuntimeError, ImportError):
        return None


class _RefIsotonic(torch.autograd.Function):
    """The reference's autograd step (src/torchisotonic/_api.py:73-97) over its own operators:
    the fit with block starts when a gradient is wanted, the backward by its isotonic_grad."""

    @staticmethod
    def forward(ctx, ops, flat_y, flat_w, increasing, exact):
        need = any(ctx.needs_input_grad[1:3])
        out, starts = ops.isotonic_tiles(flat_y.contiguous(),
                                         None if flat_w is None else flat_w.contiguous(),
                                         increasing, exact, need)
        ctx.save_for_backward(flat_y, flat_w, out, starts)
        ctx.ops = ops
        return out

    @staticmethod
    def backward(ctx, grad):
        flat_y, flat_w, out, starts = ctx.saved_tensors
        want_w = ctx.needs_input_grad[2]
        gy, gw = ctx.ops.isotonic_grad(out, starts, grad, flat_w, flat_y if want_w else None)
        return (None, gy if ctx.needs_input_grad[1] else None, gw if want_w else None, None,
                None)


def ref_isotonic(ops, y, weight, increasing, y_min, y_max, exact):
    """The steps of the reference's isotonic() on [batch, n] rows (src/torchisotonic/_api.py:43-70):
    the weight check with its host synchronisation, the cast to the accumulation dtype, the
    operator, the clamp and the cast back, each as the reference runs them."""
    out_dtype = y.dtype
    acc = torch.float64 if out_dtype == torch.float64 else torch.float32
    w = None
    if weight is not None:
        w = weight.to(device=y.device, dtype=acc).broadcast_to(y.shape)
        if not bool((w > 0).all()):
            raise ValueError("weight must be strictly positive")
    flat_y = y.reshape(-1, y.shape[-1]).to(acc)
    flat_w = None if w is None else w.reshape(-1, y.shape[-1])
    out = _RefIsotonic.apply(ops, flat_y, flat_w, increasing, exact)
    if y_min is not None or y_max is not None:
        out = out.clamp(min=y_min, max=y_max)
    return out.reshape(y.shape).to(out_dtype)


def measure_reference_cuda(ops, cfg: dict, g: torch.Tensor | None, ours_starts: torch.Tensor,
                           steps: int, warmup: int, sets: int) -> dict:
    """The reference's CUDA path on the same inputs: its operator alone (forward), its public
    API's steps around it (forward; forward + backward through autograd), and how many rows get
    the same block partition as ours (rows holding a NaN left out: the reference's multi-chunk
    kernels leave their starts unwritten)."""
    y, w = cfg["y"], cfg["w"]
    acc = torch.float64 if y.dtype == torch.float64 else torch.float32
    kw = (cfg["increasing"], cfg["y_min"], cfg["y_max"], cfg["exact"])
    ys = [y] + [y.clone() for _ in range(sets - 1)]
    ws = [w] + [None if w is None else w.clone() for _ in range(sets - 1)]
    ya = [t.to(acc).contiguous() for t in ys]
    res = {}
    _, t = timed(lambda k: ops.isotonic_tiles(ya[k % sets], ws[k % sets], cfg["increasing"],
                                              cfg["exact"], False), steps, warmup, 1)
    res["op_fwd_ms"] = 1e3 * t
    res["fwd_ms"] = api_ms(lambda k: ref_isotonic(ops, ys[k % sets], ws[k % sets], *kw), steps,
                           warmup, 1)
    if cfg["grad"]:
        yg = [t.clone().requires_grad_() for t in ys]
        wg = [t.clone().requires_grad_() for t in ws]

        def fb(k: int) -> None:
            i = k % sets
            yg[i].grad = None
            wg[i].grad = None
            ref_isotonic(ops, yg[i], wg[i], *kw).backward(g)

        res["fwd_bwd_ms"] = api_ms(fb, max(3, steps // 2), warmup, 1)
    _, st = ops.isotonic_tiles(ya[0], ws[0], cfg["increasing"], cfg["exact"], True)
    ok = ~torch.isnan(y).any(1) if y.dtype.is_floating_point else torch.ones(y.shape[0], dtype=torch.bool, device=y.device)
    same = (st == ours_starts).all(1)
    res["rows_compared"] = int(ok.sum())
    res["rows_same_partition"] = int((same & ok).sum())
    del ys, ws, ya
    return res


# ---------------------------------------------------------------------------------------------


def dist_init(gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world > 1:
        import datetime

        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def roofline(kernel: str, name: str, alg: float, seconds: float) -> dict:
    peak, peak_kind = peaks()
    achieved = alg / seconds / 1e9
    return {"bound": "hbm", "kernel": kernel, "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes_per_launch": alg, "traffic": traffic_of(kernel, name)}


def measure_config(name: str, dev: torch.device, args, rank: int, world: int, ref_ops) -> dict:
    """One config, rows sharded (every rank fits its own batch; weak scaling): the forward and,
    where the config has a gradient, forward + backward, through the C ABI (device time, max
    over ranks) and through the public API with autograd; at one GPU also the reference's CUDA
    operator on the same inputs and its CPU solver on the host."""
    import torchisotonic_b200

    cfg = config(name, dev, seed=rank, batch=args.configs_batch)
    y, w = cfg["y"], cfg["w"]
    batch, n = y.shape
    el = y.numel()
    steps, warmup = args.steps, args.warmup
    kname = fit_kernel_name(n, batch, w is not None, y.dtype == torch.float64)
    res = {"workload": cfg["desc"], "shape": [batch, n], "per_gpu_elements": el,
           "parallelism": f"rows sharded x{world}"}

    alg = fwd_bytes(cfg, False)
    sets = rotating_sets(alg)
    fitter = Fitter(cfg, sets=sets)
    tot, med = timed(fitter, steps, warmup, world)
    res["fwd"] = {"ms": 1e3 * tot / steps, "elements_per_s": world * el * steps / tot,
                  "gb_per_s": world * alg * steps / tot / 1e9,
                  "roofline": roofline(kname, name, alg, med),
                  "gpu_launches_per_step": fit_launches(n, batch),
                  "l2": f"{sets} rotating sets" if sets > 1 else "inputs larger than L2"}
    del fitter

    kw = dict(increasing=cfg["increasing"], exact=cfg["exact"], y_min=cfg["y_min"],
              y_max=cfg["y_max"])
    api_sets = rotating_sets(alg)
    ys = [y] + [y.clone() for _ in range(api_sets - 1)]
    wsl = [w] + [None if w is None else w.clone() for _ in range(api_sets - 1)]
    res["api_fwd_ms"] = api_ms(
        lambda k: torchisotonic_b200.isotonic(ys[k % api_sets], wsl[k % api_sets], **kw),
        steps, warmup, world)

    g = None
    if cfg["grad"]:
        g = torch.randn(y.shape, device=dev,
                        generator=torch.Generator(device=dev).manual_seed(7)).to(y.dtype)
        fb_alg = fwd_bytes(cfg, True) + bwd_bytes(cfg)
        fsets = rotating_sets(fb_alg)
        fg = FitGrad(cfg, g, sets=fsets)
        fb_steps = max(3, steps // 2)
        tot, med = timed(fg, fb_steps, warmup, world)
        res["fwd_bwd"] = {"ms": 1e3 * tot / fb_steps,
                          "elements_per_s": world * el * fb_steps / tot,
                          "gb_per_s": world * fb_alg * fb_steps / tot / 1e9,
                          "roofline": roofline("fwd_bwd_step", name, fb_alg, med),
                          "gpu_launches_per_step": fit_launches(n, batch) + grad_launches(n)}
        del fg
        yg = [t.clone().requires_grad_() for t in ys]
        wg = [None if t is None else t.clone().requires_grad_() for t in wsl]

        def fb(k: int) -> None:
            i = k % api_sets
            yg[i].grad = None
            if wg[i] is not None:
                wg[i].grad = None
            torchisotonic_b200.isotonic(yg[i], wg[i], **kw).backward(g)

        res["api_fwd_bwd_ms"] = api_ms(fb, fb_steps, warmup, world)
        del yg, wg
    del ys, wsl
    torch.cuda.empty_cache()

    if world == 1 and ref_ops is not None:
        from torchisotonic_b200 import _ext

        _, ours_st = _ext.isotonic_tiles(y, w, cfg["increasing"], cfg["exact"], True,
                                         cfg["y_min"], cfg["y_max"])
        rc = measure_reference_cuda(ref_ops, cfg, g, ours_st, steps, warmup, sets)
        del ours_st
        rc["speedup_fwd_api"] = rc["fwd_ms"] / res["api_fwd_ms"]
        if "fwd_bwd_ms" in rc:
            rc["speedup_fwd_bwd_api"] = rc["fwd_bwd_ms"] / res["api_fwd_bwd_ms"]
        res["reference_cuda"] = rc
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu:
        res["cpu_baseline"] = cpu_reference(cfg, budget_s=args.cpu_seconds)
    del cfg, y, w, g
    torch.cuda.empty_cache()
    return res


def measure_c5_varlen(dev: torch.device, args, rank: int, world: int) -> dict:
    """c5's rows packed at their own lengths (tiso_fit_varlen / tiso_grad_varlen: no padding
    read or written), forward and forward + backward, through the C ABI and the public API."""
    import torchisotonic_b200
    from torchisotonic_b200 import _ext

    cfg = config("c5", dev, seed=rank)
    lengths = cfg["lengths"]
    valid = torch.arange(64, device=dev)[None] < lengths[:, None]
    y = cfg["y"][valid].contiguous()
    w = cfg["w"][valid].contiguous()
    off = torch.zeros(lengths.numel() + 1, dtype=torch.int64, device=dev)
    off[1:] = torch.cumsum(lengths, 0)
    del cfg, valid
    el = y.numel()
    batch = lengths.numel()
    so = _ext.lib()
    stream = torch.cuda.current_stream().cuda_stream
    flags = _ext.INCREASING | _ext.EXACT
    alg = el * (2 + 4 + 2)  # y, w in; out written
    sets = rotating_sets(alg)
    ys = [y] + [y.clone() for _ in range(sets - 1)]
    ws = [w] + [w.clone() for _ in range(sets - 1)]
    outs = [torch.empty_like(y) for _ in range(sets)]
    sts = [torch.empty(y.shape, dtype=torch.bool, device=dev) for _ in range(sets)]
    g = torch.randn(y.shape, device=dev,
                    generator=torch.Generator(device=dev).manual_seed(7)).to(y.dtype)
    gs = [g] + [g.clone() for _ in range(sets - 1)]
    gys = [torch.empty_like(y) for _ in range(sets)]
    gws = [torch.empty_like(w) for _ in range(sets)]

    def fwd(k: int, starts: bool = False) -> None:
        i = k % sets
        rc = so.tiso_fit_varlen(_ext.BF16, ys[i].data_ptr(), ws[i].data_ptr(), outs[i].data_ptr(),
                                sts[i].data_ptr() if starts else None, off.data_ptr(), batch, 64,
                                flags, 0.0, 0.0, None, stream)
        if rc:
            raise RuntimeError(so.tiso_last_error().decode())

    def fb(k: int) -> None:
        fwd(k, True)
        i = k % sets
        rc = so.tiso_grad_varlen(_ext.BF16, ys[i].data_ptr(), ws[i].data_ptr(), sts[i].data_ptr(),
                                 gs[i].data_ptr(), gys[i].data_ptr(), gws[i].data_ptr(),
                                 off.data_ptr(), batch, 64, _ext.WANT_GRAD_W, 0.0, 0.0, stream)
        if rc:
            raise RuntimeError(so.tiso_last_error().decode())

    steps, warmup = args.steps, args.warmup
    tot, med = timed(fwd, steps, warmup, world)
    fb_alg = alg + el + el * (2 + 1 + 2 + 4 + 2 + 2 + 4)
    fb_steps = max(3, steps // 2)
    tot2, med2 = timed(fb, fb_steps, warmup, world)
    yg, wg = y.clone().requires_grad_(), w.clone().requires_grad_()

    def api_fb(k: int) -> None:
        yg.grad = None
        wg.grad = None
        torchisotonic_b200.isotonic_varlen(yg, off, wg, max_len=64).backward(g)

    api_f = api_ms(lambda k: torchisotonic_b200.isotonic_varlen(ys[k % sets], off, ws[k % sets],
                                                                max_len=64), steps, warmup, world)
    api_b = api_ms(api_fb, fb_steps, warmup, world)
    res = {"workload": "c5's rows packed at their own lengths (offsets, no padding): y bfloat16, "
                       "w float32, fwd+bwd", "rows": batch, "per_gpu_elements": el,
           "parallelism": f"rows sharded x{world}",
           "fwd": {"ms": 1e3 * tot / steps, "elements_per_s": world * el * steps / tot,
                   "roofline": roofline("fit_tile_kernel", "c5_varlen", alg, med),
                   "gpu_launches_per_step": 1},
           "fwd_bwd": {"ms": 1e3 * tot2 / fb_steps,
                       "elements_per_s": world * el * fb_steps / tot2,
                       "roofline": roofline("fwd_bwd_step", "c5_varlen", fb_alg, med2),
                       "gpu_launches_per_step": 2},
           "api_fwd_ms": api_f, "api_fwd_bwd_ms": api_b}
    del ys, ws, outs, sts, gs, gys, gws, yg, wg
    torch.cuda.empty_cache()
    return res


CONFIGS = ("c1", "c2", "c2_fast", "c3", "c4", "c5")


def measure_configs(dev: torch.device, args, rank: int, world: int) -> dict:
    """Every config of the benchmark (c1..c5, c2 in both precisions, c5 packed at its rows'
    lengths; or those --configs names); at N > 1 GPUs c4, a single row, is split into N
    segments instead of sharded (strong scaling: `c4_split`)."""
    ref_ops = ref_cuda_ops() if (world == 1 and not args.no_ref) else None
    wanted = CONFIGS + ("c5_varlen",) if not args.configs else tuple(args.configs.split(","))
    res = {}
    for name in wanted:
        if name == "c4" and world > 1:
            res["c4_split"] = measure_split(args, rank, world, dev)
        elif name == "c5_varlen":
            res["c5_varlen"] = measure_c5_varlen(dev, args, rank, world)
        else:
            res[name] = measure_config(name, dev, args, rank, world, ref_ops)
    if world == 1 and ref_ops is None and not args.no_ref:
        res["reference_cuda"] = ("unavailable: oracle/_ref/ref_cuda was not built "
                                 "(python oracle/ref_cuda.py <reference checkout>)")
    return res


def run_ours(args, rank: int, world: int, local: int) -> None:
    """The headline (the short-row batch, c2: y float32 [1e6, 16] decreasing, exact, forward;
    rows sharded) and, unless --headline-only, every config."""
    import torchisotonic_b200

    dev = torch.device("cuda", local)
    cfg = config(args.config, dev, seed=rank, batch=args.batch)
    elements = cfg["y"].numel()
    alg = fwd_bytes(cfg, False)
    sets = rotating_sets(alg)
    fitter = Fitter(cfg, with_starts=False, sets=sets)
    nlaunch = fit_launches(cfg["y"].shape[1], cfg["y"].shape[0])

    # clock warm-up: idle GPUs run slow at first
    torch.cuda._sleep(500_000_000)
    clocks = Clocks(local)
    t_max, med = timed(fitter, args.steps, args.warmup, world)
    clk = clocks.stop()
    value = world * elements * args.steps / t_max
    kname = fit_kernel_name(cfg["y"].shape[1], cfg["y"].shape[0], cfg["w"] is not None,
                            cfg["y"].dtype == torch.float64)
    roof = roofline(kname, cfg["name"], alg, med)
    if kname.startswith("short_rows") and roof["traffic"] is not None:
        roof["traffic_note"] = ("ncu DRAM bytes of one launch: the reads are the input once; "
                                "most of the output is still dirty in L2 when a launch ends and "
                                "is written back during the next one")

    # end to end through the public API: every step copies its input from pinned host memory,
    # fits it and copies the fit back to pinned host memory; steps alternate between two
    # streams, so that one step's upload overlaps the previous one's download (PCIe carries
    # both directions at once)
    host_y = cfg["y"].cpu().pin_memory()
    host_outs = [torch.empty_like(host_y).pin_memory() for _ in range(2)]
    kw = dict(increasing=cfg["increasing"], exact=cfg["exact"], y_min=cfg["y_min"],
              y_max=cfg["y_max"])
    host_w = None if cfg["w"] is None else cfg["w"].cpu().pin_memory()
    streams = [torch.cuda.Stream(dev) for _ in range(2)]

    def e2e_step(k: int) -> None:
        with torch.cuda.stream(streams[k % 2]):
            y = host_y.to(dev, non_blocking=True)
            w = None if host_w is None else host_w.to(dev, non_blocking=True)
            out = torchisotonic_b200.isotonic(y, w, **kw)
            host_outs[k % 2].copy_(out, non_blocking=True)

    def e2e_run(steps: int, warmup: int) -> float:
        for k in range(warmup):
            e2e_step(k)
        torch.cuda.synchronize()
        barrier(world)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        for st in streams:
            st.wait_stream(torch.cuda.current_stream())
        for k in range(steps):
            e2e_step(k)
        for st in streams:
            torch.cuda.current_stream().wait_stream(st)
        end.record()
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(start.elapsed_time(end) / 1e3, world)

    e2e_steps = max(3, min(args.steps, 20))
    e2e_total = e2e_run(e2e_steps, max(2, args.warmup // 2))
    h2d = host_y.numel() * host_y.element_size() + (0 if host_w is None else
                                                    host_w.numel() * host_w.element_size())
    d2h = host_outs[0].numel() * host_outs[0].element_size()

    # parity spot check of the timed output (the first set) against the public API
    ref_out = torchisotonic_b200.isotonic(fitter.ys[0], fitter.ws[0], **kw)
    same = bool(torch.equal(ref_out.isnan(), fitter.outs[0].isnan())
                and torch.equal(ref_out.nan_to_num(0.0), fitter.outs[0].nan_to_num(0.0)))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(cfg, budget_s=args.cpu_seconds)
    del fitter, ref_out, host_y, host_outs, host_w
    cfg_desc, cfg_name, cfg_shape, cfg_exact = cfg["desc"], cfg["name"], list(cfg["y"].shape), cfg["exact"]
    del cfg
    torch.cuda.empty_cache()

    configs = None
    if not args.headline_only:
        configs = measure_configs(dev, args, rank, world)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": 1e3 * t_max / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32 data, f64 sums" if cfg_exact else "f32",
            "data": "synthetic (seeded, generated on the device; rank r uses seed r)",
            "config": {"workload": cfg_desc, "name": cfg_name, "shape": cfg_shape,
                       "per_gpu_elements": elements, "parallelism": f"rows sharded x{world}",
                       "l2": f"{sets} rotating input/output sets ({sets * alg / 1e6:.0f} MB > L2)"
                       if sets > 1 else "inputs larger than L2"},
            "gb_per_s": world * alg * args.steps / t_max / 1e9,
            "roofline": roof,
            "e2e": {"value": world * elements * e2e_steps / e2e_total, "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "torchisotonic_b200.isotonic with pinned host input and output, "
                            "steps on two alternating streams (one step's upload overlapping "
                            "the previous one's download)"},
            "cpu_baseline": cpu,
            "gpu_launches": nlaunch * args.steps,
            "clocks": clk,
            "output_matches_public_api": same,
        }
        if configs is not None:
            line["configs"] = configs
        print(json.dumps(line), flush=True)


def measure_split(args, rank: int, world: int, dev: torch.device) -> dict:
    """c4 on N GPUs: the one long row split into N contiguous segments, one per rank, fitted by
    torchisotonic_b200.split.isotonic_split_row (the segments' block lists all-gathered over
    NCCL each step). Total work is fixed as N grows (strong scaling)."""
    from torchisotonic_b200 import split

    cfg = config("c4", dev, seed=0)  # every rank makes the same row and keeps its segment
    n = cfg["y"].shape[1]
    s0, s1 = n * rank // world, n * (rank + 1) // world
    y = cfg["y"][0, s0:s1].clone()
    w = cfg["w"][0, s0:s1].clone()
    first = float(cfg["y"][0, 0])  # every rank made the whole row: it knows the first element
    desc = cfg["desc"]
    del cfg
    torch.cuda.empty_cache()
    kw = dict(increasing=True, y_min=None, y_max=None, seg_start=s0, row_first=first)
    outs: list = [None]

    def step(k: int) -> None:
        outs[0] = split.isotonic_split_row(y, w, **kw)

    total, med = timed(step, args.steps, args.warmup, world)
    c = torch.randn(y.shape, device=dev, generator=torch.Generator(device=dev).manual_seed(7))
    yg = y.clone().requires_grad_()
    wg = w.clone().requires_grad_()

    def fb(k: int) -> None:
        yg.grad = None
        wg.grad = None
        split.isotonic_split_row(yg, wg, **kw).backward(c)

    fb_steps = max(3, args.steps // 2)
    fb_total, _ = timed(fb, fb_steps, args.warmup, world)
    alg = n * 4 * 3  # y, w in; out written (float32)
    res = {"workload": desc, "shape": [1, n], "per_gpu_elements": s1 - s0,
           "parallelism": f"one row split into {world} segments, block lists all-gathered "
                          "over NCCL",
           "scaling": "strong",
           "fwd": {"ms": 1e3 * total / args.steps, "elements_per_s": n * args.steps / total,
                   "roofline": roofline("split_step", "c4_split", alg / world, med)},
           "fwd_bwd": {"ms": 1e3 * fb_total / fb_steps,
                       "elements_per_s": n * fb_steps / fb_total,
                       "path": "torchisotonic_b200.split.isotonic_split_row(...).backward()"}}
    del y, w, yg, wg, c, outs
    torch.cuda.empty_cache()
    return res


def run_split(args, rank: int, world: int, local: int) -> None:
    """--config c4 on N > 1 GPUs: the split row as the line's own value (strong scaling)."""
    dev = torch.device("cuda", local)
    torch.cuda._sleep(500_000_000)
    clocks = Clocks(local)
    r = measure_split(args, rank, world, dev)
    clk = clocks.stop()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": r["fwd"]["elements_per_s"], "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["fwd"]["ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32 data, f64 sums",
            "data": "synthetic (seeded, generated on the device)",
            "config": {"workload": r["workload"], "name": "c4", "shape": r["shape"],
                       "per_gpu_elements": r["per_gpu_elements"],
                       "parallelism": r["parallelism"], "l2": "inputs larger than L2"},
            "roofline": r["fwd"]["roofline"], "fwd_bwd": r["fwd_bwd"], "cpu_baseline": None,
            "gpu_launches": 9 * args.steps, "clocks": clk,
        }), flush=True)


def cal_inputs(n: int, device: torch.device, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The calibration workload: n model scores sigmoid(N(0,1)) in float32 (many repeat: float32
    has about 1.7e7 values in [0.5, 1)) and Bernoulli(score) labels, as the reference's Criteo
    example feeds its curve (examples/ctr_calibration/calibrate.py:171-186), seeded."""
    gen = torch.Generator(device=device).manual_seed(seed)
    scores = torch.sigmoid(torch.randn(n, generator=gen, device=device))
    labels = torch.bernoulli(scores, generator=gen)
    return scores, labels


def cal_cpu_recipe(scores: torch.Tensor, labels: torch.Tensor, threads: int) -> None:
    """The reference's recipe on the host (README.md:43-50): torch.sort, unique_consecutive,
    index_add_ and sums / counts on CPU tensors, then the reference's own pava.h (oracle/_ref)."""
    import oracle

    torch.set_num_threads(threads)
    s, order = torch.sort(scores)
    xs, inverse, counts = torch.unique_consecutive(s, return_inverse=True, return_counts=True)
    sums = torch.zeros(len(xs), dtype=torch.float64)
    sums.index_add_(0, inverse, labels[order].double())
    oracle.ref_fit((sums / counts).numpy()[None], counts.double().numpy()[None], threads=threads)


def run_calibration(args, rank: int, world: int, local: int) -> None:
    """A calibration curve per GPU (--config cal): fit_calibration over n raw (score, label)
    pairs - the radix sort of the pairs, the pooling of equal scores (three passes of ours) and
    the weighted fit of the pooled means - every rank its own curve (weak scaling, as the
    reference's example fits one curve per segment). Metric: raw pairs per second."""
    import torchisotonic_b200
    from torchisotonic_b200 import _ext

    dev = torch.device("cuda", local)
    n = args.cal_n
    scores, labels = cal_inputs(n, dev, seed=rank)
    unit = "pairs/s"

    def step(k: int) -> None:
        torchisotonic_b200.fit_calibration(scores, labels)

    torch.cuda._sleep(500_000_000)
    clocks = Clocks(local)
    barrier(world)
    total, per = time_steps(step, args.steps, args.warmup)
    barrier(world)
    clk = clocks.stop()
    t_max = max_over_ranks(total, world)
    xs, fit = torchisotonic_b200.fit_calibration(scores, labels)
    groups = xs.numel()
    if args.timed_only:  # for profiling the timed steps alone
        if rank == 0:
            print(json.dumps({"config": "cal", "pairs": n, "groups": groups,
                              "ms_per_step": 1e3 * t_max / args.steps}), flush=True)
        return

    # the pooling kernels alone, on pairs that come sorted: the roofline of our passes
    ss, order = torch.sort(scores)
    sl = labels[order].contiguous()
    del order
    _, pool_per = time_steps(lambda k: _ext.calib_groups(ss, sl, presorted=True),
                             args.steps, args.warmup)
    pool_s = statistics.median(pool_per)
    alg = n * (scores.element_size() + labels.element_size()) + groups * (
        scores.element_size() + 16)
    peak, peak_kind = peaks()
    roof = {"bound": "hbm", "kernel": "group_tile_kernel + group_scan_kernel + group_write_kernel",
            "achieved": alg / pool_s / 1e9, "peak": peak, "unit": "GB/s",
            "frac": alg / pool_s / 1e9 / peak, "peak_source": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes_per_launch": alg, "ms": 1e3 * pool_s,
            "note": "sorted pairs read once, xs/mean/count written once per group; the "
                    "kernels read the pairs twice by design",
            "traffic": traffic_of("calib_groups", "cal")}

    # the pre-step and the whole curve as the reference's recipe does them on the same GPU
    # (torch.sort, unique_consecutive, index_add_, sums / counts; then this library's fit)
    def torch_pre(k: int):
        s, o = torch.sort(scores)
        u, inv, cnt = torch.unique_consecutive(s, return_inverse=True, return_counts=True)
        sums = torch.zeros(len(u), dtype=torch.float64, device=dev)
        sums.index_add_(0, inv, labels[o].double())
        return u, sums / cnt, cnt.double()

    def torch_recipe(k: int) -> None:
        _, y, w = torch_pre(k)
        torchisotonic_b200.isotonic(y, w)

    _, ours_pre = time_steps(lambda k: _ext.calib_groups(scores, labels), args.steps, args.warmup)
    _, torch_pre_per = time_steps(torch_pre, args.steps, args.warmup)
    _, torch_all_per = time_steps(torch_recipe, args.steps, args.warmup)
    u, _, _ = torch_pre(0)
    same = bool(torch.equal(u, xs))

    # end to end: pinned host pairs in, the curve (xs, fit) back to pinned host memory
    hs, hl = scores.cpu().pin_memory(), labels.cpu().pin_memory()
    hx = torch.empty(n, dtype=scores.dtype).pin_memory()
    hf = torch.empty(n, dtype=torch.float64).pin_memory()

    def e2e_step(k: int) -> None:
        a, b = hs.to(dev, non_blocking=True), hl.to(dev, non_blocking=True)
        cx, cf = torchisotonic_b200.fit_calibration(a, b)
        hx[:cx.numel()].copy_(cx, non_blocking=True)
        hf[:cf.numel()].copy_(cf, non_blocking=True)

    e2e_steps = max(3, min(args.steps, 10))
    barrier(world)
    e2e_total, _ = time_steps(e2e_step, e2e_steps, 1)
    barrier(world)
    e2e_total = max_over_ranks(e2e_total, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        m = min(n, 10_000_000)
        cs, cl = scores[:m].cpu(), labels[:m].cpu()
        runs, t0 = 0, time.perf_counter()
        while runs < 1 or (time.perf_counter() - t0 < args.cpu_seconds and runs < 20):
            cal_cpu_recipe(cs, cl, threads)
            runs += 1
        dt = time.perf_counter() - t0
        cpu = {"value": m * runs / dt, "unit": unit, "cores": threads, "kind": "reference",
               "sample": f"{runs} curves of the first {m} pairs: the reference's recipe on CPU "
                         f"tensors (torch.sort, unique_consecutive, index_add_) and its pava.h, "
                         f"{threads} threads"}

    if rank == 0:
        med = lambda v: 1e3 * statistics.median(v)  # noqa: E731
        line = {
            "metric": "calibration curve: raw (score, label) pairs/s (sort + pool + fit)",
            "value": world * n * args.steps / t_max, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 scores and labels, f64 sums and fit",
            "data": "synthetic (seeded, generated on the device; rank r uses seed r)",
            "config": {"workload": f"calibration curve of {n} pairs: scores sigmoid(N(0,1)) "
                                   f"f32, labels Bernoulli(score) f32", "name": "cal",
                       "pairs": n, "groups": groups, "parallelism": f"one curve per rank x{world}",
                       "l2": "inputs larger than L2"},
            "roofline": roof,
            "pre_step_ms": {"ours_sort_and_pool": med(ours_pre),
                            "torch_sort_unique_index_add": med(torch_pre_per),
                            "torch_recipe_with_this_fit": med(torch_all_per)},
            "output_matches_torch_recipe_xs": same,
            "e2e": {"value": world * n * e2e_steps / e2e_total, "unit": unit,
                    "h2d_bytes_per_step": n * (hs.element_size() + hl.element_size()),
                    "d2h_bytes_per_step": groups * (hx.element_size() + 8),
                    "path": "torchisotonic_b200.fit_calibration with pinned host pairs in and "
                            "the curve copied back"},
            "cpu_baseline": cpu,
            "gpu_launches": (3 + fit_launches(groups, 1)) * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)


RANK_SHAPES = [(1024, 100), (256, 1000), (64, 10_000), (8, 100_000), (1, 1_000_000)]


def run_soft_rank(args, rank: int, world: int, local: int) -> None:
    """Soft rank (--config rank): torchisotonic_b200.soft_rank forward and forward + backward on
    the shapes of the reference's soft-rank benchmark (paper/soft_rank.py:23,91-106), float32
    randn rows, strength 1; every rank its own batch (weak scaling). The headline is the
    [64, 10000] shape's forward + backward."""
    import torchisotonic_b200

    dev = torch.device("cuda", local)
    gen = torch.Generator(device=dev).manual_seed(rank)
    torch.cuda._sleep(500_000_000)
    clocks = Clocks(local)
    shapes = {}
    head = None
    for b, n in RANK_SHAPES:
        x = torch.randn(b, n, generator=gen, device=dev)
        g = torch.randn(b, n, generator=gen, device=dev)
        xr = x.clone().requires_grad_()

        def fwd(k: int) -> None:
            torchisotonic_b200.soft_rank(x, 1.0)

        def fb(k: int) -> None:
            out = torchisotonic_b200.soft_rank(xr, 1.0)
            torch.autograd.grad(out, xr, g)

        barrier(world)
        _, fper = time_steps(fwd, args.steps, args.warmup)
        barrier(world)
        ftot, bper = time_steps(fb, args.steps, args.warmup)
        barrier(world)
        ftot = max_over_ranks(ftot, world)
        shapes[f"{b}x{n}"] = {"fwd_ms": 1e3 * statistics.median(fper),
                              "fwd_bwd_ms": 1e3 * statistics.median(bper)}
        if (b, n) == (64, 10_000):
            head = (x, ftot, statistics.median(bper))
    clk = clocks.stop()
    x, ftot, fb_med = head
    elements = x.numel()
    alg = elements * 4 * 4  # x in, ranks out; upstream g in, gradient out
    peak, peak_kind = peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "soft rank: elements/s, forward + backward",
            "value": world * elements * args.steps / ftot, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * ftot / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 data, f64 sums in the fit",
            "data": "synthetic (seeded randn, generated on the device)",
            "config": {"workload": "soft_rank of float32 [64, 10000] rows, strength 1, "
                                   "forward + backward", "name": "rank",
                       "parallelism": f"rows sharded x{world}", "l2": "inputs smaller than L2 "
                       "(the step's sort and scatter re-read them; the fit kernels' reads hit "
                       "L2)"},
            "roofline": {"bound": "hbm", "kernel": "soft_rank step (sort + fit + scatter + "
                         "backward)", "achieved": alg / fb_med / 1e9, "peak": peak,
                         "unit": "GB/s", "frac": alg / fb_med / 1e9 / peak,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": alg, "traffic": None},
            "shapes": shapes,
            "gpu_launches": (fit_launches(10_000, 64) + grad_launches(10_000)) * args.steps,
            "clocks": clk,
        }), flush=True)


def run_reference(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    import oracle

    if oracle.ref_lib() is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libpava_ref.so was not built (no reference checkout)"}))
        return
    if args.config == "rank":
        gen = torch.Generator().manual_seed(0)
        x = torch.randn(64, 10_000, generator=gen).numpy()
        g = torch.randn(64, 10_000, generator=gen).numpy()
        threads = os.cpu_count() or 1
        w = np.arange(x.shape[1], 0, -1, dtype=x.dtype)

        def cpu_step() -> None:  # the composition with the reference's pava.h (-fit(-z))
            perm = np.argsort(-x, axis=-1, kind="stable")
            srt = np.take_along_axis(x, perm, axis=-1)
            neg, starts = oracle.ref_fit(w - srt, None, increasing=True, threads=threads)
            out = np.empty_like(srt)
            np.put_along_axis(out, perm, srt + neg, axis=-1)
            idx = np.cumsum(starts.ravel()) - 1
            sg = np.take_along_axis(g, perm, axis=-1).ravel()
            avg = (np.bincount(idx, weights=sg) / np.bincount(idx))[idx].reshape(x.shape)
            back = np.empty_like(avg)
            np.put_along_axis(back, perm, avg, axis=-1)
            _ = g - back

        for _ in range(args.warmup):
            cpu_step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cpu_step()
        dt = time.perf_counter() - t0
        value = x.size * args.steps / dt
        print(json.dumps({
            "impl": "reference", "metric": "soft rank: elements/s, forward + backward",
            "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)",
            "config": {"workload": "soft_rank of float32 [64, 10000] rows, strength 1, "
                                   "forward + backward", "name": "rank"},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": "the full workload per step: numpy sort and scatter, "
                                       "the reference's pava.h over rows, numpy block sums"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    if args.config == "cal":
        n = min(args.cal_n, 10_000_000)
        scores, labels = cal_inputs(n, torch.device("cpu"), seed=0)
        threads = os.cpu_count() or 1
        for _ in range(args.warmup):
            cal_cpu_recipe(scores, labels, threads)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            cal_cpu_recipe(scores, labels, threads)
        dt = time.perf_counter() - t0
        value = n * args.steps / dt
        print(json.dumps({
            "impl": "reference",
            "metric": "calibration curve: raw (score, label) pairs/s (sort + pool + fit)",
            "value": value, "unit": "pairs/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 scores and labels, f64 sums and fit", "data": "synthetic (seeded)",
            "config": {"workload": f"calibration curve of {n} pairs (a bounded sample of the "
                                   f"GPU arm's {args.cal_n})", "name": "cal"},
            "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": threads,
                             "kind": "reference",
                             "sample": f"{n} pairs per step: torch.sort, unique_consecutive, "
                                       f"index_add_ on CPU tensors and the reference's pava.h"},
            "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }), flush=True)
        return
    cfg = config(args.config, torch.device("cpu"))
    yt = cfg["y"] if cfg["y"].dtype == torch.float64 else cfg["y"].float()
    y = yt.numpy()
    w = None if cfg["w"] is None else cfg["w"].to(yt.dtype).numpy()
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        oracle.ref_fit(y, w, increasing=cfg["increasing"], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.ref_fit(y, w, increasing=cfg["increasing"], threads=threads)
    dt = time.perf_counter() - t0
    value = y.size * args.steps / dt
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": cfg["desc"], "name": cfg["name"], "shape": list(y.shape)},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": f"the full {cfg['name']} workload per step, the reference's "
                                   f"pava.h over rows with {threads} threads"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2",
                    choices=["c1", "c2", "c2_fast", "c3", "c4", "c5", "cal", "rank"])
    ap.add_argument("--cal-n", type=int, default=100_000_000,
                    help="pairs of the calibration workload (--config cal)")
    ap.add_argument("--timed-only", action="store_true",
                    help="--config cal: the timed curve fits only (for ncu launch lists)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--headline-only", action="store_true",
                    help="the headline config alone (no `configs` key)")
    ap.add_argument("--configs", default=None,
                    help="comma-separated configs to measure (default: all of them)")
    ap.add_argument("--configs-batch", type=int, default=None,
                    help="rows of the measured configs (smaller cases for profiling only)")
    ap.add_argument("--no-ref", action="store_true",
                    help="skip the reference's CUDA operators in the configs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines")
    ap.add_argument("--cpu-seconds", type=float, default=4.0,
                    help="host time per CPU baseline sample (one per config)")
    ap.add_argument("--batch", type=int, default=None,
                    help="rows of the workload (smaller cases for profiling; not a bench line)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_init(args.gpus)
    try:
        if args.config == "cal":
            run_calibration(args, rank, world, local)
        elif args.config == "rank":
            run_soft_rank(args, rank, world, local)
        elif args.config == "c4" and world > 1:
            run_split(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
