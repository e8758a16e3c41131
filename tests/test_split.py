"""One long row split into segments across devices (torchisotonic_b200.split, tiso_segment_*).

The reference has no multi-device path; the bar is the single-device fit of the whole row (the
oracle). On one GPU the ranks are emulated: every segment's block list is made, the lists are
laid out as the all-gather lays them out, and each segment is expanded from its own copy of the
gathered lists. The exchange itself (torch.distributed) is tested with gloo ranks on the CPU,
and with NCCL ranks where a box has two GPUs.
"""

from __future__ import annotations

import math
import os
import socket
import struct

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from torchisotonic_b200 import _ext, split
from tests.parity import assert_values, scale_of


# ---------------------------------------------------------------------------------------------
# CPU: the offset rule and the exchange


def _offset_numpy(v: float) -> float:
    if not (abs(v) >= 1.0) or math.isinf(v):
        return 0.0
    b = np.array([v], dtype=np.float64).view(np.int64)
    b &= ~np.int64((1 << 45) - 1)
    return float(b.view(np.float64)[0])


@pytest.mark.parametrize("v", [0.0, 0.99, -0.5, 1.0, -1.0, 1.00390625, 3.7, -123456.789, 1e300,
                               float("nan"), float("inf"), 5e-324])
def test_row_offset_rule(v: float) -> None:
    got = _ext.row_offset(v)
    assert got == _offset_numpy(v)
    if abs(v) >= 1 and math.isfinite(v):
        # 8 significant bits, same sign, not above |v|
        assert abs(got) <= abs(v) and (got > 0) == (v > 0)
        mant = struct.unpack("<q", struct.pack("<d", got))[0] & ((1 << 52) - 1)
        assert mant & ((1 << 45) - 1) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lens = [3, 0, 7][:world] if world == 3 else [5, 2]
        n = lens[rank]
        count = torch.tensor([n], dtype=torch.int32)
        a = torch.arange(100 * rank, 100 * rank + max(n, 1), dtype=torch.int64)
        b = a.double() * 0.5
        counts, (ga, gb), cap = split.gather_lists(count, [a, b])
        start, total = split.segment_starts(10 * (rank + 1))
        q.put((rank, counts.tolist(), ga.tolist(), gb.tolist(), cap, start, total))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gather_lists_gloo(world: int) -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lens = [3, 0, 7] if world == 3 else [5, 2]
    cap = max(lens)
    for rank, counts, ga, gb, got_cap, start, total in res:
        assert counts == lens and got_cap == cap
        for k, m in enumerate(lens):
            assert ga[k * cap:k * cap + m] == list(range(100 * k, 100 * k + m))
            assert gb[k * cap:k * cap + m] == [0.5 * v for v in range(100 * k, 100 * k + m)]
        assert start == sum(10 * (r + 1) for r in range(rank))
        assert total == sum(10 * (r + 1) for r in range(world))


# ---------------------------------------------------------------------------------------------
# GPU: P segments on one device against the oracle


def split_local(y: torch.Tensor, w: torch.Tensor | None, bounds: list[int], increasing: bool,
                y_min=None, y_max=None):
    """The split-row pipeline for segments [bounds[k], bounds[k+1]) of a 1-D CUDA row, all on
    one device; returns (fit, starts) of the whole row."""
    parts = len(bounds) - 1
    y0 = _ext.row_offset(float(y[0]))
    lists = []
    for k in range(parts):
        s, e = bounds[k], bounds[k + 1]
        lists.append(_ext.segment_blocks(y[s:e], None if w is None else w[s:e], s, increasing,
                                         y0))
    counts = torch.cat([c for _, _, _, c, _ in lists])
    nans = torch.cat([nn for _, _, _, _, nn in lists])
    cap = max(1, int(counts.max()))

    def padded(i, dtype):
        out = torch.zeros(parts * cap, dtype=dtype, device=y.device)
        for k in range(parts):
            m = min(cap, lists[k][i].numel())
            out[k * cap:k * cap + m] = lists[k][i][:m]
        return out

    g_st, g_t, g_w = padded(0, torch.int64), padded(1, torch.float64), padded(2, torch.float64)
    outs, sts = [], []
    for me in range(parts):
        o, st = _ext.segment_expand(y.dtype, parts, me, cap, g_st.clone(), g_t.clone(),
                                    g_w.clone(), counts, nans, bounds[me + 1] - bounds[me],
                                    bounds[me], increasing, y0, y_min, y_max, True)
        outs.append(o)
        sts.append(st)
    return torch.cat(outs), torch.cat(sts)


def _check(y, w, bounds, increasing=True, y_min=None, y_max=None):
    out, st = split_local(y.cuda(), None if w is None else w.cuda(), bounds, increasing,
                          y_min, y_max)
    want = oracle.isotonic(y, w, increasing=increasing, y_min=y_min, y_max=y_max)
    assert_values(out, want, scale_of(y))
    acc = _ext.acc_dtype(y.dtype)
    _, want_st = oracle.fit(y.to(acc).numpy()[None], None if w is None else w.numpy()[None],
                            increasing=increasing)
    got_st = st.cpu().numpy()
    if y.isnan().any():
        assert got_st[0] and not got_st[1:].any()
    else:
        bad = np.argwhere(got_st != want_st[0])
        assert not len(bad), f"block starts differ at {len(bad)} places, first {bad[:5].ravel()}"


def _bounds(n: int, parts: int, gen: np.random.Generator, ragged: bool) -> list[int]:
    if not ragged:
        return [n * k // parts for k in range(parts + 1)]
    cuts = np.sort(gen.choice(np.arange(1, n), size=parts - 1, replace=False))
    return [0, *cuts.tolist(), n]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize(("n", "parts", "ragged"),
                         [(1000, 2, False), (5000, 3, True), (70_000, 8, False),
                          (70_000, 8, True), (33, 32, True), (200_000, 5, True)])
def test_split_matches_whole_row(dtype, weighted, n, parts, ragged) -> None:
    gen = np.random.default_rng(n * 7 + parts)
    x = np.linspace(-2.0, 3.0, n)
    y = torch.from_numpy(x + gen.normal(0, 1.0, n)).to(dtype)
    w = None
    if weighted:
        # f32-representable weights: exact ties do not depend on rounding
        w = torch.from_numpy(gen.uniform(0.1, 2.0, n).astype(np.float32)).to(_ext.acc_dtype(dtype))
    _check(y, w, _bounds(n, parts, gen, ragged))


@pytest.mark.gpu
@pytest.mark.parametrize("increasing", [True, False])
def test_split_direction_and_clip(increasing: bool) -> None:
    gen = np.random.default_rng(5)
    n = 40_000
    y = torch.from_numpy(gen.normal(0, 1, n).cumsum() * 0.01 + 100.0).float()
    _check(y, None, _bounds(n, 6, gen, True), increasing=increasing)
    _check(y, None, _bounds(n, 6, gen, True), increasing=increasing, y_min=99.9, y_max=100.2)


@pytest.mark.gpu
@pytest.mark.parametrize("pattern", ["increasing", "decreasing", "constant", "sawtooth"])
def test_split_patterns(pattern: str) -> None:
    n = 30_000
    i = torch.arange(n, dtype=torch.float64)
    y = {"increasing": i, "decreasing": -i, "constant": torch.full((n,), 2.5, dtype=torch.float64),
         "sawtooth": (i % 97) - i * 0.001}[pattern]
    gen = np.random.default_rng(1)
    _check(y, None, _bounds(n, 4, gen, True))
    _check(y.float(), None, [0, 1, 2, 15_000, n])  # one-element segments


@pytest.mark.gpu
@pytest.mark.parametrize("where", [0, 12_345, 29_999])
def test_split_nan_anywhere_makes_the_row_nan(where: int) -> None:
    n = 30_000
    y = torch.randn(n, dtype=torch.float64)
    y[where] = float("nan")
    _check(y, None, [0, 7_000, 20_000, n])


def _nccl_worker(rank: int, world: int, port: int, q) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        gen = torch.Generator().manual_seed(3)
        n = 300_001
        y = (torch.linspace(0, 5, n, dtype=torch.float64) + torch.randn(n, generator=gen,
                                                                          dtype=torch.float64))
        w = torch.rand(n, generator=gen).add_(0.1)
        bounds = [n * k // world for k in range(world + 1)]
        s, e = bounds[rank], bounds[rank + 1]
        out, st = split.isotonic_split_row(y[s:e].float().cuda(), w[s:e].cuda(), y_max=4.0,
                                           with_starts=True)
        q.put((rank, out.cpu(), st.cpu()))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_split_row_over_nccl_ranks() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    gen = torch.Generator().manual_seed(3)
    n = 300_001
    y = torch.linspace(0, 5, n, dtype=torch.float64) + torch.randn(n, generator=gen,
                                                                   dtype=torch.float64)
    w = torch.rand(n, generator=gen).add_(0.1)
    want = oracle.isotonic(y.float(), w, y_max=4.0)
    out = torch.cat([r[1] for r in res])
    assert_values(out, want, scale_of(y))
