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
        lists = torch.stack([a, b.view(torch.int64)])
        metas, host, gathered, cap = split.gather_lists(
            count, lists, extra=torch.tensor([rank, 7], dtype=torch.int32))
        assert torch.equal(metas.cpu(), host)
        ga, gb = gathered[0], gathered[1].view(torch.float64)
        start, total = split.segment_starts(10 * (rank + 1))
        q.put((rank, metas.tolist(), ga.tolist(), gb.tolist(), cap, start, total))
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
    for rank, metas, ga, gb, got_cap, start, total in res:
        assert [m[0] for m in metas] == lens and got_cap == cap
        assert [m[1:] for m in metas] == [[r, 7] for r in range(world)]
        for k, m in enumerate(lens):
            assert ga[k * cap:k * cap + m] == list(range(100 * k, 100 * k + m))
            assert gb[k * cap:k * cap + m] == [0.5 * v for v in range(100 * k, 100 * k + m)]
        assert start == sum(10 * (r + 1) for r in range(rank))
        assert total == sum(10 * (r + 1) for r in range(world))


# ---------------------------------------------------------------------------------------------
# GPU: P segments on one device against the oracle


def split_local(y: torch.Tensor, w: torch.Tensor | None, bounds: list[int], increasing: bool,
                y_min=None, y_max=None, with_offs: bool = True):
    """The split-row pipeline for segments [bounds[k], bounds[k+1]) of a 1-D CUDA row, all on
    one device; returns (fit, starts) of the whole row. with_offs: the expand finds each tile's
    blocks from the segment's tile offsets (else by searching the whole list)."""
    parts = len(bounds) - 1
    y0 = _ext.row_offset(float(y[0]))
    lists = []
    for k in range(parts):
        s, e = bounds[k], bounds[k + 1]
        lists.append(_ext.segment_blocks(y[s:e], None if w is None else w[s:e], s, increasing,
                                         y0))
    counts = torch.cat([c for _, c, _, _ in lists])
    nans = torch.cat([nn for _, _, nn, _ in lists])
    cap = max(1, int(counts.max()))

    def padded(i):
        out = torch.zeros(parts * cap, dtype=torch.int64, device=y.device)
        for k in range(parts):
            m = min(cap, lists[k][0].shape[1])
            out[k * cap:k * cap + m] = lists[k][0][i, :m]
        return out

    g_st, g_t, g_w = padded(0), padded(1).view(torch.float64), padded(2).view(torch.float64)
    outs, sts = [], []
    for me in range(parts):
        o, st = _ext.segment_expand(y.dtype, parts, me, cap, g_st.clone(), g_t.clone(),
                                    g_w.clone(), counts, nans, bounds[me + 1] - bounds[me],
                                    bounds[me], increasing, y0, y_min, y_max, True,
                                    lists[me][3] if with_offs else None)
        outs.append(o)
        sts.append(st)
    return torch.cat(outs), torch.cat(sts)


def _check(y, w, bounds, increasing=True, y_min=None, y_max=None, with_offs=True):
    out, st = split_local(y.cuda(), None if w is None else w.cuda(), bounds, increasing,
                          y_min, y_max, with_offs)
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
    bounds = _bounds(n, parts, gen, ragged)
    _check(y, w, bounds)
    if dtype == torch.float32:  # the expand that searches the whole list (no tile offsets)
        _check(y, w, bounds, with_offs=False)


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
        ys = y[s:e].float().cuda().requires_grad_()
        ws = w[s:e].cuda().requires_grad_()
        out, st = split.isotonic_split_row(ys, ws, y_max=4.0, with_starts=True)
        c = torch.randn(n, generator=torch.Generator().manual_seed(5))[s:e].cuda()
        (out * c).sum().backward()
        # the caller knows where its segment starts and the row's first element: no exchange of
        # the segments' heads, the same results
        out2, st2 = split.isotonic_split_row(ys.detach(), ws.detach(), y_max=4.0,
                                             with_starts=True, seg_start=s,
                                             row_first=float(y[0].float()))
        assert torch.equal(out2, out.detach()) and torch.equal(st2, st)
        q.put((rank, out.detach().cpu(), st.cpu(), ys.grad.cpu(), ws.grad.cpu()))
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
    res = sorted((q.get(timeout=300) for _ in range(world)), key=lambda r: r[0])
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
    c = torch.randn(n, generator=torch.Generator().manual_seed(5))
    oy, ow = _oracle_grads(y.float(), w, c, y_max=4.0)
    torch.testing.assert_close(torch.cat([r[3] for r in res]), oy, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(torch.cat([r[4] for r in res]), ow, rtol=2e-5, atol=2e-4)


# ---------------------------------------------------------------------------------------------
# GPU: the split backward, segments on one device, against the oracle's gradients


def split_grad_local(y, w, c, bounds, increasing=True, y_min=None, y_max=None):
    """Gradients of sum(fit * c) for a row split at `bounds`, all segments on one device."""
    parts = len(bounds) - 1
    _, st = split_local(y, w, bounds, increasing, y_min, y_max)
    y0 = _ext.row_offset(float(y[0]))
    want_w = w is not None
    need_y = want_w or y_min is not None or y_max is not None
    runs, wss = [], []
    for k in range(parts):
        s, e = bounds[k], bounds[k + 1]
        ws = _ext.segment_grad_workspace(c.dtype, w is not None, e - s, c.device)
        wss.append(ws)
        runs.append(_ext.segment_grad_sums(y[s:e] if need_y else None,
                                           None if w is None else w[s:e], st[s:e], c[s:e], s,
                                           y0, want_w, y_min, y_max, ws))
    runs = torch.cat(runs)
    gys, gws = [], []
    for k in range(parts):
        s, e = bounds[k], bounds[k + 1]
        gy, gw = _ext.segment_grad(parts, k, runs, y[s:e] if need_y else None,
                                   None if w is None else w[s:e], st[s:e], c[s:e], s, y0,
                                   want_w, y_min, y_max, wss[k])
        gys.append(gy)
        gws.append(gw)
    return torch.cat(gys), (torch.cat(gws) if want_w else None)


def _oracle_grads(y, w, c, increasing=True, y_min=None, y_max=None):
    acc = torch.float64 if y.dtype == torch.float64 else torch.float32
    fy = y.to(acc).numpy()[None]
    fw = None if w is None else w.to(acc).numpy()[None]
    fit, starts = oracle.fit(fy, fw, increasing=increasing)
    gy, gw = oracle.grad(fit, starts, c.to(acc).numpy()[None], fw, fy if w is not None else None,
                         y_min=y_min, y_max=y_max)
    return torch.from_numpy(gy[0]), None if gw is None else torch.from_numpy(gw[0])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("weighted", [False, True])
@pytest.mark.parametrize(("n", "parts"), [(5000, 2), (70_000, 8), (300_000, 3), (33, 32)])
def test_split_gradients_match_whole_row(dtype, weighted, n, parts) -> None:
    gen = np.random.default_rng(n + parts)
    x = np.linspace(-2.0, 3.0, n)
    y = torch.from_numpy(x + gen.normal(0, 1.0, n)).to(dtype)
    w = (torch.from_numpy(gen.uniform(0.1, 2.0, n).astype(np.float32)).to(_ext.acc_dtype(dtype))
         if weighted else None)
    c = torch.from_numpy(gen.normal(0, 1, n)).to(dtype)
    bounds = _bounds(n, parts, gen, True)
    for kw in ({}, {"y_min": -1.0, "y_max": 2.0}, {"increasing": False}):
        gy, gw = split_grad_local(y.cuda(), None if w is None else w.cuda(), c.cuda(), bounds,
                                  **kw)
        oy, ow = _oracle_grads(y, w, c, **kw)
        tol = 1e-9 if dtype == torch.float64 else 2e-5
        torch.testing.assert_close(gy.cpu().double(), oy.double(), rtol=tol, atol=tol)
        if weighted:
            scale = 1 + float(y.double().abs().max())
            torch.testing.assert_close(gw.cpu().double(), ow.double(), rtol=tol, atol=tol * scale)


@pytest.mark.gpu
def test_split_gradients_long_segments_and_nan() -> None:
    # segments of more than 1024 tiles (chunked scans) and a NaN row
    n = 2_500_000
    gen = np.random.default_rng(9)
    i = np.arange(n)
    y = torch.from_numpy(np.sin(i / 40_000) + 0.3 * gen.normal(0, 1, n))
    w = torch.from_numpy(gen.uniform(0.1, 2.0, n).astype(np.float32)).double()
    c = torch.from_numpy(gen.normal(0, 1, n))
    bounds = [0, 1_300_000, n]
    gy, gw = split_grad_local(y.cuda(), w.cuda(), c.cuda(), bounds)
    oy, ow = _oracle_grads(y, w, c)
    torch.testing.assert_close(gy.cpu(), oy, rtol=1e-9, atol=1e-9)
    torch.testing.assert_close(gw.cpu(), ow, rtol=1e-9, atol=1e-8)
    y[1_700_000] = math.nan
    gy, gw = split_grad_local(y.cuda(), w.cuda(), c.cuda(), bounds)
    oy, ow = _oracle_grads(y, w, c)
    torch.testing.assert_close(gy.cpu(), oy, rtol=1e-9, atol=1e-9, equal_nan=True)
    assert bool(gw.isnan().all()) and bool(ow.isnan().all())
