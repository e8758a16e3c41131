"""One long isotonic-regression row split across the ranks of a process group.

Each rank holds a contiguous segment of the row (rank order = row order) on its own GPU. The
exchange is one step:

1. where each segment starts, and the row's offset y0 from the row's first element (one
   all-gather of two values per rank);
2. every rank fits its segment to a list of blocks (tiso_segment_blocks);
3. the lists are all-gathered over NCCL (counts first, then the lists padded to the longest);
4. every rank merges the lists (the same junction merges as within a device) and writes the
   fit of its own segment (tiso_segment_expand).

No tensor leaves its device except the gathered lists: blocks, not data. A segment's list is as
long as its number of blocks - short for the pooled data of calibration curves, as long as the
segment for increasing data (the worst case, still correct).

The backward is one exchange too: every rank reduces its segment to a run (whether a block
starts in it; the sums of g, w and w (y - y0) before its first start, from its last start on,
and over all of it: 10 numbers), the runs are all-gathered, and every rank fills its own
gradients with the sums of the blocks reaching into its segment from either side.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from torchisotonic_b200 import _ext


def gather_lists(count: Tensor, lists: Tensor, group=None,
                 extra: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor, int]:
    """All-gathers variable-length lists: each rank's `lists` ([k, capacity], int64) hold `count`
    (an int tensor of one element) valid entries per row; `extra` (int) rides along with the
    count. Two all-gathers: the counts (and extras), then - after one host read of them, which
    gives the longest list - the k rows packed side by side (one strided copy). Returns
    ([world, 1 + len(extra)] int32 of every rank's count and extras on the device, the same on
    the host, the gathered lists as [k, world * cap] with rank k's list at k * cap, cap)."""
    world = dist.get_world_size(group)
    dev = count.device
    meta = count.reshape(1).to(torch.int32)
    if extra is not None:
        meta = torch.cat([meta, extra.reshape(-1).to(device=dev, dtype=torch.int32)])
    metas = torch.empty(world * meta.numel(), dtype=torch.int32, device=dev)
    dist.all_gather_into_tensor(metas, meta, group=group)
    metas = metas.view(world, meta.numel())
    host = metas.cpu()  # the one host synchronisation of the exchange
    cap = max(1, int(host[:, 0].max()))
    k = lists.shape[0]
    send = torch.empty(k, cap, dtype=torch.int64, device=dev)
    m = min(cap, lists.shape[1])
    send[:, :m].copy_(lists[:, :m])  # entries past a rank's count are never read
    packed = torch.empty(world * k * cap, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(packed, send.view(-1), group=group)
    gathered = packed.view(world, k, cap).transpose(0, 1).reshape(k, world * cap)
    return metas, host, gathered, cap


def segment_starts(seg_n: int, group=None, device=None) -> tuple[int, int]:
    """(first element of this rank's segment in the row, length of the whole row)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([seg_n], dtype=torch.int64, device=device)
    all_n = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(all_n, n, group=group)
    return int(all_n[:rank].sum()), int(all_n.sum())


def _row_head(y: Tensor, world: int, rank: int, group) -> tuple[int, float]:
    """One all-gather of every rank's segment length and first element: (where this rank's
    segment starts in the row, the row's offset y0 from the first element of the first
    non-empty segment)."""
    head = torch.zeros(2, dtype=torch.float64, device=y.device)
    head[0] = float(y.numel())
    if y.numel():
        head[1] = y[0]
    heads = torch.empty(2 * world, dtype=torch.float64, device=y.device)
    dist.all_gather_into_tensor(heads, head, group=group)
    heads = heads.view(world, 2).cpu()
    lens = heads[:, 0].long()
    seg_start = int(lens[:rank].sum())
    have = lens.nonzero()
    y0 = _ext.row_offset(float(heads[int(have[0]), 1])) if have.numel() else 0.0
    return seg_start, y0


def _fit_segment(y: Tensor, w: Tensor | None, increasing: bool, y_min, y_max, group,
                 with_starts: bool, seg_start: int | None = None, row_first: float | None = None):
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if seg_start is None or row_first is None:
        seg_start, y0 = _row_head(y, world, rank, group)
    else:
        y0 = _ext.row_offset(float(row_first))
    bad = torch.zeros(1, dtype=torch.int32, device=y.device)
    tile_offs = None
    if y.numel():
        lists, count, nan, tile_offs = _ext.segment_blocks(y, w, seg_start, increasing, y0,
                                                           bad if w is not None else None)
    else:
        lists = torch.zeros(3, 1, dtype=torch.int64, device=y.device)
        count = torch.zeros(1, dtype=torch.int32, device=y.device)
        nan = torch.zeros(1, dtype=torch.int32, device=y.device)
    metas, host, gathered, cap = gather_lists(count, lists, group, extra=torch.cat([nan, bad]))
    if bool(host[:, 2].any()):
        raise ValueError("weight must be strictly positive")
    counts = metas[:, 0].contiguous()
    nans = metas[:, 1].contiguous()
    g_t = gathered[1].view(torch.float64)
    g_w = gathered[2].view(torch.float64)
    out, st = _ext.segment_expand(y.dtype, world, rank, cap, gathered[0], g_t, g_w, counts, nans,
                                  y.numel(), seg_start, increasing, y0, y_min, y_max,
                                  with_starts, tile_offs)
    return out, st, seg_start, y0


def _grad_segment(y: Tensor, w: Tensor | None, starts: Tensor, g: Tensor, seg_start: int,
                  y0: float, want_w: bool, y_min, y_max, group):
    """(grad_y, grad_w or None) of this rank's segment: the first pass, an all-gather of the
    segments' runs (10 float64 each), then the second pass."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = g.numel()
    need_y = want_w or y_min is not None or y_max is not None
    yy = y if need_y else None
    ws = None
    if n:
        ws = _ext.segment_grad_workspace(g.dtype, w is not None, n, g.device)
        run = _ext.segment_grad_sums(yy, w, starts, g, seg_start, y0, want_w, y_min, y_max, ws)
    else:
        run = torch.zeros(10, dtype=torch.float64, device=g.device)
    runs = torch.empty(world * 10, dtype=torch.float64, device=g.device)
    dist.all_gather_into_tensor(runs, run, group=group)
    if not n:
        gw = torch.empty(0, dtype=_ext.acc_dtype(g.dtype), device=g.device) if want_w else None
        return torch.empty_like(g), gw
    return _ext.segment_grad(world, rank, runs, yy, w, starts, g, seg_start, y0, want_w,
                             y_min, y_max, ws)


class _SplitRow(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, w, increasing, y_min, y_max, group, seg_start, row_first):
        out, st, seg_start, y0 = _fit_segment(y, w, increasing, y_min, y_max, group, True,
                                              seg_start, row_first)
        ctx.save_for_backward(y, w, st)
        ctx.info = (seg_start, y0, y_min, y_max, group)
        ctx.mark_non_differentiable(st)
        return out, st

    @staticmethod
    def backward(ctx, g, _g_starts):
        y, w, st = ctx.saved_tensors
        seg_start, y0, y_min, y_max, group = ctx.info
        want_w = w is not None and ctx.needs_input_grad[1]
        gy, gw = _grad_segment(y, w, st, g.to(y.dtype).contiguous(), seg_start, y0, want_w,
                               y_min, y_max, group)
        return gy, gw, None, None, None, None, None, None


def isotonic_split_row(
    y: Tensor,
    weight: Tensor | None = None,
    *,
    increasing: bool = True,
    y_min: float | None = None,
    y_max: float | None = None,
    group=None,
    with_starts: bool = False,
    seg_start: int | None = None,
    row_first: float | None = None,
):
    """The isotonic fit of one long row whose contiguous segments are spread over the ranks of
    `group`: this rank passes its segment `y` (1-D, CUDA) and weights; returns the fit of that
    segment (clipped, in y's float dtype) and, with `with_starts`, where its blocks start.
    Same semantics as torchisotonic_b200.isotonic on the whole row (NaN anywhere in the row
    makes all of it NaN), and differentiable in y and the weights: the backward takes one
    all-gather of 10 numbers per rank. Every rank must take part in the forward and backward.

    `seg_start` (where this rank's segment starts in the row) and `row_first` (the row's first
    element), when the caller knows both, spare the exchange of every segment's length and first
    element and its host synchronisation; every rank must then pass the same `row_first`."""
    if y.dim() != 1 or not y.is_cuda:
        raise ValueError("y must be this rank's 1-D CUDA segment of the row")
    dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
    y = y.to(dtype).contiguous()
    w = None
    if weight is not None:
        w = weight.to(device=y.device, dtype=_ext.acc_dtype(dtype)).broadcast_to(y.shape)
        w = w.contiguous()
    if torch.is_grad_enabled() and (y.requires_grad or (w is not None and w.requires_grad)):
        out, st = _SplitRow.apply(y, w, increasing, y_min, y_max, group, seg_start, row_first)
        return (out, st) if with_starts else out
    out, st, _, _ = _fit_segment(y, w, increasing, y_min, y_max, group, with_starts, seg_start,
                                 row_first)
    return (out, st) if with_starts else out
