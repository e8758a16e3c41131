"""One long isotonic-regression row split across the ranks of a process group.

Each rank holds a contiguous segment of the row (rank order = row order) on its own GPU. The
exchange is one step, as SURVEY's multi-GPU plan for the single long calibration row has it:

1. the row's offset y0 from the row's first element (an all-gather of one value per rank);
2. every rank fits its segment to a list of blocks (tiso_segment_blocks);
3. the lists are all-gathered over NCCL (counts first, then the lists padded to the longest);
4. every rank merges the lists (the same junction merges as within a device) and writes the
   fit of its own segment (tiso_segment_expand).

No tensor leaves its device except the gathered lists: blocks, not data. A segment's list is as
long as its number of blocks - short for the pooled data of calibration curves, as long as the
segment for increasing data (the worst case, still correct).
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from torchisotonic_b200 import _ext


def gather_lists(count: Tensor, arrays: list[Tensor], group=None) -> tuple[Tensor, list[Tensor], int]:
    """All-gathers variable-length lists: each rank's `arrays` hold `count` (an int tensor of one
    element) valid entries. Returns (counts of every rank, each array gathered as a
    [world * cap] tensor with rank k's list at k * cap, cap)."""
    world = dist.get_world_size(group)
    counts = torch.empty(world, dtype=count.dtype, device=count.device)
    dist.all_gather_into_tensor(counts, count.reshape(1), group=group)
    cap = max(1, int(counts.max()))
    out = []
    for a in arrays:
        pad = torch.zeros(cap, dtype=a.dtype, device=a.device)
        m = min(cap, a.numel())
        pad[:m] = a[:m]
        g = torch.empty(world * cap, dtype=a.dtype, device=a.device)
        dist.all_gather_into_tensor(g, pad, group=group)
        out.append(g)
    return counts, out, cap


def segment_starts(seg_n: int, group=None, device=None) -> tuple[int, int]:
    """(first element of this rank's segment in the row, length of the whole row)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([seg_n], dtype=torch.int64, device=device)
    all_n = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(all_n, n, group=group)
    return int(all_n[:rank].sum()), int(all_n.sum())


def isotonic_split_row(
    y: Tensor,
    weight: Tensor | None = None,
    *,
    increasing: bool = True,
    y_min: float | None = None,
    y_max: float | None = None,
    group=None,
    with_starts: bool = False,
):
    """The isotonic fit of one long row whose contiguous segments are spread over the ranks of
    `group`: this rank passes its segment `y` (1-D, CUDA) and weights; returns the fit of that
    segment (clipped, in y's float dtype) and, with `with_starts`, where its blocks start.
    Same semantics as torchisotonic_b200.isotonic on the whole row (NaN anywhere in the row
    makes all of it NaN). Forward only."""
    if y.dim() != 1 or not y.is_cuda:
        raise ValueError("y must be this rank's 1-D CUDA segment of the row")
    dtype = y.dtype if y.is_floating_point() else torch.get_default_dtype()
    y = y.to(dtype).contiguous()
    acc = _ext.acc_dtype(dtype)
    w = None
    if weight is not None:
        w = weight.to(device=y.device, dtype=acc).broadcast_to(y.shape).contiguous()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    seg_start, _ = segment_starts(y.numel(), group, y.device)
    # the row's offset comes from its first element: the first element of the first rank with
    # a non-empty segment
    head = torch.zeros(2, dtype=torch.float64, device=y.device)
    if y.numel():
        head[0] = 1.0
        head[1] = y[0].double()
    heads = torch.empty(2 * world, dtype=torch.float64, device=y.device)
    dist.all_gather_into_tensor(heads, head, group=group)
    heads = heads.view(world, 2).cpu()
    have = heads[:, 0].nonzero()
    y0 = _ext.row_offset(float(heads[int(have[0]), 1])) if have.numel() else 0.0
    bad = torch.zeros(1, dtype=torch.int32, device=y.device) if w is not None else None
    if y.numel():
        starts, t, wsum, count, nan = _ext.segment_blocks(y, w, seg_start, increasing, y0, bad)
    else:
        starts = torch.zeros(1, dtype=torch.int64, device=y.device)
        t = torch.zeros(1, dtype=torch.float64, device=y.device)
        wsum = torch.zeros(1, dtype=torch.float64, device=y.device)
        count = torch.zeros(1, dtype=torch.int32, device=y.device)
        nan = torch.zeros(1, dtype=torch.int32, device=y.device)
    counts, (g_starts, g_t, g_w), cap = gather_lists(count, [starts, t, wsum], group)
    nans = torch.empty(world, dtype=torch.int32, device=y.device)
    dist.all_gather_into_tensor(nans, nan, group=group)
    if bad is not None:
        dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=group)
        if bool(bad.item()):
            raise ValueError("weight must be strictly positive")
    out, st = _ext.segment_expand(dtype, world, rank, cap, g_starts, g_t, g_w, counts, nans,
                                  y.numel(), seg_start, increasing, y0, y_min, y_max,
                                  with_starts)
    return (out, st) if with_starts else out
