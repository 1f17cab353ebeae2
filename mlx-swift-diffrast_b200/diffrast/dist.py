"""Data parallelism over views: one process per GPU.

The chain partitions over the view batch: every kernel indexes by view, so
ranks render disjoint views with no collective in the data path.  The only
exchange per step is the sum of the shared-parameter gradients (mesh vertices,
attribute table, texture), done as one flattened all-reduce (NCCL over
NVLink on GPUs; gloo in the CPU tests).
"""
from __future__ import annotations

import datetime
import os
from typing import List, Sequence, Tuple

import torch
import torch.distributed as dist


def view_range(total_views: int, rank: int, world: int, weak: bool) -> Tuple[int, int, int]:
    """Views [lo, hi) of `rank` and the job's total view count.

    weak:   every rank renders `total_views` views of its own (views are numbered
            globally, rank r owns [r*total, (r+1)*total)); per-GPU work is fixed.
    strong: the job's `total_views` are split into equal contiguous blocks.
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    if weak:
        return rank * total_views, (rank + 1) * total_views, total_views * world
    if total_views % world:
        raise ValueError(f"{total_views} views do not split evenly over {world} ranks")
    per = total_views // world
    return rank * per, (rank + 1) * per, total_views


def allreduce_grads(grads: Sequence[torch.Tensor], group=None) -> None:
    """Sum `grads` across ranks in place with one flattened all-reduce."""
    grads = [g for g in grads if g is not None]
    if not grads or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    flat = torch._utils._flatten_dense_tensors(grads)
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    for g, f in zip(grads, torch._utils._unflatten_dense_tensors(flat, grads)):
        g.copy_(f)


class GradSync:
    """All-reduce (sum) of shared-parameter gradients overlapped with the rest
    of the backward: a post-accumulate hook on each parameter launches an
    asynchronous all-reduce as soon as that gradient is final (e.g. the
    attribute table's, while the rasterizer's VJP still runs), and `finish`
    makes the current stream wait for all of them.  Every rank runs the same
    graph, so the hooks fire — and the collectives are issued — in the same
    order everywhere.  A no-op on one rank.

    A step that accumulates gradients over several backward calls
    (micro-batches) calls `arm(last)` before each of them: only the last
    backward's hooks launch all-reduces.  A gradient is final only then, and
    an all-reduce launched earlier would both be summed again by the next one
    and race with the next backward's in-place accumulation into the same
    buffer.  `finish` re-arms, so single-backward steps need no call."""

    def __init__(self, params: Sequence[torch.Tensor], group=None):
        self.group = group
        self.handles = []
        self.armed = True
        self.active = dist.is_initialized() and dist.get_world_size(group) > 1
        if self.active:
            for p in params:
                p.register_post_accumulate_grad_hook(self._launch)

    def arm(self, last: bool) -> None:
        """Before a backward: launch the all-reduces from it only if it is the
        step's last one."""
        self.armed = bool(last)

    def _launch(self, p: torch.Tensor) -> None:
        if not self.armed:
            return
        self.handles.append(dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def finish(self) -> None:
        for h in self.handles:
            h.wait()
        self.handles.clear()
        self.armed = True


def init_from_env(timeout_s: float = 300.0) -> Tuple[int, int, int]:
    """Initialise the process group from torchrun's environment; returns
    (world, rank, local_rank).  NCCL when CUDA is present, gloo otherwise."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return world, rank, local


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a per-rank scalar (step times are reported as the max)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
