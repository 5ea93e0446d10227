"""Batch-sharded data parallelism for the LTC layer: one process per GPU, parameters
replicated, samples split contiguously across ranks, and the parameter gradients
summed across ranks with one all-reduce over a flat bucket (NCCL over NVLink on
B200 nodes; gloo on CPU for tests).

The loss of the benchmark is a sum over samples, so the single-process gradient
is the SUM of the per-shard gradients (not the mean DDP would take).  The
reference has no multi-GPU code; this is the exchange step the sharded solver
needs and nothing more (the forward pass communicates nothing).
"""
from __future__ import annotations

from typing import Iterable, List, Tuple

import torch
import torch.distributed as dist


def shard_range(total: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [lo, hi) slice of `total` samples for `rank` (sizes differ by at most 1)."""
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class FlatGradBucket:
    """Gives every parameter a ``.grad`` that is a view into one flat buffer, so that
    autograd accumulates straight into it and a single collective reduces all of it."""

    def __init__(self, params: Iterable[torch.nn.Parameter]):
        self.params: List[torch.nn.Parameter] = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        dev, dt = self.params[0].device, self.params[0].dtype
        n = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(n, device=dev, dtype=dt)
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()

    def zero(self) -> None:
        self.flat.zero_()

    def check_views(self) -> None:
        """Raise if autograd replaced a .grad instead of accumulating into the bucket."""
        base = self.flat.untyped_storage().data_ptr()
        for p in self.params:
            if p.grad is None or p.grad.untyped_storage().data_ptr() != base:
                raise RuntimeError("a parameter gradient left the flat bucket")

    def all_reduce(self, group=None) -> None:
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)

    @property
    def nbytes(self) -> int:
        return self.flat.numel() * self.flat.element_size()


def training_step(model, x: torch.Tensor, bucket: FlatGradBucket, optimizer, group=None) -> torch.Tensor:
    """Forward, sum loss, backward, gradient all-reduce (SUM), optimizer step."""
    bucket.zero()
    out, _ = model(x)
    loss = out.sum()
    loss.backward()
    bucket.all_reduce(group)
    optimizer.step()
    return loss.detach()
