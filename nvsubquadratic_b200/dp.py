"""Batch (data-parallel) sharding of the fused Hyena mixer across GPUs.

The 2D high-resolution configuration shards the batch: each rank runs the fused mixer
on its slice of the batch with the full filter, D and short-conv weights, so the
gradients of those parameters are partial sums over that slice. One all-reduce (sum)
over NCCL turns them into the full-batch gradients, which is what the reference
training stack obtains from DDP's gradient all-reduce around the same module
(nvSubquadratic tests/modules/torchrun_sequence_mixer_cp_test.py:214-218 wraps the
mixer in DDP). Activations need no collective: every batch item is independent.

``GradBucket`` packs the gradients into one flat float32 buffer so the reduction is a
single collective call whatever the number of parameters (the filter gradient
dominates: C x prod(K) floats).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["batch_shard", "GradBucket"]


def batch_shard(x: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rank ``rank``'s contiguous slice of the batch (dim 0); the batch must divide evenly."""
    B = x.shape[0]
    if B % world != 0:
        raise ValueError(f"batch {B} does not split evenly over {world} ranks")
    b = B // world
    return x[rank * b:(rank + 1) * b]


class GradBucket:
    """One flat float32 buffer for the gradients of ``params``.

    ``reduce(group)`` copies every parameter's current ``.grad`` into the buffer, sums
    the buffer over ``group`` with one ``all_reduce`` and returns it; ``grads()`` gives
    the per-parameter views of the reduced buffer (shapes of the parameters). With no
    group, or a group of one rank, the buffer is filled but no collective runs.
    """

    def __init__(self, params, device=None):
        self.params = [p for p in params if p is not None]
        if not self.params:
            raise ValueError("no parameters")
        dev = device if device is not None else self.params[0].device
        self.sizes = [p.numel() for p in self.params]
        self.flat = torch.empty(sum(self.sizes), dtype=torch.float32, device=dev)

    def pack(self) -> torch.Tensor:
        off = 0
        for p, n in zip(self.params, self.sizes):
            dst = self.flat[off:off + n]
            if p.grad is None:
                dst.zero_()
            else:
                dst.copy_(p.grad.reshape(-1))
            off += n
        return self.flat

    def reduce(self, group=None) -> torch.Tensor:
        self.pack()
        if group is not None and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
        return self.flat

    def grads(self) -> list[torch.Tensor]:
        out, off = [], 0
        for p, n in zip(self.params, self.sizes):
            out.append(self.flat[off:off + n].view(p.shape))
            off += n
        return out
