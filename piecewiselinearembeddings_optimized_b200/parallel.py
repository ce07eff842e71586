"""Data-parallel helpers: batch sharding and one packed gradient all-reduce.

Rows of a batch are independent in the forward and in grad_x, so each rank
processes a contiguous shard of the global batch; only the parameter
gradients (``linear.weight [F, B, D]`` plus ``linear.bias`` or
``linear0.weight`` / ``linear0.bias``, each ``[F, D]``) need one exchange.
``GradientBucket`` owns one flat fp32 buffer whose views are handed to the
fused backward (C ABI / ``embeddings_backward``) or filled from ``.grad``, and
reduces it with a single ``all_reduce`` (NCCL over NVLink on GPUs, gloo on
CPU).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n_global: int, world_size: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range ``[start, stop)`` of ``rank``."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must be in [0, world_size)")
    base, extra = divmod(n_global, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class GradientBucket:
    """One flat fp32 buffer holding every parameter gradient of a module."""

    def __init__(self, params, device=None):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        device = device or self.params[0].device
        self.numel = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.views = []
        off = 0
        for p in self.params:
            self.views.append(self.flat[off: off + p.numel()].view_as(p))
            off += p.numel()

    def gather(self) -> None:
        """Copy each parameter's ``.grad`` into the bucket (zeros when absent)."""
        for p, v in zip(self.params, self.views):
            if p.grad is None:
                v.zero_()
            else:
                v.copy_(p.grad)

    def scatter(self) -> None:
        """Point each parameter's ``.grad`` at its (reduced) bucket view."""
        for p, v in zip(self.params, self.views):
            p.grad = v

    def all_reduce(self, average: bool = False, group=None) -> None:
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
            if average:
                self.flat.div_(dist.get_world_size(group))


def allreduce_gradients(module: torch.nn.Module, average: bool = False, group=None) -> GradientBucket:
    """Sum (or average) the parameter gradients of ``module`` across ranks with
    one collective; afterwards every ``.grad`` is a view of the reduced bucket."""
    bucket = getattr(module, "_ple_grad_bucket", None)
    if bucket is None or bucket.flat.device != next(module.parameters()).device:
        bucket = GradientBucket(module.parameters())
        module._ple_grad_bucket = bucket
    bucket.gather()
    bucket.all_reduce(average=average, group=group)
    bucket.scatter()
    return bucket
