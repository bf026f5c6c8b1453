"""(batch x head) sharding of the scan over the GPUs of one node.

Chains (b, h, m) are independent, so a rank scans its own rows of the batch
(or, when the batch is smaller than the world, its own heads) with no
data-path communication; the only collective is one all-gather of the
per-lane outputs after the scan (``all_gather_into_tensor``, NCCL over
NVLink/NVSwitch on GPUs, gloo in the CPU tests).  Every rank keeps all M
lanes of its heads, so the lane-shared q/k/v reads stay local.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class Shard:
    axis: str      # "batch" or "head"
    start: int
    stop: int

    def take(self, x: torch.Tensor, dim_batch: int = 0, dim_head: int = 2) -> torch.Tensor:
        d = dim_batch if self.axis == "batch" else dim_head
        return x.narrow(d, self.start, self.stop - self.start)


def shard_for(B: int, H: int, world: int, rank: int) -> Shard:
    """Whole batch rows first (B divisible by world), else heads (H divisible by world)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if B % world == 0:
        n = B // world
        return Shard("batch", rank * n, (rank + 1) * n)
    if H % world == 0:
        n = H // world
        return Shard("head", rank * n, (rank + 1) * n)
    raise ValueError(f"cannot split B={B} or H={H} evenly over {world} ranks")


def sharded_scan(scan_fn: Callable, inputs: dict, world: int, rank: int, group=None,
                 gather: bool = True) -> torch.Tensor:
    """Scan this rank's shard with ``scan_fn(**shard_inputs) -> y [b,T,h,M,V]`` and
    (optionally) all-gather the full ``[B,T,H,M,V]`` output on every rank.

    ``inputs`` holds tensors with batch at dim 0 and heads at dim 2
    ([B,T,H,...]) plus non-tensor keyword arguments passed through.
    """
    import torch.distributed as dist
    B, _, H = inputs["k"].shape[:3]
    sh = shard_for(B, H, world, rank)
    local = {n: (sh.take(t) if torch.is_tensor(t) and t.dim() >= 3 else t) for n, t in inputs.items()}
    y = scan_fn(**local).contiguous()
    if not gather or world == 1:
        return y
    parts = torch.empty((world * y.shape[0],) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(parts, y, group=group)  # rank r's shard at rows [r*b, (r+1)*b)
    if sh.axis == "batch":
        return parts
    # heads: [world*B, T, h, M, V] -> [B, T, world*h, M, V]
    parts = parts.reshape((world,) + tuple(y.shape))
    return parts.permute(1, 2, 0, 3, 4, 5).reshape(y.shape[0], y.shape[1], H, *y.shape[3:])
