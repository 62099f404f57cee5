"""Batch-sharded data-parallel inference across the GPUs of one node.

Every layer of a spiking ResNet is per-sample (eval-mode BN, per-sample LIF
state), so the batch shards with no per-layer exchange: rank r runs samples
``[r*B/g, (r+1)*B/g)`` on its own GPU with a full weight replica, and the only
collective is one all-gather of the logits [T, B/g, classes] at the end of a
forward (NCCL over NVLink; gloo on CPU for tests).  One process per GPU
(``torchrun``); a process-group timeout turns a lost rank into an error on
the others instead of a hang.
"""
from __future__ import annotations

import datetime
import os
from typing import Callable, Optional

import torch
import torch.distributed as dist


def init_inference_group(backend: Optional[str] = None, timeout_s: float = 60.0):
    """Initialise the default process group from the torchrun environment
    (RANK, WORLD_SIZE, MASTER_ADDR, MASTER_PORT, LOCAL_RANK)."""
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    kw = {}
    if backend == "nccl":
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size()


def shard_bounds(batch: int, rank: int, world: int):
    """Contiguous, balanced shard [lo, hi) of a global batch (the first
    batch % world ranks get one extra sample)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_batch(x_seq: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """x_seq [T, B, ...] -> this rank's slice along B."""
    lo, hi = shard_bounds(x_seq.shape[1], rank, world)
    return x_seq[:, lo:hi]


def gather_logits(local: torch.Tensor, global_batch: int, group=None) -> torch.Tensor:
    """All-gather per-rank logits [T, b_r, K] into [T, global_batch, K]
    (shards may differ by one sample: padded to the largest, then trimmed)."""
    world = dist.get_world_size(group)
    T, _, K = local.shape
    sizes = [shard_bounds(global_batch, r, world) for r in range(world)]
    bmax = max(hi - lo for lo, hi in sizes)
    buf = torch.zeros((T, bmax, K), dtype=local.dtype, device=local.device)
    buf[:, :local.shape[1]] = local
    out = torch.empty((world, T, bmax, K), dtype=local.dtype, device=local.device)
    if hasattr(dist, "all_gather_into_tensor") and local.is_cuda:
        dist.all_gather_into_tensor(out, buf.unsqueeze(0).contiguous(), group=group)
    else:
        parts = list(out.unbind(0))
        dist.all_gather(parts, buf, group=group)
        out = torch.stack(parts)
    return torch.cat([out[r, :, :hi - lo] for r, (lo, hi) in enumerate(sizes)], dim=1)


class ShardedInference:
    """Run ``forward(x_local) -> logits_local`` on this rank's shard of a global
    batch and return the gathered logits of the whole batch on every rank."""

    def __init__(self, forward: Callable[[torch.Tensor], torch.Tensor], group=None):
        self.forward = forward
        self.group = group

    def __call__(self, x_seq_global: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size(self.group)
        rank = dist.get_rank(self.group)
        local = self.forward(shard_batch(x_seq_global, rank, world).contiguous())
        return gather_logits(local, x_seq_global.shape[1], self.group)
