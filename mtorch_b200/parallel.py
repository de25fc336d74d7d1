"""Batch sharding of the denoising job over the GPUs of one node.

The reference is single-process; the UNet workload shards naturally by sample (GroupNorm
statistics are per (sample, group), attention per (sample, head), conv and linear per row), so
each rank denoises its slice of the batch with replicated weights and no collective on the data
path, and the output latents are all-gathered once at the end (NCCL over NVLink on the GPU
box; gloo in the CPU tests).  Every kernel's tiling is independent of the batch size, so the
gathered result equals a single-GPU run bit for bit.
"""
from __future__ import annotations

import datetime


def shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of this rank's samples; the batch must divide evenly (as the bench uses)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    if batch % world:
        raise ValueError(f"batch {batch} does not shard evenly over {world} ranks")
    per = batch // world
    return rank * per, (rank + 1) * per


def init(backend: str = "nccl", timeout_s: float = 300.0, device_id=None):
    """Initialises the default process group from the torchrun environment (RANK, WORLD_SIZE,
    MASTER_ADDR, MASTER_PORT) with a bounded timeout, so a rank that never joins or dies makes
    the others fail instead of hanging."""
    import torch.distributed as dist

    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device_id is not None:
        kw["device_id"] = device_id
    dist.init_process_group(backend, **kw)
    return dist


def gather_shards(local, group=None):
    """All-gathers equally sized 1-D byte buffers (torch uint8 tensors: a device buffer with
    NCCL, a host buffer with gloo) in rank order and returns the concatenation."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = torch.empty(local.numel() * world, dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:  # gloo has no all_gather_into_tensor on every build: gather into views of `out`
        parts = list(out.chunk(world))
        dist.all_gather(parts, local, group=group)
    return out
