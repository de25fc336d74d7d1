"""Batch sharding of the denoising job over the GPUs of one node.

The reference is single-process; the UNet workload shards naturally by sample (GroupNorm
statistics are per (sample, group), attention per (sample, head), conv and linear per row), so
each rank denoises its slice of the batch with replicated weights and no collective on the data
path, and the output latents are all-gathered once at the end (NCCL over NVLink on the GPU
box; gloo in the CPU tests).  Every kernel's tiling is independent of the batch size, so the
gathered result equals a single-GPU run bit for bit.

The device all-gather is NCCL called through the library's C ABI (`NcclCommunicator`:
`mt_nccl_comm_init` / `mt_nccl_all_gather` on the library stream).  Only the host-side
rendezvous — handing rank 0's NCCL unique id to the other ranks — needs a key-value store, and
any object with blocking `set(key, bytes)` / `get(key) -> bytes` serves (torch.distributed's
TCPStore in bench.py).  `init` / `gather_shards` are the host (gloo) process-group helpers the
CPU tests use.
"""
from __future__ import annotations

import ctypes as C
import datetime

from . import _lib as L
from . import runtime


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


class NcclCommunicator:
    """An NCCL communicator over this process's current device, built from a rendezvous store."""

    ID_BYTES = 128

    def __init__(self, rank: int, world: int, store, key: str = "mtorch_b200/nccl_id"):
        lib = L.lib()
        if not lib.mt_nccl_available():
            raise RuntimeError("NCCL (libnccl.so.2) could not be loaded")
        self.rank, self.world = int(rank), int(world)
        self.device = runtime.current_device()
        if self.rank == 0:
            uid = (C.c_uint8 * self.ID_BYTES)()
            L.check(lib.mt_nccl_unique_id(uid, self.ID_BYTES), "nccl unique id")
            store.set(key, bytes(uid))
        raw = bytes(store.get(key))
        if len(raw) != self.ID_BYTES:
            raise RuntimeError(f"NCCL unique id from the store has {len(raw)} bytes, not {self.ID_BYTES}")
        uid = (C.c_uint8 * self.ID_BYTES).from_buffer_copy(raw)
        comm = C.c_void_p()
        L.check(lib.mt_nccl_comm_init(C.byref(comm), uid, self.ID_BYTES, self.world, self.rank), "nccl init")
        self.comm = comm.value

    def all_gather(self, local):
        """Concatenates every rank's contiguous device tensor `local` (same shape everywhere)
        along dim 0 in rank order; returns a new device tensor on the library stream."""
        from .tensor import empty

        src = local.contiguous()
        out = empty(src.shape[0] * self.world, *src.shape[1:], dtype=src.dtype, device=src.device)
        nbytes = src.numel() * src.dtype.itemsize
        L.check(L.lib().mt_nccl_all_gather(src.data_ptr(), out.data_ptr(), nbytes, self.comm,
                                           runtime.stream_ptr(src._idx())), "nccl all_gather")
        return out

    def close(self):
        if self.comm:
            L.check(L.lib().mt_nccl_comm_destroy(self.comm), "nccl destroy")
            self.comm = None
