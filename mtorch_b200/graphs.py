"""CUDA-graph capture of a device computation built from mtorch_b200 ops.

The UNet forward is ~600 kernel launches issued from Python through the C ABI; at small
per-GPU batches (the 8-GPU shard of the 64-sample job is 8 samples) the host would be the
bottleneck.  `Graphed` records the launches once into a CUDA graph on torch's capture stream
(every kernel of this library is launched on the current stream, and device buffers come from
torch's allocator, which gives the capture a private pool) and replays it with one call.

Rules for the captured function: fixed shapes, inputs read from the static buffers created here,
no host synchronisation inside (e.g. no `.cpu()` / `.numpy()`), and any per-weight caches
(packed conv weights, interleaved GEGLU weights) already built — the constructor runs the
function twice before capturing, which also sizes the shared kernel workspace.
"""
from __future__ import annotations

from ._lib import lib
from .tensor import Tensor, _t


class Graphed:
    def __init__(self, fn, *example_inputs: Tensor, warmup: int = 2):
        torch = _t()
        self.fn = fn
        self.static_in = [t.clone() for t in example_inputs]
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*self.static_in)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        n0 = lib().mt_cuda_launch_count()
        with torch.cuda.graph(self.graph):
            self.static_out = fn(*self.static_in)
        self.kernels_per_replay = lib().mt_cuda_launch_count() - n0  # this library's kernels in the graph
        self.replays = 0

    def __call__(self, *inputs: Tensor):
        """Copies `inputs` into the static buffers (skipping those passed as the static buffer
        itself) and replays the graph on the current stream; returns the static output."""
        for dst, src in zip(self.static_in, inputs):
            if src is not dst:
                dst.copy_(src)
        self.graph.replay()
        self.replays += 1
        return self.static_out
