"""CUDA-graph capture of a device computation built from mtorch_b200 ops.

The UNet forward is ~600 kernel launches issued from Python through the C ABI; at small
per-GPU batches (the 8-GPU shard of the 64-sample job is 8 samples) the host would be the
bottleneck.  `Graphed` records the launches once into a CUDA graph on the device's library
stream (`mt_cuda_graph_begin` / `mt_cuda_graph_end`: every kernel of this library is launched on
that stream, and while the capture is open the library's allocator serves a pool private to the
graph) and replays it with one call (`mt_cuda_graph_launch`).

Rules for the captured function: fixed shapes, inputs read from the static buffers created here,
no host synchronisation inside (e.g. no `.cpu()` / `.numpy()`), and any per-weight caches
(packed conv weights, interleaved GEGLU weights) already built — the constructor runs the
function twice before capturing, which also sizes the shared kernel workspace.
"""
from __future__ import annotations

import ctypes as C

from . import _lib as L
from . import runtime
from .tensor import Tensor


class Graphed:
    def __init__(self, fn, *example_inputs: Tensor, warmup: int = 2):
        lib = L.lib()
        self.fn = fn
        self.device = example_inputs[0]._idx()
        self.static_in = [t.clone() for t in example_inputs]
        for _ in range(warmup):
            fn(*self.static_in)
        runtime.synchronize()
        self.stream = runtime.stream_ptr(self.device)
        self._graph = None
        n0 = lib.mt_cuda_launch_count()
        L.check(lib.mt_cuda_graph_begin(self.stream), "graph capture begin")
        runtime.capturing.add(self.device)
        g = C.c_void_p()
        try:
            self.static_out = fn(*self.static_in)
        finally:
            runtime.capturing.discard(self.device)
            rc = lib.mt_cuda_graph_end(self.stream, C.byref(g))
        L.check(rc, "graph capture end")
        self._graph = g.value
        self.kernels_per_replay = lib.mt_cuda_launch_count() - n0  # this library's kernels in the graph
        self.replays = 0

    def __call__(self, *inputs: Tensor):
        """Copies `inputs` into the static buffers (skipping those passed as the static buffer
        itself) and replays the graph on the library stream; returns the static output."""
        for dst, src in zip(self.static_in, inputs):
            if src is not dst:
                dst.copy_(src)
        L.check(L.lib().mt_cuda_graph_launch(self._graph, self.stream), "graph launch")
        self.replays += 1
        return self.static_out

    def __del__(self):
        lib = L._LIB
        if lib is not None and getattr(self, "_graph", None):
            lib.mt_cuda_graph_destroy(self._graph)
            self._graph = None
