"""The library's own device runtime (no torch anywhere on these paths): the caching allocator
that backs `cuda` tensors, the library stream and timing events, CUDA-graph capture with a
private pool, pinned host memory, and the NCCL all-gather through the C ABI (one rank here; the
batch-sharded bench uses it at 2-8 ranks).

The allocator is the device counterpart of the reference's `Storage` (cpp/mtorch/core/tensor.h:
60-63): every view shares one block, and the block returns to the free list when the last view
goes."""
import gc

import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import _lib, ops, parallel, runtime
from mtorch_b200.graphs import Graphed

pytestmark = pytest.mark.gpu


def test_allocator_reuses_freed_blocks_and_views_share_storage():
    mt.cuda.synchronize()
    gc.collect()
    s0 = mt.cuda.memory_stats()
    a = mt.empty(1 << 20, dtype="float32", device="cuda")  # 4 MiB
    s1 = mt.cuda.memory_stats()
    assert s1["allocated_bytes"] - s0["allocated_bytes"] == 4 << 20
    ptr = a.data_ptr()
    v = a.view(1024, 1024)[3:]
    assert v._buf is a._buf
    del a
    gc.collect()
    assert mt.cuda.memory_stats()["allocated_bytes"] == s1["allocated_bytes"]  # the view keeps it
    del v
    gc.collect()
    s2 = mt.cuda.memory_stats()
    assert s2["allocated_bytes"] == s0["allocated_bytes"]
    b = mt.empty(1 << 20, dtype="float32", device="cuda")
    s3 = mt.cuda.memory_stats()
    assert s3["cached_bytes"] == s2["cached_bytes"] - (4 << 20)  # served from the free list
    assert ptr and b.data_ptr()


def test_free_of_foreign_pointer_is_rejected():
    assert _lib.lib().mt_cuda_free(0x1000) == _lib.MT_ERR_INVALID


def test_events_time_work_on_the_library_stream():
    x = mt.empty(4096, 4096, dtype="bfloat16", device="cuda").uniform_(-1, 1)
    e0, e1 = mt.cuda.Event(), mt.cuda.Event()
    e0.record()
    for _ in range(5):
        ops.matmul(x, x)
    e1.record()
    ms = e0.elapsed_time(e1)
    assert 0.0 < ms < 1000.0


def test_graph_replay_matches_eager_and_uses_a_private_pool():
    mt.manual_seed(3)
    w = mt.randn(256, 256).to("bfloat16").cuda()
    x = mt.randn(64, 256).to("bfloat16").cuda()

    def fn(inp):
        h = ops.linear(inp, w)
        return ops.silu(ops.linear(h, w))

    eager = fn(x).numpy()
    g = Graphed(fn, x)
    out_ptr = g.static_out.data_ptr()
    for _ in range(3):
        y = g(x)
    mt.cuda.synchronize()
    np.testing.assert_array_equal(y.numpy(), eager)
    # allocations outside the graph never receive the graph's blocks
    others = [mt.empty(64, 256, dtype="bfloat16", device="cuda") for _ in range(8)]
    assert out_ptr not in {t.data_ptr() for t in others}
    x2 = mt.randn(64, 256).to("bfloat16").cuda()
    np.testing.assert_array_equal(g(x2).numpy(), fn(x2).numpy())
    del g, y
    gc.collect()


def test_pinned_round_trip():
    h = mt.randn(3, 1000)
    p = h.pin_memory()
    d = p.cuda()
    np.testing.assert_array_equal(d.numpy(), h.numpy())


class _DictStore:
    def __init__(self):
        self.d = {}

    def set(self, k, v):
        self.d[k] = v

    def get(self, k):
        return self.d[k]


def test_nccl_all_gather_single_rank_through_the_c_abi():
    if not _lib.lib().mt_nccl_available():
        pytest.skip("libnccl.so.2 not loadable")
    comm = parallel.NcclCommunicator(0, 1, _DictStore())
    x = mt.randn(2, 4, 8, 8).to("bfloat16").cuda()
    y = comm.all_gather(x)
    mt.cuda.synchronize()
    assert y.shape == (2, 4, 8, 8)
    np.testing.assert_array_equal(y.numpy(), x.numpy())
    comm.close()


def test_library_stream_is_the_tensors_stream():
    t = mt.empty(4, device="cuda")
    assert t._stream() == runtime.current_stream().cuda_stream != 0
