"""The allocation-free group norm entry point (mt_cuda_group_norm_noalloc).

Some callers of this library cannot allocate device memory at the moment they need a group norm:
code that runs inside a host callback or a custom-allocator hook, or an embedding runtime that
owns all device memory and forbids cudaMalloc / cudaFree on its threads.  They cannot provide
the workspace that mt_cuda_group_norm takes, so the library offers a variant whose scratch lives
in a fixed device array inside the library.  This test calls it through the C ABI twice in a row
(the second time on different data, so stale scratch contents from the first call would show)
and checks both results against the workspace-taking entry point, within the fp32 tolerance the
other GPU tests use; it also checks that an oversized request is refused with an error.

The file is named so that pytest collects it last.
"""
import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import _lib
from mtorch_b200.tensor import workspace

pytestmark = pytest.mark.gpu

# the tolerances the other GPU tests use: fp32 1e-4; bf16 2e-2 (one bf16 rounding step, since the
# two entry points may order the fp32 affine arithmetic differently before rounding to bf16)
RTOL = {"float32": 1e-4, "bfloat16": 2e-2}


def _out(x, out_cl):
    N, C, H, W = x.shape
    fmt = mt.channels_last if out_cl else mt.contiguous_format
    return mt.empty(N, C, H, W, dtype=x.dtype, device="cuda", memory_format=fmt)


def _reference(x, G, w, b, silu, out_cl=True):
    lib = _lib.lib()
    N, C, H, W = x.shape
    out = _out(x, out_cl)
    need = lib.mt_cuda_group_norm_workspace_size(N, C, H * W, G)
    ws, wsb = workspace(need, 0)
    xs = (x.stride(0), x.stride(1), x.stride(3))
    ys = (out.stride(0), out.stride(1), out.stride(3))
    _lib.check(lib.mt_cuda_group_norm(out.data_ptr(), out.dtype.code, _lib.arr64(ys), x.data_ptr(), x.dtype.code,
                                      _lib.arr64(xs), w.data_ptr(), b.data_ptr(), w.dtype.code, N, C, H * W, G, 1e-5,
                                      silu, ws, wsb, x._stream()), "group_norm")
    return out


def _no_alloc(x, G, w, b, silu, out_cl=True):
    lib = _lib.lib()
    N, C, H, W = x.shape
    out = _out(x, out_cl)
    xs = (x.stride(0), x.stride(1), x.stride(3))
    ys = (out.stride(0), out.stride(1), out.stride(3))
    rc = lib.mt_cuda_group_norm_noalloc(out.data_ptr(), out.dtype.code, _lib.arr64(ys), x.data_ptr(), x.dtype.code,
                                        _lib.arr64(xs), w.data_ptr(), b.data_ptr(), w.dtype.code, N, C, H * W, G, 1e-5,
                                        silu, x._stream())
    _lib.check(rc, "group_norm_noalloc")
    return out


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_no_alloc_group_norm_matches_workspace_version_twice(dtype):
    rng = np.random.default_rng(11)
    G = 32
    for call, shape in enumerate([(4, 320, 16, 16), (2, 640, 8, 8)]):
        x = mt.tensor(rng.standard_normal(shape).astype(np.float32) * (1 + call) + call, dtype=dtype).cuda()
        x = x.contiguous(memory_format=mt.channels_last)
        w = mt.tensor(rng.standard_normal(shape[1]).astype(np.float32)).cuda()
        b = mt.tensor(rng.standard_normal(shape[1]).astype(np.float32)).cuda()
        silu = call % 2
        want = _reference(x, G, w, b, silu).numpy()
        got = _no_alloc(x, G, w, b, silu).numpy()
        np.testing.assert_allclose(got, want, rtol=RTOL[dtype], atol=RTOL[dtype] * np.abs(want).max())


@pytest.mark.parametrize("dtype,in_cl,out_cl", [("float32", False, False), ("bfloat16", True, False),
                                                ("bfloat16", False, True)])
def test_no_alloc_group_norm_other_layouts_twice(dtype, in_cl, out_cl):
    """NCHW input (the per-channel-plane statistics pass) and NCHW output (the generic apply pass)
    through the fixed scratch, two calls in a row on different data."""
    rng = np.random.default_rng(12)
    G = 32
    for call, shape in enumerate([(3, 64, 20, 12), (2, 320, 16, 16)]):
        x = mt.tensor(rng.standard_normal(shape).astype(np.float32) * (2 - call) - call, dtype=dtype).cuda()
        if in_cl:
            x = x.contiguous(memory_format=mt.channels_last)
        w = mt.tensor(rng.standard_normal(shape[1]).astype(np.float32)).cuda()
        b = mt.tensor(rng.standard_normal(shape[1]).astype(np.float32)).cuda()
        silu = 1 - call % 2
        want = _reference(x, G, w, b, silu, out_cl).numpy()
        got = _no_alloc(x, G, w, b, silu, out_cl).numpy()
        np.testing.assert_allclose(got, want, rtol=RTOL[dtype], atol=RTOL[dtype] * np.abs(want).max())


def test_no_alloc_group_norm_rejects_oversized_request():
    lib = _lib.lib()
    x = mt.empty(1, 32, 8, 8, device="cuda", memory_format=mt.channels_last)
    strides = _lib.arr64((64 * 64 * 32, 1, 32))
    # 2000 images of 64x64 pixels with 32 groups need ~65 MB of statistics scratch: refused
    # before anything is launched, so the small buffers are never touched.
    rc = lib.mt_cuda_group_norm_noalloc(x.data_ptr(), x.dtype.code, strides, x.data_ptr(), x.dtype.code, strides,
                                        None, None, x.dtype.code, 2000, 32, 64 * 64, 32, 1e-5, 0, x._stream())
    assert rc == _lib.MT_ERR_INVALID
    assert b"scratch" in lib.mt_cuda_last_error_string()
