"""mtorch's seeded generator, bit-compatible with the reference (module.cpp:47-183).

The reference draws SplitMix64 numbers, maps them to (0, 1) doubles and builds normals with the
Marsaglia polar method, keeping the odd "spare" normal across calls.  The host generator lives
in the C ABI (``mt_rng_*``, the same arithmetic compiled with the same libm), so
``manual_seed(0); randn(...)`` reproduces mtorch's values exactly, including the call-order
dependence.  ``uniform_`` on a contiguous cuda tensor is generated ON the device
(``mt_cuda_fill_uniform``): SplitMix64's k-th draw is a pure function of (state, k), so every
element is computed in parallel and the host state is then advanced by the number of draws.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .tensor import Tensor, _new, _CPU, bfloat16, device as _device, float32, float64, to_dtype, _host_assign

_GOLDEN = 0x9E3779B97F4A7C15
_MASK = (1 << 64) - 1


class Generator:
    def __init__(self, device="cpu"):
        self._state = L.RngState()
        self._initial = 0
        L.lib().mt_rng_seed(C.byref(self._state), 0)

    def manual_seed(self, seed):
        seed = int(seed) & _MASK
        L.lib().mt_rng_seed(C.byref(self._state), seed)
        self._initial = seed
        return self

    def initial_seed(self):
        return self._initial


default_generator = Generator()


def manual_seed(seed):
    return default_generator.manual_seed(seed)


def initial_seed():
    return default_generator.initial_seed()


def _gen(g):
    return default_generator if g is None else g


def _host_fill(t: Tensor, fn, *args, generator=None):
    """Fills a host tensor in logical (row-major) order, as the reference does for contiguous
    float32/float64 storage."""
    n = t.numel()
    wide = t.dtype is float64
    buf = np.empty(max(n, 1), dtype=np.float64 if wide else np.float32)
    fn(C.byref(_gen(generator)._state), buf.ctypes.data, L.MT_F64 if wide else L.MT_F32, n, *args)
    _host_assign(t, buf[:n].reshape(t._shape))


def _fill_normal(t: Tensor, mean, std, generator=None):
    if t.device.type == "cpu":
        _host_fill(t, L.lib().mt_rng_fill_normal, float(mean), float(std), generator=generator)
        return
    h = _new(t._shape, t.dtype if t.dtype is not bfloat16 else float32, _CPU)
    _host_fill(h, L.lib().mt_rng_fill_normal, float(mean), float(std), generator=generator)
    t.copy_(h)


def _fill_uniform(t: Tensor, a, b, generator=None):
    if t.device.type == "cuda" and t.is_contiguous():
        g = _gen(generator)
        n = t.numel()
        L.check(L.lib().mt_cuda_fill_uniform(t.data_ptr(), t.dtype.code, n, g._state.state, float(a), float(b),
                                             t._stream()), "uniform_")
        g._state.state = (g._state.state + n * _GOLDEN) & _MASK
        return
    if t.device.type == "cpu":
        _host_fill(t, L.lib().mt_rng_fill_uniform, float(a), float(b), generator=generator)
        return
    h = _new(t._shape, float32, _CPU)
    _host_fill(h, L.lib().mt_rng_fill_uniform, float(a), float(b), generator=generator)
    t.copy_(h)


def _factory(shape, dtype, device):
    from .tensor import _shape_arg

    return _new(_shape_arg(shape), to_dtype(dtype), _device(device) if device is not None else _CPU)


def randn(*shape, dtype=None, device=None, generator=None, requires_grad=False):
    t = _factory(shape, dtype, device)
    return t.normal_(0.0, 1.0, generator=generator)


def rand(*shape, dtype=None, device=None, generator=None, requires_grad=False):
    t = _factory(shape, dtype, device)
    return t.uniform_(0.0, 1.0, generator=generator)


def randn_like(t, dtype=None, device=None):
    return randn(t.shape, dtype=dtype or t.dtype, device=device or t.device)
