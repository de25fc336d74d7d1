"""mtorch_b200 — the B200 (sm_100a) `cuda` backend for mtorch's Stable-Diffusion hot path.

The public names mirror mtorch's torch-shaped API (mtorch/__init__.py) for the device path:
``Tensor.to('cuda')``, ``nn.Linear/Conv2d/GroupNorm/LayerNorm``, ``nn.functional.*``
(``scaled_dot_product_attention``, ``conv2d``, ``linear``, ``group_norm``, ``layer_norm``,
``softmax``, ``silu``, ``gelu``), ``matmul/bmm/addmm/baddbmm``, ``manual_seed/randn/rand`` (bit-
compatible with mtorch's generator) and ``cuda.*``.  All device compute runs in
``libmtorch_cuda.so`` (hand-written sm_100a kernels behind the C ABI of include/mtorch_cuda.h).
"""
from __future__ import annotations

import contextlib

from . import _lib
from . import runtime as _runtime
from .tensor import (Size, Tensor, add, bfloat16, bool_, device, div, dtype, empty, empty_like, float16, float32,
                     float64, from_numpy, full, int32, int64, mul, ones, sub, tensor, zeros, zeros_like)

float = float32  # noqa: A001  (torch-style aliases)
half = float16
double = float64
long = int64
bool = bool_  # noqa: A001
from .random import Generator, default_generator, initial_seed, manual_seed, rand, randn, randn_like
from .ops import (addmm, baddbmm, bmm, cat, conv2d, gelu, group_norm, layer_norm, linear, log_softmax, matmul, mm,
                  scaled_dot_product_attention, silu, softmax)
from . import nn

channels_last = "channels_last"
contiguous_format = "contiguous_format"


@contextlib.contextmanager
def no_grad():
    yield


@contextlib.contextmanager
def inference_mode(mode=True):
    yield


def is_grad_enabled():
    return False


class _Cuda:
    """``mtorch.cuda`` — real device queries (the reference's stubs return False / 0)."""

    @staticmethod
    def is_available() -> bool:
        try:
            return _lib.lib().mt_cuda_device_count() > 0
        except (ImportError, OSError):
            return False

    @staticmethod
    def device_count() -> int:
        try:
            return _lib.lib().mt_cuda_device_count()
        except (ImportError, OSError):
            return 0

    @staticmethod
    def synchronize(device=None):
        _runtime.synchronize(device)

    @staticmethod
    def is_bf16_supported() -> bool:
        return _Cuda.is_available()

    @staticmethod
    def manual_seed(seed):
        return None

    current_device = staticmethod(_runtime.current_device)
    set_device = staticmethod(_runtime.set_device)
    current_stream = staticmethod(_runtime.current_stream)
    Stream = _runtime.Stream
    Event = _runtime.Event
    memory_stats = staticmethod(_runtime.memory_stats)
    empty_cache = staticmethod(_runtime.empty_cache)


cuda = _Cuda()

__all__ = [n for n in dir() if not n.startswith("_")]
