"""The reference-side binding: adds a `cuda` device to the reference mtorch package itself.

`install(mtorch)` patches an imported reference `mtorch` module in place so that its own public
API reaches this library's kernels:

* `Tensor.to('cuda')` / `Tensor.cuda()` move a reference tensor to the device (an mtorch_b200
  tensor, same values and dtype), and `Module.to('cuda')` moves a reference module's parameters
  and buffers (the reference routes both through `_convert_module_tensor`, mtorch/__init__.py
  3036-3053, and accepts device names listed in `_DEVICE_NAMES`, 2993-2998);
* `mtorch.nn.functional.{conv2d, linear, scaled_dot_product_attention, group_norm, layer_norm,
  silu, gelu, softmax, interpolate}` and `mtorch.{matmul, mm, bmm, addmm, baddbmm, cat, softmax,
  add, sub, mul, div}` run on the device when an argument is a device tensor and call the
  reference's own function otherwise — the reference's nn modules call these names at run time
  (e.g. `Linear.forward` -> `functional.linear`, `Conv2d.forward` -> `functional.conv2d`), so they
  run on the device unchanged;
* factories (`randn`, `rand`, `zeros`, `ones`, `empty`, `full`, `tensor`) given `device='cuda'`
  draw on the reference's own CPU generator and move the result, so seeded values are the
  reference's; `mtorch.cuda` answers with real device queries.

Device ops that this library does not implement raise `NotImplementedError` (never a silent CPU
fallback); a device tensor passed to a reference op that is not routed here fails in the
reference's own argument checks.  This is the Python-level form of the C++ hooks INTEGRATION.md
describes (a device branch at the top of each op function).
"""
from __future__ import annotations

import functools

import numpy as np

from . import ops
from .tensor import Tensor

_FUNCTIONAL = ("conv2d", "linear", "scaled_dot_product_attention", "group_norm", "layer_norm", "silu", "gelu",
               "softmax", "interpolate")
_TOPLEVEL = ("matmul", "mm", "bmm", "addmm", "baddbmm", "cat", "softmax", "add", "sub", "mul", "div")
_FACTORIES = ("randn", "rand", "zeros", "ones", "empty", "full", "tensor")


def _is_cuda(dev) -> bool:
    return dev is not None and str(dev).partition(":")[0] == "cuda"


def _dtype_name(d):
    """Reference dtype objects (str() gives e.g. 'float32') and strings -> this package's names."""
    return None if d is None else str(d).rpartition(".")[2]


def _has_device_tensor(args, kwargs) -> bool:
    for v in (*args, *kwargs.values()):
        if isinstance(v, Tensor):
            return True
        if isinstance(v, (list, tuple)) and any(isinstance(x, Tensor) for x in v):
            return True
    return False


def _device_args(args, kwargs):
    """Reference dtype objects in the arguments become dtype names."""
    def conv(v):
        return _dtype_name(v) if type(v).__name__ == "dtype" else v

    return tuple(conv(a) for a in args), {k: conv(v) for k, v in kwargs.items()}


def _interpolate(x, size=None, scale_factor=None, mode="nearest", align_corners=None, recompute_scale_factor=None,
                 antialias=False):
    """`interpolate` (tensor.cpp:10897) on the device: nearest-neighbour 2x (the SD up block)."""
    sf = scale_factor
    if isinstance(sf, (tuple, list)):
        sf = sf[0] if len(set(sf)) == 1 else None
    if mode == "nearest" and size is None and sf is not None and float(sf) == 2.0 and x.dim() == 4:
        return ops.interpolate_nearest2x(x)
    if mode == "nearest" and size is not None and x.dim() == 4:
        s = tuple(size) if isinstance(size, (tuple, list)) else (size, size)
        if s == (2 * x.shape[2], 2 * x.shape[3]):
            return ops.interpolate_nearest2x(x)
    raise NotImplementedError("interpolate on the cuda device: only mode='nearest' with scale 2")


def _silu(x, inplace=False):
    if inplace:
        raise NotImplementedError("silu(inplace=True) on the cuda device")
    return ops.silu(x)


def _softmax(x, dim=None, _stacklevel=3, dtype=None):
    return ops.softmax(x, -1 if dim is None else dim, dtype=dtype)


def _binary(name):
    def f(a, b, *, alpha=1, out=None):
        if out is not None:
            raise NotImplementedError(f"{name}(out=...) on the cuda device")
        if alpha != 1:
            b = b * alpha
        return {"add": lambda: a + b, "sub": lambda: a - b, "mul": lambda: a * b, "div": lambda: a / b}[name]()
    return f


_DEVICE_IMPL = {
    "conv2d": ops.conv2d, "linear": ops.linear, "scaled_dot_product_attention": ops.scaled_dot_product_attention,
    "group_norm": ops.group_norm, "layer_norm": ops.layer_norm, "silu": _silu, "gelu": ops.gelu,
    "softmax": _softmax, "interpolate": _interpolate, "matmul": ops.matmul, "mm": ops.mm, "bmm": ops.bmm,
    "addmm": ops.addmm, "baddbmm": ops.baddbmm, "cat": ops.cat,
    "add": _binary("add"), "sub": _binary("sub"), "mul": _binary("mul"), "div": _binary("div"),
}


def _dispatch(ref_fn, dev_fn):
    @functools.wraps(ref_fn)
    def f(*args, **kwargs):
        if _has_device_tensor(args, kwargs):
            a, k = _device_args(args, kwargs)
            return dev_fn(*a, **k)
        return ref_fn(*args, **kwargs)

    f.__mtorch_b200_reference__ = ref_fn
    return f


def install(m):
    """Adds the `cuda` device to the reference module `m` (idempotent); returns `m`."""
    if getattr(m, "__mtorch_b200_installed__", False):
        return m
    from . import cuda as _cuda
    from .tensor import tensor as _dev_tensor

    def to_device(t, device, dtype=None):
        arr = np.asarray(t.numpy())
        return _dev_tensor(arr, dtype=_dtype_name(dtype) or _dtype_name(t.dtype)).to(str(device))

    ref_to = m.Tensor.to

    def tensor_to(self, *args, **kwargs):
        dev = kwargs.get("device")
        dtype = kwargs.get("dtype")
        for a in args:
            if isinstance(a, str) or type(a).__name__ == "device":
                dev = a
            elif type(a).__name__ == "dtype":
                dtype = a
        if _is_cuda(dev):
            return to_device(self, dev, dtype)
        return ref_to(self, *args, **kwargs)

    def tensor_cuda(self, device=None, non_blocking=False):
        return tensor_to(self, "cuda" if device is None else (f"cuda:{device}" if isinstance(device, int) else device))

    m.Tensor.to = tensor_to
    m.Tensor.cuda = tensor_cuda

    ref_convert = m._convert_module_tensor

    def convert_module_tensor(value, target_device, target_dtype, target_memory_format):
        if isinstance(value, Tensor):  # already on the device
            if target_device is not None and not _is_cuda(target_device):
                raise NotImplementedError("moving a cuda module back to the cpu is not supported")
            return value.to(_dtype_name(target_dtype)) if target_dtype is not None else value
        if _is_cuda(target_device) and value is not None:
            out = to_device(value, target_device, target_dtype if value.is_floating_point() else None)
            if target_memory_format is not None and "channels_last" in str(target_memory_format) and out.dim() == 4:
                out = out.contiguous(memory_format="channels_last")
            return out
        return ref_convert(value, target_device, target_dtype, target_memory_format)

    m._convert_module_tensor = convert_module_tensor
    names = set(m._DEVICE_NAMES)
    names.add("cuda")
    m._DEVICE_NAMES = names

    F = m.nn.functional
    for name in _FUNCTIONAL:
        setattr(F, name, _dispatch(getattr(F, name), _DEVICE_IMPL[name]))
    for name in _TOPLEVEL:
        if hasattr(m, name):
            setattr(m, name, _dispatch(getattr(m, name), _DEVICE_IMPL[name]))

    def factory(ref_fn):
        @functools.wraps(ref_fn)
        def f(*args, **kwargs):
            dev = kwargs.get("device")
            if _is_cuda(dev):
                kwargs = dict(kwargs)
                kwargs["device"] = "cpu"
                return to_device(ref_fn(*args, **kwargs), dev)
            return ref_fn(*args, **kwargs)
        return f

    for name in _FACTORIES:
        if hasattr(m, name):
            setattr(m, name, factory(getattr(m, name)))
    m.cuda = _cuda
    m.__mtorch_b200_installed__ = True
    return m
