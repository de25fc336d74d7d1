"""Tensor, dtype and device objects of the `cuda` backend, mirroring mtorch's Python surface.

The reference keeps tensors as ``Storage`` (a byte vector) plus view metadata
(cpp/mtorch/core/tensor.h:60-126).  Here a tensor is likewise a byte storage plus
(offset, sizes, strides, dtype, device):

* ``cpu`` storage is a numpy array (host memory), used for creation, the seeded generator and
  transfers — compute on CPU tensors stays with mtorch itself and raises here;
* ``cuda`` storage is a device byte buffer from ``libmtorch_cuda.so``'s caching allocator
  (``runtime.DeviceBuffer``), and every byte of compute on it is a kernel of the same library
  called through the C ABI on the device's library stream.

Views (reshape/permute/transpose/narrow/expand/...) are metadata only, exactly like the reference
(``reshape`` tensor.cpp:8584, ``transpose`` 8653, ``permute`` 8680); ``contiguous`` and dtype
casts are device copies (``mt_cuda_copy_strided``).
"""
from __future__ import annotations

import ctypes as C
import math
from typing import Iterable, Sequence

import numpy as np

from . import _lib as L

# ---------------------------------------------------------------------------------------------
# dtypes


class dtype:
    __slots__ = ("name", "itemsize", "code", "np", "is_floating_point")

    def __init__(self, name, itemsize, code, np_dtype, is_float):
        self.name, self.itemsize, self.code, self.np, self.is_floating_point = name, itemsize, code, np_dtype, is_float

    def __repr__(self):
        return f"mtorch.{self.name}"

    def __str__(self):
        return f"mtorch.{self.name}"


float32 = dtype("float32", 4, L.MT_F32, np.float32, True)
bfloat16 = dtype("bfloat16", 2, L.MT_BF16, np.uint16, True)  # host storage: raw bf16 bits
float16 = dtype("float16", 2, L.MT_F16, np.float16, True)
float64 = dtype("float64", 8, L.MT_F64, np.float64, True)
int32 = dtype("int32", 4, L.MT_I32, np.int32, False)
int64 = dtype("int64", 8, L.MT_I64, np.int64, False)
bool_ = dtype("bool", 1, L.MT_BOOL, np.bool_, False)

_BY_NAME = {d.name: d for d in (float32, bfloat16, float16, float64, int32, int64, bool_)}
_BY_NAME.update({"float": float32, "half": float16, "double": float64, "long": int64, "int": int32})


def to_dtype(x) -> dtype:
    """Parses a dtype argument.  Unlike the reference binding's substring match
    (module.cpp:852-867, where "bfloat16" silently became float16), bfloat16 is recognised
    first and unknown names raise."""
    if x is None:
        return float32
    if isinstance(x, dtype):
        return x
    s = str(x).replace("torch.", "").replace("mtorch.", "")
    if "bfloat16" in s:
        return bfloat16
    if s in _BY_NAME:
        return _BY_NAME[s]
    raise TypeError(f"unsupported dtype {x!r}")


def _promote(a: dtype, b: dtype) -> dtype:
    if a is b:
        return a
    order = [bool_, int32, int64, float16, bfloat16, float32, float64]
    if {a, b} == {float16, bfloat16}:
        return float32
    return a if order.index(a) > order.index(b) else b


# ---------------------------------------------------------------------------------------------
# devices


class device:
    __slots__ = ("type", "index")

    def __init__(self, spec="cpu", index=None):
        if isinstance(spec, device):
            self.type, self.index = spec.type, spec.index
            return
        s = str(spec)
        if s.startswith("cuda"):
            self.type = "cuda"
            self.index = int(s.split(":")[1]) if ":" in s else (index if index is not None else 0)
        elif s.startswith("cpu"):
            self.type, self.index = "cpu", None
        elif s.startswith("mps"):
            raise NotImplementedError("Metal device execution is not implemented")
        else:
            raise RuntimeError(f"Expected one of cpu, cuda device type at start of device string: {s}")

    def __eq__(self, other):
        other = device(other)
        return self.type == other.type and (self.index or 0) == (other.index or 0)

    def __hash__(self):
        return hash((self.type, self.index))

    def __repr__(self):
        return f"device(type='{self.type}'" + (f", index={self.index})" if self.index is not None else ")")

    def __str__(self):
        return self.type if self.index is None else f"{self.type}:{self.index}"


_CPU = device("cpu")

# ---------------------------------------------------------------------------------------------
# device memory, streams and workspaces: the library's own device runtime (runtime.py)

from . import runtime as _rt  # noqa: E402
from .runtime import DeviceBuffer, _ensure_device, stream_ptr  # noqa: E402


def _alloc(nbytes: int, idx: int) -> DeviceBuffer:
    return DeviceBuffer(nbytes, idx)


_WS: dict = {}
_WS_RETIRED: list = []


def workspace(nbytes: int, idx: int):
    """Per-device scratch buffer handed to the kernels (grown on demand, reused in stream order)."""
    if nbytes <= 0:
        return None, 0
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        if buf is not None and idx in _rt.capturing:
            _WS_RETIRED.append(buf)  # kernels captured earlier in this graph still use it
        buf = _alloc(int(nbytes * 1.25) + 4096, idx)
        _WS[idx] = buf
    return buf.data_ptr(), buf.numel()


# ---------------------------------------------------------------------------------------------
# host bf16 conversion (round to nearest even)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32)
    rounded = bits + (((bits >> 16) & 1) + 0x7FFF)
    out = (rounded >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _contig_strides(shape: Sequence[int]) -> tuple:
    st, acc = [], 1
    for s in reversed(shape):
        st.append(acc)
        acc *= max(int(s), 1)
    return tuple(reversed(st))


class _NoGrad:
    enabled = True


# ---------------------------------------------------------------------------------------------


class Size(tuple):
    def numel(self):
        return math.prod(self)


class Tensor:
    """A strided view over host or device bytes (see module docstring)."""

    __slots__ = ("_buf", "_offset", "_shape", "_strides", "dtype", "device", "_version", "requires_grad", "grad",
                 "_cache", "__weakref__")

    def __init__(self, buf, offset, shape, strides, dt, dev):
        self._buf = buf
        self._offset = int(offset)
        self._shape = tuple(int(s) for s in shape)
        self._strides = tuple(int(s) for s in strides)
        self.dtype = dt
        self.device = dev
        self._version = 0
        self.requires_grad = False
        self.grad = None
        self._cache = None

    # ---- metadata -----------------------------------------------------------------------
    @property
    def shape(self):
        return Size(self._shape)

    def size(self, dim=None):
        return Size(self._shape) if dim is None else self._shape[dim]

    def stride(self, dim=None):
        return self._strides if dim is None else self._strides[dim]

    def dim(self):
        return len(self._shape)

    ndim = property(dim)

    def numel(self):
        return math.prod(self._shape)

    def element_size(self):
        return self.dtype.itemsize

    @property
    def is_cuda(self):
        return self.device.type == "cuda"

    def is_contiguous(self, memory_format=None):
        if memory_format is not None and "channels_last" in str(memory_format):
            if self.dim() != 4:
                return False
            n, c, h, w = self._shape
            want = (h * w * c, 1, w * c, c)
            return all(s == 1 or st == ws for s, st, ws in zip(self._shape, self._strides, want))
        exp = _contig_strides(self._shape)
        return all(s == 1 or a == b for s, a, b in zip(self._shape, self._strides, exp))

    def data_ptr(self):
        if self.device.type == "cuda":
            return self._buf.data_ptr() + self._offset * self.dtype.itemsize
        return self._buf.ctypes.data + self._offset * self.dtype.itemsize

    def _idx(self):
        return self.device.index or 0

    def _stream(self):
        return stream_ptr(self._idx())

    def __repr__(self):
        return f"mtorch.Tensor(shape={tuple(self._shape)}, dtype={self.dtype.name}, device={self.device})"

    def __len__(self):
        return self._shape[0]

    # ---- views ----------------------------------------------------------------------------
    def _view(self, shape, strides, offset=None):
        t = Tensor(self._buf, self._offset if offset is None else offset, shape, strides, self.dtype, self.device)
        return t

    def as_strided(self, size, stride, storage_offset=None):
        return self._view(size, stride, storage_offset)

    def view(self, *shape):
        shape = _shape_arg(shape)
        shape = _infer(shape, self.numel())
        if not self.is_contiguous():
            raise RuntimeError("view size is not compatible with input tensor's size and stride; use .reshape(...)")
        return self._view(shape, _contig_strides(shape))

    def reshape(self, *shape):
        shape = _infer(_shape_arg(shape), self.numel())
        t = self if self.is_contiguous() else self.contiguous()
        return t._view(shape, _contig_strides(shape))

    def flatten(self, start_dim=0, end_dim=-1):
        nd = self.dim()
        s, e = start_dim % max(nd, 1), end_dim % max(nd, 1)
        shape = self._shape[:s] + (math.prod(self._shape[s:e + 1]),) + self._shape[e + 1:]
        return self.reshape(shape)

    def permute(self, *dims):
        dims = [d % self.dim() for d in _shape_arg(dims)]
        return self._view([self._shape[d] for d in dims], [self._strides[d] for d in dims])

    def transpose(self, a, b):
        dims = list(range(self.dim()))
        a, b = a % self.dim(), b % self.dim()
        dims[a], dims[b] = dims[b], dims[a]
        return self.permute(dims)

    @property
    def T(self):
        return self.permute(list(reversed(range(self.dim()))))

    def t(self):
        return self.transpose(0, 1) if self.dim() == 2 else self

    def unsqueeze(self, d):
        d = d % (self.dim() + 1)
        st = self._strides[d] * self._shape[d] if d < self.dim() else 1
        return self._view(self._shape[:d] + (1,) + self._shape[d:], self._strides[:d] + (st,) + self._strides[d:])

    def squeeze(self, d=None):
        if d is None:
            keep = [i for i, s in enumerate(self._shape) if s != 1]
        else:
            d = d % self.dim()
            keep = [i for i in range(self.dim()) if i != d or self._shape[i] != 1]
        return self._view([self._shape[i] for i in keep], [self._strides[i] for i in keep])

    def expand(self, *shape):
        shape = list(_shape_arg(shape))
        nd = len(shape)
        src_shape = (1,) * (nd - self.dim()) + self._shape
        src_st = (0,) * (nd - self.dim()) + self._strides
        out_st = []
        for i in range(nd):
            if shape[i] == -1:
                shape[i] = src_shape[i]
            if src_shape[i] == shape[i]:
                out_st.append(src_st[i])
            elif src_shape[i] == 1:
                out_st.append(0)
            else:
                raise RuntimeError(f"cannot expand {self._shape} to {tuple(shape)}")
        return self._view(shape, out_st)

    def expand_as(self, other):
        return self.expand(other.shape)

    def narrow(self, dim, start, length):
        dim = dim % self.dim()
        shape = list(self._shape)
        shape[dim] = length
        return self._view(shape, self._strides, self._offset + start * self._strides[dim])

    def select(self, dim, index):
        dim = dim % self.dim()
        index = index % self._shape[dim]
        return self._view(self._shape[:dim] + self._shape[dim + 1:], self._strides[:dim] + self._strides[dim + 1:],
                          self._offset + index * self._strides[dim])

    def __getitem__(self, idx):
        if not isinstance(idx, tuple):
            idx = (idx,)
        if any(it is Ellipsis for it in idx):
            e = next(i for i, it in enumerate(idx) if it is Ellipsis)
            used = sum(1 for it in idx if it is not None and it is not Ellipsis)
            idx = idx[:e] + (slice(None),) * (self.dim() - used) + idx[e + 1:]
        t, dim = self, 0
        for it in idx:
            if it is None:
                t = t.unsqueeze(dim)
                dim += 1
            elif isinstance(it, int):
                t = t.select(dim, it)
            elif isinstance(it, slice):
                start, stop, step = it.indices(t._shape[dim])
                n = max(0, (stop - start + step - 1) // step)
                shape = list(t._shape)
                strides = list(t._strides)
                shape[dim] = n
                off = t._offset + start * strides[dim]
                strides[dim] *= step
                t = t._view(shape, strides, off)
                dim += 1
            else:
                raise NotImplementedError("advanced indexing is not supported on the cuda backend")
        return t

    def chunk(self, chunks, dim=0):
        dim = dim % self.dim()
        n = self._shape[dim]
        step = -(-n // chunks)
        return tuple(self.narrow(dim, s, min(step, n - s)) for s in range(0, n, step))

    def split(self, size, dim=0):
        dim = dim % self.dim()
        n = self._shape[dim]
        if isinstance(size, int):
            return tuple(self.narrow(dim, s, min(size, n - s)) for s in range(0, n, size))
        out, s = [], 0
        for k in size:
            out.append(self.narrow(dim, s, k))
            s += k
        return tuple(out)

    # ---- copies / transfers ---------------------------------------------------------------
    def contiguous(self, memory_format=None):
        if memory_format is not None and "channels_last" in str(memory_format):
            if self.is_contiguous(memory_format):
                return self
            return _copy_to_layout(self, "channels_last")
        if self.is_contiguous():
            return self
        return _copy_to_layout(self, "contiguous")

    def clone(self):
        return _copy_to_layout(self, "contiguous", force=True)

    def to(self, *args, **kwargs):
        dev, dt, memory_format = None, None, kwargs.get("memory_format")
        if kwargs.get("dtype") is not None:
            dt = to_dtype(kwargs["dtype"])
        for a in list(args) + [kwargs.get("device")]:
            if a is None:
                continue
            if isinstance(a, Tensor):
                dev, dt = a.device, a.dtype
            elif isinstance(a, dtype) or "float" in str(a) or "bfloat" in str(a) or "int" in str(a):
                dt = to_dtype(a)
            else:
                dev = device(a)
        t = self
        if dev is not None and dev != t.device:
            t = _transfer(t, dev)
        if dt is not None and dt is not t.dtype:
            t = _cast(t, dt)
        if memory_format is not None:
            t = t.contiguous(memory_format=memory_format)
        return t

    def cuda(self, index=None):
        return self.to(device("cuda", index if index is not None else 0) if not isinstance(index, str) else index)

    def cpu(self):
        return self.to("cpu")

    def pin_memory(self):
        """A contiguous copy of this CPU tensor in page-locked host memory (asynchronous
        host<->device copies from / into it overlap with the device)."""
        if self.device.type != "cpu":
            raise RuntimeError("cannot pin a cuda tensor: only CPU tensors live in host memory")
        src = self.contiguous()
        buf = _rt.pinned_array(src.numel(), src._buf.dtype)
        buf[:src.numel()] = src._buf[src._offset:src._offset + src.numel()]
        return Tensor(buf, 0, src._shape, _contig_strides(src._shape), src.dtype, src.device)

    def float(self):
        return self.to(float32)

    def half(self):
        return self.to(float16)

    def bfloat16(self):
        return self.to(bfloat16)

    def double(self):
        return self.to(float64)

    def numpy(self):
        t = self.cpu().contiguous()
        a = t._buf[t._offset:t._offset + t.numel()].reshape(t._shape)
        if t.dtype is bfloat16:
            return bf16_bits_to_f32(a).reshape(t._shape)
        return a

    def tolist(self):
        return self.numpy().tolist()

    def item(self):
        return self.numpy().reshape(-1)[0].item()

    def detach(self):
        return self

    def requires_grad_(self, flag=True):
        self.requires_grad = flag
        return self

    # ---- in-place initialisers (used by nn.init) -----------------------------------------
    def _mark_modified(self):
        self._version += 1
        self._cache = None

    def copy_(self, src):
        src = src if isinstance(src, Tensor) else tensor(src)
        if src.device != self.device:
            src = _transfer(src, self.device)
        if self.device.type == "cpu":
            s = src.numpy() if src.dtype is bfloat16 else src.numpy()
            _host_assign(self, np.broadcast_to(s, self._shape))
        else:
            src = src.expand(self._shape)
            L.check(L.lib().mt_cuda_copy_strided(
                self.data_ptr(), self.dtype.code, L.arr64(self._strides), src.data_ptr(), src.dtype.code,
                L.arr64(src._strides), L.arr64(self._shape), self.dim(), self._stream()), "copy_")
        self._mark_modified()
        return self

    def fill_(self, value):
        if self.device.type == "cpu":
            _host_assign(self, np.full(self._shape, value, dtype=np.float64))
        elif self.is_contiguous():
            L.check(L.lib().mt_cuda_fill(self.data_ptr(), self.dtype.code, self.numel(), float(value),
                                          self._stream()), "fill_")
        else:
            self.copy_(full(self._shape, value, dtype=self.dtype, device=self.device))
        self._mark_modified()
        return self

    def zero_(self):
        return self.fill_(0.0)

    def normal_(self, mean=0.0, std=1.0, generator=None):
        from .random import _fill_normal

        _fill_normal(self, mean, std, generator)
        self._mark_modified()
        return self

    def uniform_(self, a=0.0, b=1.0, generator=None):
        from .random import _fill_uniform

        _fill_uniform(self, a, b, generator)
        self._mark_modified()
        return self

    # ---- arithmetic ---------------------------------------------------------------------
    def __add__(self, o):
        return add(self, o)

    def __radd__(self, o):
        return add(self, o)

    def __sub__(self, o):
        return sub(self, o)

    def __rsub__(self, o):
        return add(mul(self, -1.0), o)

    def __mul__(self, o):
        return mul(self, o)

    def __rmul__(self, o):
        return mul(self, o)

    def __truediv__(self, o):
        return div(self, o)

    def __neg__(self):
        return mul(self, -1.0)

    def __matmul__(self, o):
        from .ops import matmul

        return matmul(self, o)

    def __iadd__(self, o):
        return _binary_into(self, self, o, "add")

    def __imul__(self, o):
        return _binary_into(self, self, o, "mul")

    def add_(self, o, alpha=1.0):
        if alpha != 1.0:
            o = mul(o, alpha)
        return _binary_into(self, self, o, "add")

    def mul_(self, o):
        return _binary_into(self, self, o, "mul")

    def add(self, o, alpha=1.0):
        return add(self, o if alpha == 1.0 else mul(o, alpha))

    def mul(self, o):
        return mul(self, o)

    def sub(self, o):
        return sub(self, o)

    def div(self, o):
        return div(self, o)

    def matmul(self, o):
        from .ops import matmul

        return matmul(self, o)

    def softmax(self, dim, dtype=None):
        from .ops import softmax

        return softmax(self, dim, dtype=dtype)


def _shape_arg(shape):
    if len(shape) == 1 and isinstance(shape[0], (tuple, list, Size)):
        return tuple(shape[0])
    return tuple(shape)


def _infer(shape, numel):
    shape = list(shape)
    if -1 in shape:
        i = shape.index(-1)
        rest = math.prod(s for j, s in enumerate(shape) if j != i)
        shape[i] = numel // rest if rest else 0
    if math.prod(shape) != numel:
        raise RuntimeError(f"shape {tuple(shape)} is invalid for input of size {numel}")
    return tuple(shape)


def _host_assign(t: Tensor, values: np.ndarray) -> None:
    view = np.lib.stride_tricks.as_strided(
        t._buf[t._offset:], shape=t._shape, strides=[s * t._buf.itemsize for s in t._strides])
    if t.dtype is bfloat16:
        view[...] = f32_to_bf16_bits(np.asarray(values, dtype=np.float32))
    else:
        view[...] = values


# ---------------------------------------------------------------------------------------------
# creation


def _new(shape, dt: dtype, dev: device, channels_last=False) -> Tensor:
    shape = tuple(int(s) for s in shape)
    n = math.prod(shape)
    if channels_last and len(shape) == 4:
        nb, c, h, w = shape
        strides = (h * w * c, 1, w * c, c)
    else:
        strides = _contig_strides(shape)
    if dev.type == "cpu":
        buf = np.zeros(max(n, 1), dtype=dt.np)
    else:
        buf = _alloc(n * dt.itemsize, dev.index or 0)
    return Tensor(buf, 0, shape, strides, dt, dev)


def empty(*shape, dtype=None, device=None, memory_format=None, requires_grad=False):
    dev = _CPU if device is None else globals()["device"](device)
    return _new(_shape_arg(shape), to_dtype(dtype), dev, channels_last=memory_format is not None and
                "channels_last" in str(memory_format))


def zeros(*shape, dtype=None, device=None, requires_grad=False):
    t = empty(*shape, dtype=dtype, device=device)
    if t.device.type == "cuda":
        L.check(L.lib().mt_cuda_memset(t.data_ptr(), 0, t.numel() * t.dtype.itemsize, t._stream()), "zeros")
    return t


def ones(*shape, dtype=None, device=None, requires_grad=False):
    return full(_shape_arg(shape), 1.0, dtype=dtype, device=device)


def full(shape, value, dtype=None, device=None):
    t = empty(*_shape_arg((shape,)), dtype=dtype, device=device)
    return t.fill_(value)


def empty_like(t, dtype=None, device=None):
    return empty(t.shape, dtype=dtype or t.dtype, device=device or t.device)


def zeros_like(t, dtype=None, device=None):
    return zeros(t.shape, dtype=dtype or t.dtype, device=device or t.device)


def from_numpy(a: np.ndarray) -> Tensor:
    a = np.ascontiguousarray(a)
    dt = {np.dtype(np.float32): float32, np.dtype(np.float64): float64, np.dtype(np.float16): float16,
          np.dtype(np.int32): int32, np.dtype(np.int64): int64, np.dtype(np.bool_): bool_}[a.dtype]
    return Tensor(a.reshape(-1).copy() if a.size else np.zeros(1, a.dtype), 0, a.shape,
                  _contig_strides(a.shape), dt, _CPU)


def tensor(data, dtype=None, device=None, requires_grad=False):
    if isinstance(data, Tensor):
        t = data
    else:
        arr = np.asarray(data)
        if dtype is None:
            dt = float32 if arr.dtype.kind == "f" else (int64 if arr.dtype.kind in "iu" else (
                bool_ if arr.dtype.kind == "b" else float32))
        else:
            dt = to_dtype(dtype)
        if dt is bfloat16:
            bits = f32_to_bf16_bits(arr.astype(np.float32))
            t = Tensor(bits.reshape(-1) if bits.size else np.zeros(1, np.uint16), 0, arr.shape,
                       _contig_strides(arr.shape), bfloat16, _CPU)
        else:
            t = from_numpy(arr.astype(dt.np))
    if dtype is not None and to_dtype(dtype) is not t.dtype:
        t = t.to(to_dtype(dtype))
    if device is not None:
        t = t.to(device)
    return t


# ---------------------------------------------------------------------------------------------
# copies, transfers, casts


def _copy_to_layout(t: Tensor, layout: str, force=False, dt: dtype | None = None) -> Tensor:
    dt = dt or t.dtype
    if t.device.type == "cpu":
        a = _host_array(t)
        out = tensor(a.astype(np.float32) if dt is bfloat16 else a.astype(dt.np), dtype=dt)
        if layout == "channels_last":
            raise NotImplementedError("channels_last host tensors are not supported")
        return out
    out = _new(t._shape, dt, t.device, channels_last=(layout == "channels_last"))
    L.check(L.lib().mt_cuda_copy_strided(out.data_ptr(), dt.code, L.arr64(out._strides), t.data_ptr(), t.dtype.code,
                                         L.arr64(t._strides), L.arr64(t._shape), t.dim(), t._stream()),
            "contiguous")
    return out


def _host_array(t: Tensor) -> np.ndarray:
    """numpy view of a host tensor's values (bf16 widened to float32)."""
    if t.numel() == 0:
        return np.zeros(t._shape, dtype=np.float32 if t.dtype is bfloat16 else t.dtype.np)
    v = np.lib.stride_tricks.as_strided(t._buf[t._offset:], shape=t._shape,
                                        strides=[s * t._buf.itemsize for s in t._strides])
    if t.dtype is bfloat16:
        return bf16_bits_to_f32(np.ascontiguousarray(v)).reshape(t._shape)
    return np.ascontiguousarray(v)


def _transfer(t: Tensor, dev: device) -> Tensor:
    lib = L.lib()
    if t.device.type == "cpu" and dev.type == "cuda":
        a = np.ascontiguousarray(
            np.lib.stride_tricks.as_strided(t._buf[t._offset:], shape=t._shape,
                                            strides=[s * t._buf.itemsize for s in t._strides])
            if t.numel() else np.zeros(0, t._buf.dtype))
        out = _new(t._shape, t.dtype, dev)
        L.check(lib.mt_cuda_memcpy(out.data_ptr(), a.ctypes.data, a.nbytes, 0, out._stream()), "to(cuda)")
        L.check(lib.mt_cuda_synchronize(out._stream()), "to(cuda)")  # host array may be freed after return
        return out
    if t.device.type == "cuda" and dev.type == "cpu":
        src = t.contiguous()
        out = _new(t._shape, t.dtype, _CPU)
        nbytes = t.numel() * t.dtype.itemsize
        L.check(lib.mt_cuda_memcpy(out._buf.ctypes.data, src.data_ptr(), nbytes, 1, src._stream()), "to(cpu)")
        L.check(lib.mt_cuda_synchronize(src._stream()), "to(cpu)")
        return out
    if t.device.type == "cuda" and dev.type == "cuda":
        return _transfer(_transfer(t, _CPU), dev)
    return t


def _cast(t: Tensor, dt: dtype) -> Tensor:
    if t.device.type == "cpu":
        a = _host_array(t)
        return tensor(a, dtype=dt)
    return _copy_to_layout(t, "contiguous" if not t.is_contiguous("channels_last") or t.is_contiguous()
                           else "channels_last", dt=dt)


# ---------------------------------------------------------------------------------------------
# broadcast binary ops (binary_tensor_tensor / binary_tensor_scalar, tensor.cpp:18965-19106)


def _broadcast_shape(a, b):
    nd = max(len(a), len(b))
    a = (1,) * (nd - len(a)) + tuple(a)
    b = (1,) * (nd - len(b)) + tuple(b)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise RuntimeError(f"The size of tensor a ({x}) must match the size of tensor b ({y})")
        out.append(max(x, y) if x and y else 0)
    return tuple(out)


def _require_cuda(*ts):
    for t in ts:
        if isinstance(t, Tensor) and t.device.type != "cuda":
            raise NotImplementedError(
                "mtorch_b200 computes on the cuda device only; CPU compute is mtorch's own CPU backend "
                "(no silent fallback)")


def _binary_into(out: Tensor | None, a, b, op: str):
    if not isinstance(a, Tensor):
        a, b = b, a
        if op in ("sub", "div"):
            raise NotImplementedError("scalar-left sub/div")
    _require_cuda(a, b)
    if isinstance(b, Tensor):
        shape = _broadcast_shape(a._shape, b._shape)
        dt = _promote(a.dtype, b.dtype)
    else:
        shape = a._shape
        dt = a.dtype
    if out is None:
        out = _new(shape, dt, a.device, channels_last=a.is_contiguous("channels_last") and not a.is_contiguous()
                   and len(shape) == 4)
    elif tuple(out._shape) != tuple(shape):
        raise RuntimeError(f"output with shape {out._shape} doesn't match the broadcast shape {shape}")
    ae = a.expand(shape)
    if isinstance(b, Tensor):
        be = b.expand(shape)
        bp, bd, bs, sc = be.data_ptr(), be.dtype.code, L.arr64(be._strides), 0.0
    else:
        bp, bd, bs, sc = None, a.dtype.code, None, float(b)
    L.check(L.lib().mt_cuda_binary(L.BINARY[op], out.data_ptr(), out.dtype.code, L.arr64(out._strides),
                                   ae.data_ptr(), ae.dtype.code, L.arr64(ae._strides), bp, bd, bs, sc,
                                   L.arr64(shape), len(shape), a._stream()), op)
    out._mark_modified()
    return out


def add(a, b, alpha=1.0):
    if alpha != 1.0:
        b = mul(b, alpha)
    return _binary_into(None, a, b, "add")


def sub(a, b):
    return _binary_into(None, a, b, "sub")


def mul(a, b):
    return _binary_into(None, a, b, "mul")


def div(a, b):
    return _binary_into(None, a, b, "div")
