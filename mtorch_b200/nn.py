"""``mtorch.nn`` modules on the hot path (mtorch/__init__.py:2383-2960, 3306-3532, 4657-4834,
5050-5204), forward-only and device-aware through ``mtorch_b200.ops``.

Default parameter init follows torch (Kaiming-uniform(a=sqrt(5)) weights, U(+-1/sqrt(fan_in))
biases) drawn from mtorch's seeded generator; the reference's own default is a deterministic
arithmetic pattern built from Python lists (mtorch/__init__.py:3330-3332), which parity tests
replace by explicit ``nn.init`` calls or ``copy_``.
"""
from __future__ import annotations

import math
from collections import OrderedDict

from . import _lib as L
from . import ops
from .tensor import Tensor, empty, float32, to_dtype, device as _device


class Parameter(Tensor):
    pass


def _as_param(t: Tensor) -> Tensor:
    t.requires_grad = False  # device path is autograd-free
    return t


class Module:
    def __init__(self):
        object.__setattr__(self, "_parameters", OrderedDict())
        object.__setattr__(self, "_buffers", OrderedDict())
        object.__setattr__(self, "_modules", OrderedDict())
        object.__setattr__(self, "training", True)

    def __setattr__(self, name, value):
        if isinstance(value, Module):
            self._modules[name] = value
        elif isinstance(value, Tensor) and name in getattr(self, "_param_names", ()):
            self._parameters[name] = value
        elif isinstance(value, Tensor) and name in self._parameters:
            self._parameters[name] = value
        object.__setattr__(self, name, value)

    def register_parameter(self, name, t):
        self._parameters[name] = t
        object.__setattr__(self, name, t)

    def register_buffer(self, name, t):
        self._buffers[name] = t
        object.__setattr__(self, name, t)

    def __call__(self, *args, **kwargs):
        return self.forward(*args, **kwargs)

    def forward(self, *args, **kwargs):
        raise NotImplementedError

    def children(self):
        return iter(self._modules.values())

    def modules(self):
        yield self
        for m in self._modules.values():
            yield from m.modules()

    def named_parameters(self, prefix=""):
        for n, p in self._parameters.items():
            if p is not None:
                yield (prefix + n, p)
        for mn, m in self._modules.items():
            yield from m.named_parameters(prefix + mn + ".")

    def parameters(self):
        for _, p in self.named_parameters():
            yield p

    def state_dict(self):
        return OrderedDict(self.named_parameters())

    def load_state_dict(self, sd, strict=True):
        own = dict(self.named_parameters())
        for k, v in sd.items():
            if k in own:
                own[k].copy_(v)
            elif strict:
                raise KeyError(f"unexpected key {k}")
        return self

    def _apply(self, fn):
        for n, p in list(self._parameters.items()):
            if p is not None:
                q = fn(p)
                self._parameters[n] = q
                object.__setattr__(self, n, q)
        for n, b in list(self._buffers.items()):
            if b is not None:
                q = fn(b)
                self._buffers[n] = q
                object.__setattr__(self, n, q)
        for m in self._modules.values():
            m._apply(fn)
        return self

    def to(self, *args, **kwargs):
        """Module.to (mtorch/__init__.py:2848-2904): device and/or floating dtype."""
        return self._apply(lambda t: t.to(*args, **kwargs))

    def cuda(self, index=0):
        return self.to(f"cuda:{index}")

    def cpu(self):
        return self.to("cpu")

    def bfloat16(self):
        return self.to(to_dtype("bfloat16"))

    def half(self):
        return self.to(to_dtype("float16"))

    def float(self):
        return self.to(float32)

    def eval(self):
        for m in self.modules():
            object.__setattr__(m, "training", False)
        return self

    def train(self, mode=True):
        for m in self.modules():
            object.__setattr__(m, "training", mode)
        return self

    def requires_grad_(self, flag=True):
        return self


class Identity(Module):
    def forward(self, x):
        return x


class Sequential(Module):
    def __init__(self, *mods):
        super().__init__()
        for i, m in enumerate(mods):
            self._modules[str(i)] = m

    def forward(self, x):
        for m in self._modules.values():
            x = m(x)
        return x

    def __getitem__(self, i):
        return list(self._modules.values())[i]

    def __len__(self):
        return len(self._modules)


class ModuleList(Module):
    def __init__(self, mods=()):
        super().__init__()
        for m in mods:
            self.append(m)

    def append(self, m):
        self._modules[str(len(self._modules))] = m
        return self

    def __getitem__(self, i):
        return list(self._modules.values())[i]

    def __iter__(self):
        return iter(self._modules.values())

    def __len__(self):
        return len(self._modules)


def _init_linear_like(weight: Tensor, bias: Tensor | None, fan_in: int):
    init.kaiming_uniform_(weight, a=math.sqrt(5))
    if bias is not None:
        bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0.0
        init.uniform_(bias, -bound, bound)


class Linear(Module):
    def __init__(self, in_features, out_features, bias=True, device=None, dtype=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.register_parameter("weight", empty(out_features, in_features, dtype=dtype, device=device))
        self.register_parameter("bias", empty(out_features, dtype=dtype, device=device) if bias else None)
        _init_linear_like(self.weight, self.bias, in_features)

    def forward(self, x):
        return ops.linear(x, self.weight, self.bias)


class Conv2d(Module):
    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1, groups=1, bias=True,
                 padding_mode="zeros", device=None, dtype=None):
        super().__init__()
        if padding_mode != "zeros":
            raise NotImplementedError("only padding_mode='zeros' is supported on the cuda device")
        k = (kernel_size, kernel_size) if isinstance(kernel_size, int) else tuple(kernel_size)
        self.in_channels, self.out_channels, self.kernel_size = in_channels, out_channels, k
        self.stride, self.padding, self.dilation, self.groups = stride, padding, dilation, groups
        self.register_parameter("weight", empty(out_channels, in_channels // groups, *k, dtype=dtype, device=device))
        self.register_parameter("bias", empty(out_channels, dtype=dtype, device=device) if bias else None)
        _init_linear_like(self.weight, self.bias, (in_channels // groups) * k[0] * k[1])
        self._packed = None

    def packed_weight(self):
        """Implicit-GEMM weight layout, rebuilt when the weight tensor or its version changes
        (the reference keeps version-keyed fp16 weight caches the same way, tensor.h:64-78)."""
        w = self.weight
        key = (id(w), w._version, w.dtype.name, str(w.device))
        if w.device.type != "cuda" or self.groups != 1:  # grouped convs take the unpacked weight
            return None
        if self._packed is None or self._packed[0] != key:
            self._packed = (key, ops.pack_conv_weight(w))
        return self._packed[1]

    def forward(self, x, residual=None, bias=None, bias_batch_stride=0):
        return ops.conv2d(x, self.weight, self.bias if bias is None else bias, self.stride, self.padding,
                          self.dilation, self.groups, residual=residual, bias_batch_stride=bias_batch_stride,
                          packed=self.packed_weight())


class GroupNorm(Module):
    def __init__(self, num_groups, num_channels, eps=1e-5, affine=True, device=None, dtype=None):
        super().__init__()
        self.num_groups, self.num_channels, self.eps = num_groups, num_channels, eps
        if affine:
            self.register_parameter("weight", empty(num_channels, dtype=dtype, device=device).fill_(1.0))
            self.register_parameter("bias", empty(num_channels, dtype=dtype, device=device).fill_(0.0))
        else:
            self.weight = self.bias = None

    def forward(self, x, fuse_silu=False):
        return ops.group_norm(x, self.num_groups, self.weight, self.bias, self.eps, fuse_silu=fuse_silu)


class LayerNorm(Module):
    def __init__(self, normalized_shape, eps=1e-5, elementwise_affine=True, bias=True, device=None, dtype=None):
        super().__init__()
        self.normalized_shape = (normalized_shape,) if isinstance(normalized_shape, int) else tuple(normalized_shape)
        self.eps = eps
        if elementwise_affine:
            self.register_parameter("weight", empty(*self.normalized_shape, dtype=dtype, device=device).fill_(1.0))
            self.register_parameter("bias", empty(*self.normalized_shape, dtype=dtype, device=device).fill_(0.0)
                                    if bias else None)
        else:
            self.weight = self.bias = None

    def forward(self, x):
        return ops.layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)


class SiLU(Module):
    def forward(self, x):
        return ops.silu(x)


class GELU(Module):
    def __init__(self, approximate="none"):
        super().__init__()
        self.approximate = approximate

    def forward(self, x):
        return ops.gelu(x, self.approximate)


class Dropout(Module):
    def __init__(self, p=0.5):
        super().__init__()
        self.p = p

    def forward(self, x):
        if self.training and self.p > 0:
            raise NotImplementedError("training-mode dropout is not part of the inference device path")
        return x


class Upsample(Module):
    def __init__(self, scale_factor=2, mode="nearest"):
        super().__init__()
        if scale_factor != 2 or mode != "nearest":
            raise NotImplementedError("only nearest 2x upsampling is implemented on the cuda device")

    def forward(self, x):
        return ops.interpolate_nearest2x(x)


class _Init:
    """``nn.init`` (mtorch/__init__.py:5436-5592) on mtorch's generator."""

    @staticmethod
    def _fans(t: Tensor):
        if t.dim() < 2:
            raise ValueError("Fan in and fan out can not be computed for tensor with fewer than 2 dimensions")
        rf = math.prod(t._shape[2:]) if t.dim() > 2 else 1
        return t._shape[1] * rf, t._shape[0] * rf

    def calculate_gain(self, nonlinearity, param=None):
        if nonlinearity in ("linear", "conv2d", "sigmoid", "conv1d", "conv3d"):
            return 1.0
        if nonlinearity == "tanh":
            return 5.0 / 3
        if nonlinearity == "relu":
            return math.sqrt(2.0)
        if nonlinearity == "leaky_relu":
            slope = 0.01 if param is None else param
            return math.sqrt(2.0 / (1 + slope ** 2))
        raise ValueError(f"Unsupported nonlinearity {nonlinearity}")

    def uniform_(self, t, a=0.0, b=1.0, generator=None):
        return t.uniform_(a, b, generator=generator)

    def normal_(self, t, mean=0.0, std=1.0, generator=None):
        return t.normal_(mean, std, generator=generator)

    def zeros_(self, t):
        return t.fill_(0.0)

    def ones_(self, t):
        return t.fill_(1.0)

    def constant_(self, t, v):
        return t.fill_(v)

    def kaiming_uniform_(self, t, a=0, mode="fan_in", nonlinearity="leaky_relu", generator=None):
        fan_in, fan_out = self._fans(t)
        fan = fan_in if mode == "fan_in" else fan_out
        gain = self.calculate_gain(nonlinearity, a)
        bound = math.sqrt(3.0) * gain / math.sqrt(fan)
        return t.uniform_(-bound, bound, generator=generator)

    def xavier_uniform_(self, t, gain=1.0, generator=None):
        fan_in, fan_out = self._fans(t)
        a = gain * math.sqrt(6.0 / (fan_in + fan_out))
        return t.uniform_(-a, a, generator=generator)


init = _Init()


class _Functional:
    """``nn.functional`` (mtorch/__init__.py:5515-5573) for the device path."""

    linear = staticmethod(ops.linear)
    conv2d = staticmethod(ops.conv2d)
    scaled_dot_product_attention = staticmethod(ops.scaled_dot_product_attention)
    softmax = staticmethod(ops.softmax)
    log_softmax = staticmethod(ops.log_softmax)
    layer_norm = staticmethod(ops.layer_norm)
    group_norm = staticmethod(ops.group_norm)
    silu = staticmethod(ops.silu)
    gelu = staticmethod(ops.gelu)
    relu = staticmethod(ops.relu)
    sigmoid = staticmethod(ops.sigmoid)
    embedding = staticmethod(ops.embedding)

    @staticmethod
    def interpolate(x, size=None, scale_factor=None, mode="nearest", align_corners=None):
        if mode == "nearest" and scale_factor in (2, 2.0) and size is None:
            return ops.interpolate_nearest2x(x)
        if mode == "nearest" and size is not None and tuple(size) == (2 * x.shape[2], 2 * x.shape[3]):
            return ops.interpolate_nearest2x(x)
        raise NotImplementedError("interpolate: only nearest 2x is implemented on the cuda device")


functional = _Functional()
