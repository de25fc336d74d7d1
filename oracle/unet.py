"""Whole-UNet oracle: the SD-style UNet forward + one DDIM step composed from reference-semantics
ops — TEST INFRASTRUCTURE ONLY (imported by tests/ and tests/golden/ scripts, never by the
product).

The reference has no UNet model; its Stable-Diffusion workload is composed from public ops in
its scenario functions (tests/compat/benchmarking.py: ResNet block 5894-5925, spatial transformer
5929-5979, up block with nearest-2x + skip cat 5981-6000, DDIM step 6148-6168, the MiniUNet
pipeline 6879-6920 / 7245-7263).  This module restates the SD-1.5 UNet wiring in those ops,
UNFUSED and in the reference's op order:

  ResnetBlock      h = conv3x3(silu(GN32(x))) + linear(temb_silu)[:, :, None, None]
                   y = conv3x3(silu(GN32(h))) + (x | conv1x1(x))
  SpatialTransf.   t = proj_in(tokens(GN32(x, eps 1e-6)));  t += out1(SDPA(qkv(LN1 t)))
                   t += out2(SDPA(q2(LN2 t), kv2(ctx)));  t += ff_out(value * gelu(gate))
                   y = image(proj_out(t)) + x
  time embedding   temb_silu = silu(lin2(silu(lin1(t_emb))))
  down / mid / up  conv_in, [resnet (+ transformer)] x layers (+ stride-2 conv), mid resnet +
                   transformer + resnet, up: resnet(cat(h, skip)) (+ transformer) x (layers+1)
                   (+ nearest-2x + conv3x3), silu(GN32) -> conv_out

``ops`` is an adapter: ``NumpyOps`` runs the C restatement (oracle/mtorch_oracle.c), and
``ReferenceOps`` runs the reference mtorch itself (built by oracle/build_ref.py), so the same
composition gives the pinned golden (tests/golden/make_golden_unet.py) and the oracle used on the
GPU box.  Parameters come from mtorch's seeded generator (bit-identical in the reference and in
mtorch_b200's host generator), scaled by powers of two so that both sides hold identical values.
"""
from __future__ import annotations

import math

import numpy as np

from . import cfg_ddim_f32, conv2d_f32, gelu_f32, group_norm_f32, layer_norm_f32, linear_f32, sdpa_f32, silu_f32

# the golden configuration: SD-1.5 widths (head dims 40 and 80), three levels, one ResNet block
# per level, attention at the first two, 16x16 latents, batch 2, 77x768 context
GOLDEN_CFG = dict(in_ch=4, out_ch=4, chans=(320, 640, 640), attn=(True, True, False), layers=1, heads=8,
                  ctx_dim=768, batch=2, size=16, ctx_len=77, timestep=601, param_seed=20, input_seed=21)


def param_spec(cfg) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) of every parameter, in the order mtorch_b200.unet.UNet registers them."""
    chans, attn, layers, ctx_dim = cfg["chans"], cfg["attn"], cfg["layers"], cfg["ctx_dim"]
    tdim = chans[0] * 4
    spec: list[tuple[str, tuple[int, ...]]] = []

    def lin(p, i, o, bias=True):
        spec.append((p + ".weight", (o, i)))
        if bias:
            spec.append((p + ".bias", (o,)))

    def conv(p, i, o, k):
        spec.append((p + ".weight", (o, i, k, k)))
        spec.append((p + ".bias", (o,)))

    def norm(p, c):
        spec.append((p + ".weight", (c,)))
        spec.append((p + ".bias", (c,)))

    def resnet(p, i, o):
        norm(p + ".norm1", i)
        conv(p + ".conv1", i, o, 3)
        lin(p + ".time_emb_proj", tdim, o)
        norm(p + ".norm2", o)
        conv(p + ".conv2", o, o, 3)
        if i != o:
            conv(p + ".conv_shortcut", i, o, 1)

    def transformer(p, c):
        norm(p + ".norm", c)
        lin(p + ".proj_in", c, c)
        b = p + ".block"
        norm(b + ".norm1", c)
        lin(b + ".to_qkv", c, 3 * c, bias=False)
        lin(b + ".to_out1", c, c)
        norm(b + ".norm2", c)
        lin(b + ".to_q2", c, c, bias=False)
        lin(b + ".to_kv2", ctx_dim, 2 * c, bias=False)
        lin(b + ".to_out2", c, c)
        norm(b + ".norm3", c)
        lin(b + ".ff.proj", c, 8 * c)
        lin(b + ".ff.out", 4 * c, c)
        lin(p + ".proj_out", c, c)

    lin("time_lin1", chans[0], tdim)
    lin("time_lin2", tdim, tdim)
    conv("conv_in", cfg["in_ch"], chans[0], 3)
    c, i, skip = chans[0], 0, [chans[0]]
    for lvl, co in enumerate(chans):
        for _ in range(layers):
            resnet(f"down.{i}", c, co)
            c = co
            if attn[lvl]:
                transformer(f"down.{i + 1}", c)
            i += 2
            skip.append(c)
        if lvl != len(chans) - 1:
            conv(f"down.{i}.conv", c, c, 3)
            i += 1
            skip.append(c)
    resnet("mid1", c, c)
    transformer("mid_attn", c)
    resnet("mid2", c, c)
    i = 0
    for lvl, co in reversed(list(enumerate(chans))):
        for _ in range(layers + 1):
            resnet(f"up.{i}", c + skip.pop(), co)
            c = co
            if attn[lvl]:
                transformer(f"up.{i + 1}", c)
            i += 2
        if lvl != 0:
            conv(f"up.{i}.conv", c, c, 3)
            i += 1
    norm("norm_out", c)
    conv("conv_out", c, cfg["out_ch"], 3)
    return spec


def _weight_shift(shape) -> int:
    """Weights are N(0,1) * 2^-k with 2^k the power of two nearest sqrt(fan_in)."""
    fan_in = int(np.prod(shape[1:]))
    return int(round(math.log2(math.sqrt(fan_in))))


def make_params(cfg, randn, ops) -> dict:
    """Draws every parameter from ``randn(shape)`` (mtorch's seeded normal generator, already
    seeded by the caller) in ``param_spec`` order:  weights N(0,1)/2^k (2^k ~ sqrt(fan_in)), biases
    N(0,1)/16, norm weights 1 + N(0,1)/8, norm biases N(0,1)/8.  Only power-of-two scalings and
    one correctly rounded fp32 add are applied, so every side gets identical values."""
    P = {}
    for name, shape in param_spec(cfg):
        r = randn(shape)
        is_norm = ".norm" in name or name.startswith("norm")
        if name.endswith(".weight") and len(shape) >= 2:
            P[name] = ops.scale(r, 2.0 ** -_weight_shift(shape))
        elif name.endswith(".weight") and is_norm:
            P[name] = ops.add_scalar(ops.scale(r, 0.125), 1.0)
        elif is_norm:
            P[name] = ops.scale(r, 0.125)
        else:
            P[name] = ops.scale(r, 0.0625)
    return P


def make_inputs(cfg, randn):
    """x [N, 4, S, S] and ctx [N, L, ctx_dim] from the generator (seeded by the caller), and the
    sinusoidal timestep embedding (cos first, fp64 -> fp32) of ``cfg['timestep']``."""
    n, s = cfg["batch"], cfg["size"]
    x = randn((n, cfg["in_ch"], s, s))
    ctx = randn((n, cfg["ctx_len"], cfg["ctx_dim"]))
    half = cfg["chans"][0] // 2
    freqs = np.exp(-math.log(10000.0) * np.arange(half, dtype=np.float64) / half)
    args = np.full(n, float(cfg["timestep"]))[:, None] * freqs[None]
    temb = np.concatenate([np.cos(args), np.sin(args)], axis=1).astype(np.float32)
    return x, ctx, temb


def ddim_alphas(t, steps=50, train_steps=1000, beta_start=0.00085, beta_end=0.012):
    """a_t, a_prev of SD's scaled-linear schedule (benchmarking.py:6138-6141) for DDIM with
    ``steps`` evenly spaced inference steps."""
    betas = np.linspace(beta_start ** 0.5, beta_end ** 0.5, train_steps, dtype=np.float64) ** 2
    ac = np.cumprod(1.0 - betas)
    prev = max(int(t) - train_steps // steps, 0)
    return float(ac[int(t)]), float(ac[prev])


def unet_forward(P, x, temb, ctx, cfg, ops):
    """eps = UNet(x, temb, ctx) composed from ``ops`` (see the module docstring)."""
    chans, attn, layers, heads = cfg["chans"], cfg["attn"], cfg["layers"], cfg["heads"]

    def lin(t, p, bias=True):
        return ops.linear(t, P[p + ".weight"], P[p + ".bias"] if bias else None)

    def gn(t, p, eps=1e-5):
        return ops.group_norm(t, 32, P[p + ".weight"], P[p + ".bias"], eps)

    def conv(t, p, stride=1, pad=1):
        return ops.conv2d(t, P[p + ".weight"], P[p + ".bias"], stride, pad)

    t_silu = ops.silu(lin(ops.silu(lin(temb, "time_lin1")), "time_lin2"))

    def resnet(h, p):
        y = conv(ops.silu(gn(h, p + ".norm1")), p + ".conv1")
        y = ops.add(y, ops.expand_hw(lin(t_silu, p + ".time_emb_proj")))
        y = conv(ops.silu(gn(y, p + ".norm2")), p + ".conv2")
        sc = conv(h, p + ".conv_shortcut", 1, 0) if p + ".conv_shortcut.weight" in P else h
        return ops.add(y, sc)

    def transformer(h, p):
        n, c, hh, ww = ops.shape(h)
        s = hh * ww
        t = lin(ops.tokens(gn(h, p + ".norm", 1e-6)), p + ".proj_in")
        b = p + ".block"

        def attend(q, k, v, sk):
            return ops.merge_heads(ops.sdpa(ops.split_heads(q, n, s, heads), ops.split_heads(k, n, sk, heads),
                                            ops.split_heads(v, n, sk, heads)), n, s)

        y = ops.layer_norm(t, P[b + ".norm1.weight"], P[b + ".norm1.bias"])
        qkv = lin(y, b + ".to_qkv", bias=False)
        a = attend(ops.cols(qkv, 0, c), ops.cols(qkv, c, 2 * c), ops.cols(qkv, 2 * c, 3 * c), s)
        t = ops.add(t, lin(a, b + ".to_out1"))
        y = ops.layer_norm(t, P[b + ".norm2.weight"], P[b + ".norm2.bias"])
        q = lin(y, b + ".to_q2", bias=False)
        sk = ops.shape(ctx)[1]
        kv = lin(ops.flat_rows(ctx), b + ".to_kv2", bias=False)
        a = attend(q, ops.cols(kv, 0, c), ops.cols(kv, c, 2 * c), sk)
        t = ops.add(t, lin(a, b + ".to_out2"))
        y = ops.layer_norm(t, P[b + ".norm3.weight"], P[b + ".norm3.bias"])
        hc = lin(y, b + ".ff.proj")
        g = ops.mul(ops.cols(hc, 0, 4 * c), ops.gelu(ops.cols(hc, 4 * c, 8 * c)))
        t = ops.add(t, lin(g, b + ".ff.out"))
        t = lin(t, p + ".proj_out")
        return ops.add(ops.image(t, n, hh, ww), h)

    h = conv(x, "conv_in")
    skips = [h]
    i = 0
    for lvl in range(len(chans)):
        for _ in range(layers):
            h = resnet(h, f"down.{i}")
            if attn[lvl]:
                h = transformer(h, f"down.{i + 1}")
            i += 2
            skips.append(h)
        if lvl != len(chans) - 1:
            h = conv(h, f"down.{i}.conv", stride=2)
            i += 1
            skips.append(h)
    h = resnet(h, "mid1")
    h = transformer(h, "mid_attn")
    h = resnet(h, "mid2")
    i = 0
    for lvl in reversed(range(len(chans))):
        for _ in range(layers + 1):
            h = resnet(ops.cat_channels(h, skips.pop()), f"up.{i}")
            if attn[lvl]:
                h = transformer(h, f"up.{i + 1}")
            i += 2
        if lvl != 0:
            h = conv(ops.upsample2x(h), f"up.{i}.conv")
            i += 1
    return conv(ops.silu(gn(h, "norm_out")), "conv_out")


def ddim_step(x, eps, t, ops):
    """The reference's DDIM step with the x0 clamp (benchmarking.py:6148-6168)."""
    a_t, a_prev = ddim_alphas(t)
    return ops.ddim(x, eps, a_t, a_prev)


class NumpyOps:
    """The C restatement (numpy arrays in and out)."""

    scale = staticmethod(lambda a, s: (a * np.float32(s)).astype(np.float32))
    add_scalar = staticmethod(lambda a, c: (a + np.float32(c)).astype(np.float32))
    linear = staticmethod(linear_f32)
    silu = staticmethod(silu_f32)
    gelu = staticmethod(gelu_f32)
    add = staticmethod(lambda a, b: (a + b).astype(np.float32))
    mul = staticmethod(lambda a, b: (a * b).astype(np.float32))
    expand_hw = staticmethod(lambda v: v[:, :, None, None])
    shape = staticmethod(lambda a: a.shape)
    tokens = staticmethod(lambda a: np.ascontiguousarray(a.transpose(0, 2, 3, 1).reshape(-1, a.shape[1])))
    image = staticmethod(lambda t, n, h, w: np.ascontiguousarray(t.reshape(n, h, w, -1).transpose(0, 3, 1, 2)))
    cols = staticmethod(lambda a, lo, hi: np.ascontiguousarray(a[:, lo:hi]))
    flat_rows = staticmethod(lambda a: a.reshape(-1, a.shape[-1]))
    cat_channels = staticmethod(lambda a, b: np.concatenate([a, b], axis=1))
    upsample2x = staticmethod(lambda a: np.ascontiguousarray(a.repeat(2, axis=2).repeat(2, axis=3)))
    sdpa = staticmethod(sdpa_f32)

    @staticmethod
    def split_heads(t, n, s, heads):
        return np.ascontiguousarray(t.reshape(n, s, heads, -1).transpose(0, 2, 1, 3))

    @staticmethod
    def merge_heads(o, n, s):
        return np.ascontiguousarray(o.transpose(0, 2, 1, 3).reshape(n * s, -1))

    @staticmethod
    def conv2d(x, w, b, stride, pad):
        return conv2d_f32(x, w, b, stride, pad)

    @staticmethod
    def group_norm(x, groups, w, b, eps):
        return group_norm_f32(x, groups, w, b, eps)

    @staticmethod
    def layer_norm(x, w, b):
        return layer_norm_f32(x, w, b)

    @staticmethod
    def ddim(x, eps, a_t, a_prev):
        # the unguided step is the guided one with equal halves: u + (u - u) * g == u exactly
        return cfg_ddim_f32(x, np.concatenate([eps, eps]), 1.0, a_t, a_prev, clip=True)


class ReferenceOps:
    """The reference mtorch itself (its portable CPU code), through its public API."""

    def __init__(self, mtorch):
        self.m = mtorch
        self.F = mtorch.nn.functional

    def scale(self, a, s):
        return a * s

    def add_scalar(self, a, c):
        return a + c

    def linear(self, x, w, b):
        return self.F.linear(x, w, b)

    def silu(self, x):
        return self.F.silu(x)

    def gelu(self, x):
        return self.F.gelu(x)

    def add(self, a, b):
        return a + b

    def mul(self, a, b):
        return a * b

    def expand_hw(self, v):
        return v.reshape(v.shape[0], v.shape[1], 1, 1)

    def shape(self, a):
        return tuple(a.shape)

    def tokens(self, a):
        return a.permute(0, 2, 3, 1).contiguous().reshape(-1, a.shape[1])

    def image(self, t, n, h, w):
        return t.reshape(n, h, w, t.shape[-1]).permute(0, 3, 1, 2).contiguous()

    def cols(self, a, lo, hi):
        return a[:, lo:hi].contiguous()

    def flat_rows(self, a):
        return a.reshape(-1, a.shape[-1])

    def cat_channels(self, a, b):
        return self.m.cat([a, b], dim=1)

    def upsample2x(self, a):
        return self.F.interpolate(a, scale_factor=2, mode="nearest")

    def sdpa(self, q, k, v):
        return self.F.scaled_dot_product_attention(q, k, v)

    def split_heads(self, t, n, s, heads):
        return t.reshape(n, s, heads, t.shape[-1] // heads).permute(0, 2, 1, 3).contiguous()

    def merge_heads(self, o, n, s):
        return o.permute(0, 2, 1, 3).contiguous().reshape(n * s, -1)

    def conv2d(self, x, w, b, stride, pad):
        return self.F.conv2d(x, w, b, stride, pad)

    def group_norm(self, x, groups, w, b, eps):
        return self.F.group_norm(x, groups, w, b, eps)

    def layer_norm(self, x, w, b):
        return self.F.layer_norm(x, [x.shape[-1]], w, b, 1e-5)

    def ddim(self, x, eps, a_t, a_prev):
        # benchmarking.py:6148-6168 in the reference's own tensor ops
        x0 = (x - eps * math.sqrt(1.0 - a_t)) / math.sqrt(a_t)
        x0 = self.m.clamp(x0, -1.0, 1.0)
        e = (x - x0 * math.sqrt(a_t)) / math.sqrt(1.0 - a_t)
        return x0 * math.sqrt(a_prev) + e * math.sqrt(1.0 - a_prev)
