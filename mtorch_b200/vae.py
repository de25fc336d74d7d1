"""SD-1.5 VAE decoder (AutoencoderKL decoder shape) on the device path.

The reference has no VAE model; its Stable-Diffusion workload composes the decoder from public
ops (tests/compat/benchmarking.py:6445-6480 the VAE attention block, 6578-6607 the decode head,
6692-6745 the ResNet + nearest-upsample decode block).  This module composes the same ops at
SD-1.5's decoder shape: post-quant 1x1 conv 4->4, conv_in 4->512, a mid block (ResNet, single-head
attention over the 64x64 tokens with head dim 512, ResNet), four up levels of three ResNet blocks
(512, 512, 256, 128 channels) with nearest-2x upsampling after the first three (64 -> 512 pixels),
GroupNorm + SiLU and conv_out 128->3.  GroupNorm eps is 1e-6 throughout, as in SD's VAE.

Layout and fusions follow the UNet: channels-last activations, GroupNorm+SiLU in one kernel, the
shortcut added in conv2's epilogue, nearest-2x upsample fused into its 3x3 conv.  The attention
has head dim 512 (beyond the flash kernels' 256), so it runs as the reference's legacy
composition on the tensor cores: scores = Q K^T * C^-1/2 (batched GEMM, fp32 out), row softmax
(fp32 in, model dtype out), O = P V (batched GEMM), then the output projection with the residual
in its epilogue.
"""
from __future__ import annotations

import math

from . import ops
from .nn import Conv2d, GroupNorm, Linear, Module, ModuleList
from .tensor import Tensor, float32
from .unet import Upsample, _image, _tokens


class VAEResnetBlock(Module):
    def __init__(self, cin, cout, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.norm1 = GroupNorm(32, cin, eps=1e-6, **kw)
        self.conv1 = Conv2d(cin, cout, 3, padding=1, **kw)
        self.norm2 = GroupNorm(32, cout, eps=1e-6, **kw)
        self.conv2 = Conv2d(cout, cout, 3, padding=1, **kw)
        self.conv_shortcut = Conv2d(cin, cout, 1, **kw) if cin != cout else None

    def forward(self, x):
        h = self.conv1(self.norm1(x, fuse_silu=True))
        h = self.norm2(h, fuse_silu=True)
        res = x if self.conv_shortcut is None else self.conv_shortcut(x)
        return self.conv2(h, residual=res)


class VAEAttention(Module):
    """GroupNorm -> single-head self-attention over the H*W tokens -> output projection + x."""

    def __init__(self, c, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.c = c
        self.norm = GroupNorm(32, c, eps=1e-6, **kw)
        self.to_qkv = Linear(c, 3 * c, **kw)
        self.to_out = Linear(c, c, **kw)

    def forward(self, x):
        n, c, hh, ww = x.shape
        s = hh * ww
        t = _tokens(self.norm(x))
        qkv = ops.linear(t, self.to_qkv.weight, self.to_qkv.bias)  # [n*s, 3c]
        p = qkv.stride(0)
        q = qkv[:, 0:c]._view((n, s, c), (s * p, p, 1))
        kt = qkv[:, c:2 * c]._view((n, c, s), (s * p, 1, p))
        v = qkv[:, 2 * c:3 * c]._view((n, s, c), (s * p, p, 1))
        scores = ops.gemm(q, kt, alpha=1.0 / math.sqrt(c), out_dtype=float32)
        probs = ops.softmax(scores, -1, dtype=x.dtype)
        o = ops.gemm(probs, v).reshape(n * s, c)
        t = ops.linear(o, self.to_out.weight, self.to_out.bias, residual=_tokens(x))
        return _image(t, n, hh, ww)


class VAEDecoder(Module):
    """latents [n, 4, h, w] (already divided by the 0.18215 scaling factor) -> images
    [n, 3, 8h, 8w] (NCHW).  Random-init weights with the module defaults."""

    def __init__(self, latent_ch=4, out_ch=3, chans=(128, 256, 512, 512), layers=2, device=None, dtype=None):
        super().__init__()
        kw = dict(device=device, dtype=dtype)
        self.post_quant_conv = Conv2d(latent_ch, latent_ch, 1, **kw)
        top = chans[-1]
        self.conv_in = Conv2d(latent_ch, top, 3, padding=1, **kw)
        self.mid1 = VAEResnetBlock(top, top, **kw)
        self.mid_attn = VAEAttention(top, **kw)
        self.mid2 = VAEResnetBlock(top, top, **kw)
        self.up = ModuleList()
        c = top
        for lvl, co in enumerate(reversed(chans)):
            for _ in range(layers + 1):
                self.up.append(VAEResnetBlock(c, co, **kw))
                c = co
            if lvl != len(chans) - 1:
                self.up.append(Upsample(c, **kw))
        self.norm_out = GroupNorm(32, c, eps=1e-6, **kw)
        self.conv_out = Conv2d(c, out_ch, 3, padding=1, **kw)

    def forward(self, z: Tensor) -> Tensor:
        h = ops.conv2d(z, self.post_quant_conv.weight, self.post_quant_conv.bias, packed=self.post_quant_conv.packed_weight())
        h = ops.conv2d(h, self.conv_in.weight, self.conv_in.bias, 1, 1, packed=self.conv_in.packed_weight(),
                       out_channels_last=True)
        h = self.mid2(self.mid_attn(self.mid1(h)))
        for m in self.up:
            h = m(h)
        h = self.norm_out(h, fuse_silu=True)
        return ops.conv2d(h, self.conv_out.weight, self.conv_out.bias, 1, 1, packed=self.conv_out.packed_weight(),
                          out_channels_last=False)


def vae_decoder_flops(h=64, w=64, chans=(128, 256, 512, 512), layers=2, latent_ch=4, out_ch=3) -> float:
    """Multiply-add FLOPs (2 per MAC) of one decode of a [h, w] latent: convolutions, the mid
    attention's projections and its two S x S products."""
    def conv(cin, cout, k, hh, ww):
        return 2.0 * hh * ww * cin * cout * k * k

    def resnet(cin, cout, hh, ww):
        return conv(cin, cout, 3, hh, ww) + conv(cout, cout, 3, hh, ww) + (conv(cin, cout, 1, hh, ww) if cin != cout
                                                                           else 0.0)
    top = chans[-1]
    s = h * w
    fl = conv(latent_ch, latent_ch, 1, h, w) + conv(latent_ch, top, 3, h, w)
    fl += 2 * resnet(top, top, h, w) + 2.0 * s * top * 4 * top + 4.0 * s * s * top
    c, hh, ww = top, h, w
    for lvl, co in enumerate(reversed(chans)):
        for _ in range(layers + 1):
            fl += resnet(c, co, hh, ww)
            c = co
        if lvl != len(chans) - 1:
            hh, ww = 2 * hh, 2 * ww
            fl += conv(c, c, 3, hh, ww)
    return fl + conv(c, out_ch, 3, hh, ww)
