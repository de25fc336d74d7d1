"""the full SD-1.5-shaped UNet (channel multipliers 320/640/1280/1280, 2 ResNet
blocks per level, transformers at the first three levels, 8 heads, 859.5M parameters) in fp32 on
one latent [1, 4, 64, 64] with context [1, 77, 768], one denoising step (UNet + DDIM update).

The whole forward at this size would take the CPU oracle about half an hour, so parity at full
size is checked layer by layer on the tensors the forward actually produced (the wiring is pinned
by the whole-UNet golden test at reduced depth, test_gpu_unet_parity.py): the level-0 self-
attention (4096 tokens, head dim 40, fp32 SIMT kernel) on a subset of its query rows against all
keys, the first up-block ResNet block (2560 -> 1280 channels with the 1x1 shortcut, 8x8) and the
first fused nearest-2x + conv upsampler (1280 channels, 8x8 -> 16x16), all at fp32 rtol 1e-4.
"""
import numpy as np
import pytest

import oracle
import mtorch_b200 as mt
from mtorch_b200 import ops
from mtorch_b200 import unet as U

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def check(name, got, ref, rtol=RTOL):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (name, got.shape, ref.shape)
    e = np.abs(got - ref).max() / np.abs(ref).max()
    print(f"C4 {name}: max|d|/max|ref| = {e:.3e}")
    assert e <= rtol, (name, e)


def npw(t):
    return t.numpy().astype(np.float32)


@pytest.fixture(scope="module")
def c4_run():
    mt.manual_seed(0)
    net = U.UNet(device="cuda", dtype="float32")
    mt.manual_seed(1)
    lat = mt.randn(1, 4, 64, 64).cuda()
    ctx = mt.randn(1, 77, 768).cuda()
    temb = mt.tensor(U.timestep_embedding(np.array([999.0]))).cuda()
    rec = {}

    orig_sdpa = ops.scaled_dot_product_attention

    def sdpa_spy(q, k, v, *a, **kw):
        o = orig_sdpa(q, k, v, *a, **kw)
        if "attn0" not in rec and q.shape[-2] == 4096 and k.shape[-2] == 4096:
            out = kw.get("out", o)
            rec["attn0"] = tuple(t.numpy() for t in (q[:, :, :512], k, v, out[:, :, :512]))
        return o

    def spy(mod, key):
        fwd = mod.forward

        def wrapped(*args):
            y = fwd(*args)
            if key not in rec:
                rec[key] = ([a.numpy() for a in args], y.numpy())
            return y

        mod.forward = wrapped
        return fwd

    up_res, up_samp = net.up[0], next(m for m in net.up if isinstance(m, U.Upsample))
    fr, fu = spy(up_res, "up_res"), spy(up_samp, "up_samp")
    ops.scaled_dot_product_attention = sdpa_spy
    try:
        eps = net(lat, temb, ctx)
        x_next = U.DDIM(steps=50).step(lat, eps, 999)
        out = (eps.numpy(), x_next.numpy())
    finally:
        ops.scaled_dot_product_attention = orig_sdpa
        up_res.forward, up_samp.forward = fr, fu
    # device time of the whole fp32 step (printed; the bench's `--workload c4` reports it)
    ev = [mt.cuda.Event() for _ in range(2)]
    ev[0].record()
    U.DDIM(steps=50).step(lat, net(lat, temb, ctx), 999)
    ev[1].record()
    mt.cuda.synchronize()
    print(f"C4 fp32 UNet step: {ev[0].elapsed_time(ev[1]):.1f} ms")
    return net, rec, out


def test_c4_runs_and_is_finite(c4_run):
    _, rec, (eps, x_next) = c4_run
    assert eps.shape == (1, 4, 64, 64) and x_next.shape == (1, 4, 64, 64)
    assert np.isfinite(eps).all() and np.isfinite(x_next).all()
    assert {"attn0", "up_res", "up_samp"} <= set(rec)


def test_c4_level0_self_attention_rows(c4_run):
    _, rec, _ = c4_run
    q, k, v, o = rec["attn0"]
    check("level-0 self-attention (512 of 4096 query rows)", o, oracle.sdpa_f32(q, k, v))


def _f64_resnet(x, tsilu, blk):
    """The same block in float64 numpy (exact to ~1e-15): GroupNorm with exact sums, im2col convs."""
    def gn(a, w, b):
        n, c = a.shape[:2]
        g = a.reshape(n, 32, -1)
        m, v = g.mean(-1, keepdims=True), g.var(-1, keepdims=True)
        return ((g - m) / np.sqrt(v + 1e-5)).reshape(a.shape) * w[None, :, None, None] + b[None, :, None, None]

    def silu(a):
        return a / (1 + np.exp(-a))

    def conv(a, w, b, pad):
        n, c, hh, ww = a.shape
        k, _, r, s = w.shape
        ap = np.pad(a, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
        cols = np.stack([ap[:, :, i:i + hh, j:j + ww] for i in range(r) for j in range(s)], axis=2)  # n,c,rs,h,w
        cols = cols.reshape(n, c * r * s, hh * ww)
        y = np.einsum("kc,ncp->nkp", w.reshape(k, -1), cols).reshape(n, k, hh, ww)
        return y + b[None, :, None, None]

    d = lambda t: t.numpy().astype(np.float64)  # noqa: E731
    x = x.astype(np.float64)
    h = conv(silu(gn(x, d(blk.norm1.weight), d(blk.norm1.bias))), d(blk.conv1.weight), d(blk.conv1.bias), 1)
    h = h + (tsilu.astype(np.float64) @ d(blk.time_emb_proj.weight).T + d(blk.time_emb_proj.bias))[:, :, None, None]
    h = conv(silu(gn(h, d(blk.norm2.weight), d(blk.norm2.bias))), d(blk.conv2.weight), d(blk.conv2.bias), 1)
    return h + conv(x, d(blk.conv_shortcut.weight), d(blk.conv_shortcut.bias), 0)


def test_c4_up_block_resnet(c4_run):
    """Against the oracle (the reference's arithmetic) and against an exact float64 composition,
    both at the fp32 bar 1e-4: the block's convolutions reduce over K = 23040 and 11520, where the
    fp32 path must add its partial sums in IEEE arithmetic (the split reduction) to stay there."""
    net, rec, _ = c4_run
    blk = net.up[0]
    (h, tsilu, skip), got = rec["up_res"]  # the block's input is cat([h, skip], dim=1)
    x = np.concatenate([h, skip], axis=1)
    assert x.shape == (1, 2560, 8, 8)
    h = oracle.silu_f32(oracle.group_norm_f32(x, 32, npw(blk.norm1.weight), npw(blk.norm1.bias)))
    h = oracle.conv2d_f32(h, npw(blk.conv1.weight), npw(blk.conv1.bias), 1, 1)
    h = h + oracle.linear_f32(tsilu, npw(blk.time_emb_proj.weight), npw(blk.time_emb_proj.bias))[:, :, None, None]
    h = oracle.silu_f32(oracle.group_norm_f32(h, 32, npw(blk.norm2.weight), npw(blk.norm2.bias)))
    h = oracle.conv2d_f32(h, npw(blk.conv2.weight), npw(blk.conv2.bias), 1, 1)
    ref = h + oracle.conv2d_f32(x, npw(blk.conv_shortcut.weight), npw(blk.conv_shortcut.bias))
    exact = _f64_resnet(x, tsilu, blk)
    print(f"C4 oracle (reference arithmetic) vs exact: {np.abs(ref - exact).max() / np.abs(exact).max():.3e}")
    check("up-block ResNet 2560->1280 at 8x8 vs oracle", got, ref)
    check("up-block ResNet 2560->1280 at 8x8 vs exact float64", got, exact)


def test_c4_fused_upsample_conv(c4_run):
    net, rec, _ = c4_run
    m = next(m for m in net.up if isinstance(m, U.Upsample))
    (x,), got = rec["up_samp"]
    assert x.shape == (1, 1280, 8, 8)
    up = x.repeat(2, axis=2).repeat(2, axis=3)
    check("nearest-2x + conv3x3 1280 at 8x8 -> 16x16", got,
          oracle.conv2d_f32(up, npw(m.conv.weight), npw(m.conv.bias), 1, 1))
