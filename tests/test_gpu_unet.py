"""UNet building blocks on the device vs the oracle composed op by op (fp32, rtol 1e-4), the DDIM
update vs the reference formula, and batch-position independence of the whole UNet (the property
the multi-GPU batch sharding relies on: bitwise equal results)."""
import numpy as np
import pytest

import oracle
import mtorch_b200 as mt
from mtorch_b200 import unet as U

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def check(got, ref, rtol=RTOL):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(ref, np.float64), rtol=rtol,
                               atol=rtol * np.abs(ref).max())


def npw(t):
    return t.numpy().astype(np.float32)


def cl(a):
    return mt.tensor(a).cuda().contiguous(memory_format=mt.channels_last)


def test_resnet_block_fp32():
    mt.manual_seed(3)
    blk = U.ResnetBlock(64, 128, temb=96, device="cuda")
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 64, 8, 8)).astype(np.float32)
    te = rng.standard_normal((2, 96)).astype(np.float32)
    got = blk(cl(x), mt.tensor(te).cuda()).numpy()
    h = oracle.silu_f32(oracle.group_norm_f32(x, 32, npw(blk.norm1.weight), npw(blk.norm1.bias)))
    h = oracle.conv2d_f32(h, npw(blk.conv1.weight), npw(blk.conv1.bias), 1, 1)
    h = h + oracle.linear_f32(te, npw(blk.time_emb_proj.weight), npw(blk.time_emb_proj.bias))[:, :, None, None]
    h = oracle.silu_f32(oracle.group_norm_f32(h, 32, npw(blk.norm2.weight), npw(blk.norm2.bias)))
    h = oracle.conv2d_f32(h, npw(blk.conv2.weight), npw(blk.conv2.bias), 1, 1)
    ref = h + oracle.conv2d_f32(x, npw(blk.conv_shortcut.weight), npw(blk.conv_shortcut.bias))
    check(got, ref)


def test_spatial_transformer_fp32():
    mt.manual_seed(4)
    st = U.SpatialTransformer(64, heads=2, ctx_dim=48, device="cuda")
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 64, 6, 6)).astype(np.float32)
    ctx = rng.standard_normal((2, 7, 48)).astype(np.float32)
    got = st(cl(x), mt.tensor(ctx).cuda()).numpy()
    b = st.block
    n, c, s = 2, 64, 36
    t = oracle.group_norm_f32(x, 32, npw(st.norm.weight), npw(st.norm.bias), eps=1e-6)
    t = t.transpose(0, 2, 3, 1).reshape(n * s, c)
    t = oracle.linear_f32(t, npw(st.proj_in.weight), npw(st.proj_in.bias))

    def attn(q, k, v, sq, sk):
        heads = lambda a, L: a.reshape(n, L, 2, c // 2).transpose(0, 2, 1, 3)  # noqa: E731
        o = oracle.sdpa_f32(heads(q, sq), heads(k, sk), heads(v, sk))
        return o.transpose(0, 2, 1, 3).reshape(n * sq, c)

    y = oracle.layer_norm_f32(t, npw(b.norm1.weight), npw(b.norm1.bias))
    qkv = oracle.linear_f32(y, npw(b.to_qkv.weight))
    t = t + oracle.linear_f32(attn(qkv[:, :c], qkv[:, c:2 * c], qkv[:, 2 * c:], s, s), npw(b.to_out1.weight),
                              npw(b.to_out1.bias))
    y = oracle.layer_norm_f32(t, npw(b.norm2.weight), npw(b.norm2.bias))
    q = oracle.linear_f32(y, npw(b.to_q2.weight))
    kv = oracle.linear_f32(ctx.reshape(-1, 48), npw(b.to_kv2.weight))
    t = t + oracle.linear_f32(attn(q, kv[:, :c], kv[:, c:], s, 7), npw(b.to_out2.weight), npw(b.to_out2.bias))
    y = oracle.layer_norm_f32(t, npw(b.norm3.weight), npw(b.norm3.bias))
    hcat = oracle.linear_f32(y, npw(b.ff.proj.weight), npw(b.ff.proj.bias))
    g = hcat[:, :4 * c] * oracle.gelu_f32(hcat[:, 4 * c:])
    t = t + oracle.linear_f32(g, npw(b.ff.out.weight), npw(b.ff.out.bias))
    t = oracle.linear_f32(t, npw(st.proj_out.weight), npw(st.proj_out.bias))
    ref = t.reshape(n, 6, 6, c).transpose(0, 3, 1, 2) + x
    check(got, ref)


def test_ddim_step_matches_reference_formula():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((2, 4, 8, 8)).astype(np.float32)
    e = rng.standard_normal((2, 4, 8, 8)).astype(np.float32)
    sched = U.DDIM(steps=50)
    t = sched.timesteps[10]
    a_t, a_p = sched.alphas(t)
    got = sched.step(mt.tensor(x).cuda(), mt.tensor(e).cuda(), t).numpy()
    x0 = np.clip((x - np.sqrt(1 - a_t) * e) / np.sqrt(a_t), -1, 1)
    e2 = (x - np.sqrt(a_t) * x0) / np.sqrt(1 - a_t)
    check(got, np.sqrt(a_p) * x0 + np.sqrt(1 - a_p) * e2, 1e-5)


def test_cuda_graph_replay_matches_eager():
    from mtorch_b200.graphs import Graphed

    mt.manual_seed(0)
    net = U.UNet(chans=(64, 128), attn=(True, False), layers=1, heads=2, ctx_dim=64, device="cuda", dtype="bfloat16")
    rng = np.random.default_rng(5)
    x = mt.tensor(rng.standard_normal((2, 4, 16, 16)).astype(np.float32), dtype="bfloat16").cuda()
    ctx = mt.tensor(rng.standard_normal((2, 5, 64)).astype(np.float32), dtype="bfloat16").cuda()
    te = mt.tensor(U.timestep_embedding(np.full(2, 300.0), 64), dtype="bfloat16").cuda()
    g = Graphed(net, x, te, ctx)
    assert g.kernels_per_replay > 50
    eager = net(x, te, ctx).numpy()
    np.testing.assert_array_equal(g(x, te, ctx).numpy(), eager)
    x2 = mt.tensor(rng.standard_normal((2, 4, 16, 16)).astype(np.float32), dtype="bfloat16").cuda()
    np.testing.assert_array_equal(g(x2, te, ctx).numpy(), net(x2, te, ctx).numpy())


def test_tiny_unet_bf16_runs_and_is_batch_independent():
    mt.manual_seed(0)
    net = U.UNet(chans=(64, 128), attn=(True, False), layers=1, heads=2, ctx_dim=64, device="cuda", dtype="bfloat16")
    rng = np.random.default_rng(3)
    x = mt.tensor(rng.standard_normal((4, 4, 16, 16)).astype(np.float32), dtype="bfloat16").cuda()
    ctx = mt.tensor(rng.standard_normal((4, 5, 64)).astype(np.float32), dtype="bfloat16").cuda()
    te = mt.tensor(U.timestep_embedding(np.full(4, 500.0), 64), dtype="bfloat16").cuda()
    y = net(x, te, ctx).numpy()
    assert y.shape == (4, 4, 16, 16) and np.isfinite(y).all()
    y2 = net(x[2:], te[2:], ctx[2:]).numpy()
    np.testing.assert_array_equal(y[2:], y2)


def test_full_unet_batch8_equals_batch64_bitwise():
    """The SD-1.5 UNet (bf16) on 8 samples equals, bit for bit, the same 8 samples inside a batch
    of 64: the per-GPU work of the 8-GPU job against the 1-GPU job.  Split-K counts, GroupNorm
    chunking and attention tiling depend only on the per-image shape; column-tile widths may
    change with the row count (they do not change any element's K-reduction order)."""
    mt.manual_seed(0)
    net = U.UNet(device="cuda", dtype="bfloat16")
    mt.manual_seed(1)
    x = mt.randn(64, 4, 64, 64).to("bfloat16").cuda()
    ctx = mt.randn(64, 77, 768).to("bfloat16").cuda()
    te = mt.tensor(U.timestep_embedding(np.full(64, 741.0)), dtype="bfloat16").cuda()
    y64 = net(x, te, ctx).numpy()
    for lo in (0, 56):
        y8 = net(x[lo:lo + 8], te[lo:lo + 8], ctx[lo:lo + 8]).numpy()
        np.testing.assert_array_equal(y8, y64[lo:lo + 8])
