"""BASELINE configurations at full size, against the oracle.

C1  fp32 matmul 2048 x 2048 @ 2048 x 2048, inputs from mtorch.manual_seed(0) / randn (the
    reference's own generator), checked element-wise against the double-accumulating oracle.
C2  SD ResNet block fp32 at [2, 320, 64, 64] (GroupNorm 32 -> SiLU -> conv3x3 -> GroupNorm ->
    SiLU -> conv3x3 + residual, Kaiming-uniform weights, seed 0); the oracle composition runs
    for a subset of 16 output channels of the final conv (the whole chain up to that conv is
    checked in full) so the CPU side stays within seconds.
C3  SD attention block bf16 (B 2, 8 heads, head dim 40, 4096 queries; self-attention and
    cross-attention to a 77-token context, projections, GEGLU FFN) against the fp32 oracle on
    the same bf16-rounded inputs, for a subset of 256 query rows.
fp16 device path: GEMM, conv and attention with fp16 operands (kind::f16 with F16 inputs).
"""
import numpy as np
import pytest

import oracle
import mtorch_b200 as mt
from mtorch_b200 import unet as U

pytestmark = pytest.mark.gpu
FP32_RTOL = 1e-4
BF16_RTOL = 2e-2


def check(got, ref, rtol):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=rtol * np.abs(ref).max())


def test_c1_matmul_2048_fp32_seeded():
    mt.manual_seed(0)
    a, b = mt.randn(2048, 2048), mt.randn(2048, 2048)
    got = mt.matmul(a.cuda(), b.cuda()).numpy()
    check(got, oracle.matmul_f32(a.numpy(), b.numpy()), FP32_RTOL)


def test_c2_resnet_block_fp32():
    mt.manual_seed(0)
    x = mt.randn(2, 320, 64, 64)
    blk_gn1 = mt.nn.GroupNorm(32, 320)
    conv1 = mt.nn.Conv2d(320, 320, 3, padding=1)
    blk_gn2 = mt.nn.GroupNorm(32, 320)
    conv2 = mt.nn.Conv2d(320, 320, 3, padding=1)
    xd = x.cuda()
    h = mt.nn.functional.silu(mt.group_norm(xd, 32, blk_gn1.weight.cuda(), blk_gn1.bias.cuda()))
    h1 = mt.conv2d(h, conv1.weight.cuda(), conv1.bias.cuda(), 1, 1)
    h2 = mt.nn.functional.silu(mt.group_norm(h1, 32, blk_gn2.weight.cuda(), blk_gn2.bias.cuda()))
    out = mt.conv2d(h2, conv2.weight.cuda(), conv2.bias.cuda(), 1, 1, residual=xd)
    xn = x.numpy()
    r_h = oracle.silu_f32(oracle.group_norm_f32(xn, 32, blk_gn1.weight.numpy(), blk_gn1.bias.numpy()))
    check(h.numpy(), r_h, FP32_RTOL)
    # conv1 is checked on 16 output channels from the device-computed input (isolates the conv)
    sel = np.arange(0, 320, 20)
    w1 = conv1.weight.numpy()[sel]
    check(h1.numpy()[:, sel], oracle.conv2d_f32(h.numpy(), w1, conv1.bias.numpy()[sel], 1, 1), FP32_RTOL)
    w2 = conv2.weight.numpy()[sel]
    ref = oracle.conv2d_f32(h2.numpy(), w2, conv2.bias.numpy()[sel], 1, 1) + xn[:, sel]
    check(out.numpy()[:, sel], ref, FP32_RTOL)


def test_c3_attention_block_bf16_subset():
    mt.manual_seed(0)
    st = U.SpatialTransformer(320, heads=8, ctx_dim=768, device="cuda")
    for p in st.parameters():
        p.normal_(0.0, 0.02)
    st = st.to("bfloat16")
    mt.manual_seed(1)
    x = mt.randn(2, 320, 64, 64).to("bfloat16")
    ctx = mt.randn(2, 77, 768).to("bfloat16")
    got = st(x.cuda().contiguous(memory_format=mt.channels_last), ctx.cuda()).numpy()
    f = lambda t: t.float().numpy()  # noqa: E731
    b = st.block
    n, c, s, H = 2, 320, 4096, 8
    xn, cn = x.numpy(), ctx.numpy()
    t = oracle.group_norm_f32(xn, 32, f(st.norm.weight), f(st.norm.bias), eps=1e-6).transpose(0, 2, 3, 1).reshape(-1, c)
    t = oracle.linear_f32(t, f(st.proj_in.weight), f(st.proj_in.bias))
    rows = np.arange(0, s, 16)  # 256 query rows per sample
    y = oracle.layer_norm_f32(t, f(b.norm1.weight), f(b.norm1.bias))
    qkv = oracle.linear_f32(y, f(b.to_qkv.weight)).reshape(n, s, 3, H, 40)
    q = qkv[:, rows, 0].transpose(0, 2, 1, 3)
    k, v = qkv[:, :, 1].transpose(0, 2, 1, 3), qkv[:, :, 2].transpose(0, 2, 1, 3)
    a = oracle.sdpa_f32(q, k, v).transpose(0, 2, 1, 3).reshape(-1, c)
    tr = t.reshape(n, s, c)[:, rows].reshape(-1, c)
    tr = tr + oracle.linear_f32(a, f(b.to_out1.weight), f(b.to_out1.bias))
    y = oracle.layer_norm_f32(tr, f(b.norm2.weight), f(b.norm2.bias))
    q2 = oracle.linear_f32(y, f(b.to_q2.weight)).reshape(n, len(rows), H, 40).transpose(0, 2, 1, 3)
    kv = oracle.linear_f32(cn.reshape(-1, 768), f(b.to_kv2.weight)).reshape(n, 77, 2, H, 40)
    a2 = oracle.sdpa_f32(q2, kv[:, :, 0].transpose(0, 2, 1, 3), kv[:, :, 1].transpose(0, 2, 1, 3))
    tr = tr + oracle.linear_f32(a2.transpose(0, 2, 1, 3).reshape(-1, c), f(b.to_out2.weight), f(b.to_out2.bias))
    y = oracle.layer_norm_f32(tr, f(b.norm3.weight), f(b.norm3.bias))
    hc = oracle.linear_f32(y, f(b.ff.proj.weight), f(b.ff.proj.bias))
    tr = tr + oracle.linear_f32(hc[:, :1280] * oracle.gelu_f32(hc[:, 1280:]), f(b.ff.out.weight), f(b.ff.out.bias))
    tr = oracle.linear_f32(tr, f(st.proj_out.weight), f(st.proj_out.bias))
    ref = tr.reshape(n, len(rows), c) + xn.transpose(0, 2, 3, 1).reshape(n, s, c)[:, rows]
    got_rows = got.transpose(0, 2, 3, 1).reshape(n, s, c)[:, rows]
    check(got_rows, ref, BF16_RTOL)


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def test_fp16_device_path():
    rng = np.random.default_rng(7)
    x, w = rng.standard_normal((300, 320)).astype(np.float32), (rng.standard_normal((640, 320)) * 0.05).astype(np.float32)
    got = mt.linear(mt.tensor(x, dtype="float16").cuda(), mt.tensor(w, dtype="float16").cuda()).float().numpy()
    check(got, oracle.linear_f32(_f16(x), _f16(w)), BF16_RTOL)
    xi = rng.standard_normal((2, 64, 16, 16)).astype(np.float32)
    wc = (rng.standard_normal((64, 64, 3, 3)) * 0.05).astype(np.float32)
    xl = mt.tensor(xi, dtype="float16").cuda().contiguous(memory_format=mt.channels_last)
    got = mt.conv2d(xl, mt.tensor(wc, dtype="float16").cuda(), None, 1, 1).float().numpy()
    check(got, oracle.conv2d_f32(_f16(xi), _f16(wc), None, 1, 1), BF16_RTOL)
    q, k, v = (rng.standard_normal((2, 4, 200, 40)).astype(np.float32) for _ in range(3))
    got = mt.scaled_dot_product_attention(*(mt.tensor(t, dtype="float16").cuda() for t in (q, k, v))).float().numpy()
    check(got, oracle.sdpa_f32(_f16(q), _f16(k), _f16(v)), BF16_RTOL)


F16_RTOL = 5e-3  # fp16 keeps 11 significant bits: one output rounding is 2^-11 relative


@pytest.mark.parametrize("cl", [False, True])
def test_fp16_group_norm_silu(cl):
    """GroupNorm (+ fused SiLU) in fp16, NCHW and channels-last: the reference's own SD dtype
    (its channels-last fp16 fast path is tensor.cpp:18683-18791)."""
    rng = np.random.default_rng(8)
    x = (rng.standard_normal((2, 320, 16, 16)) * 2 + 0.5).astype(np.float32)
    w, b = rng.standard_normal(320).astype(np.float32), rng.standard_normal(320).astype(np.float32)
    xd = mt.tensor(x, dtype="float16").cuda()
    if cl:
        xd = xd.contiguous(memory_format=mt.channels_last)
    wd, bd = mt.tensor(w, dtype="float16").cuda(), mt.tensor(b, dtype="float16").cuda()
    ref = oracle.group_norm_f32(_f16(x), 32, _f16(w), _f16(b))
    check(mt.group_norm(xd, 32, wd, bd).float().numpy(), ref, F16_RTOL)
    check(mt.group_norm(xd, 32, wd, bd, fuse_silu=True).float().numpy(), oracle.silu_f32(ref), F16_RTOL)


@pytest.mark.parametrize("cols", [320, 640, 1280, 77])
def test_fp16_layer_norm_softmax(cols):
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((300, cols)) * 3).astype(np.float32)
    w, b = rng.standard_normal(cols).astype(np.float32), rng.standard_normal(cols).astype(np.float32)
    xd = mt.tensor(x, dtype="float16").cuda()
    got = mt.layer_norm(xd, (cols,), mt.tensor(w, dtype="float16").cuda(), mt.tensor(b, dtype="float16").cuda())
    check(got.float().numpy(), oracle.layer_norm_f32(_f16(x), _f16(w), _f16(b)), F16_RTOL)
    check(mt.softmax(xd, -1).float().numpy(), oracle.softmax_f32(_f16(x)), F16_RTOL)


def test_fp16_pointwise():
    rng = np.random.default_rng(10)
    x = (rng.standard_normal((4, 320, 8, 8)) * 3).astype(np.float32)
    y = rng.standard_normal((1, 320, 1, 1)).astype(np.float32)
    xd, yd = mt.tensor(x, dtype="float16").cuda(), mt.tensor(y, dtype="float16").cuda()
    check(mt.silu(xd).float().numpy(), oracle.silu_f32(_f16(x)), F16_RTOL)
    check(mt.gelu(xd).float().numpy(), oracle.gelu_f32(_f16(x)), F16_RTOL)
    check(mt.gelu(xd, approximate="tanh").float().numpy(), oracle.gelu_f32(_f16(x), "tanh"), F16_RTOL)
    check((xd + yd).float().numpy(), _f16(x) + _f16(y), F16_RTOL)
    check((xd * yd).float().numpy(), _f16(x) * _f16(y), F16_RTOL)
