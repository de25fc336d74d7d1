"""Device parity: every hot-path op on cuda vs the CPU oracle (the restated reference arithmetic,
pinned to the reference in test_oracle_pins.py) on the same seeded inputs.

Tolerances: fp32 paths rtol 1e-4 (3xTF32 / fp32 SIMT), bf16 paths
rtol 2e-2 against the fp32 oracle evaluated on the same bf16-rounded inputs.  Because relative
error is meaningless for outputs that cancel to ~0, each check also allows an absolute error of
rtol * max|reference|.
"""
import os

import numpy as np
import pytest

import oracle
import mtorch_b200 as mt

pytestmark = pytest.mark.gpu

FP32_RTOL = 1e-4
BF16_RTOL = 2e-2


def check(got, ref, rtol):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=rtol * max(np.abs(ref).max(), 1e-30))


def cu(a, dtype=None):
    t = mt.tensor(np.asarray(a, np.float32))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def bf16_round(a):
    return mt.tensor(np.asarray(a, np.float32)).to("bfloat16").numpy()


def rnd(*shape, seed=0, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * scale).astype(np.float32)


# ---------------------------------------------------------------------------------------------
# elementwise / norms


def test_binary_broadcast_exact():
    a, b = rnd(2, 3, 5, 7), rnd(3, 1, 7, seed=1)
    for op, f in (("add", np.add), ("sub", np.subtract), ("mul", np.multiply), ("div", np.divide)):
        got = getattr(mt, op)(cu(a), cu(b)).numpy()
        np.testing.assert_array_equal(got, f(a, b).astype(np.float32))
    np.testing.assert_array_equal((cu(a) * 2.5).numpy(), a * np.float32(2.5))
    x = cu(a, "bfloat16")
    np.testing.assert_array_equal((x + x).numpy(), bf16_round(bf16_round(a) * 2))


def test_strided_copy_and_cast():
    a = rnd(4, 6, 8)
    t = cu(a)
    np.testing.assert_array_equal(t.permute(2, 0, 1).contiguous().numpy(), a.transpose(2, 0, 1))
    np.testing.assert_array_equal(t.to("bfloat16").float().numpy(), bf16_round(a))
    np.testing.assert_array_equal(mt.cat([t, t[:, :2]], dim=1).numpy(), np.concatenate([a, a[:, :2]], 1))
    x = cu(rnd(2, 3, 4, 5)).contiguous(memory_format=mt.channels_last)
    up = mt.nn.functional.interpolate(x, scale_factor=2).numpy()
    np.testing.assert_array_equal(up, x.numpy().repeat(2, 2).repeat(2, 3))


def test_channels_last_cat_and_upsample_bf16_exact():
    """The UNet's skip concat and nearest-2x upsample on channels-last bf16 (16-byte row path)."""
    a = cu(rnd(2, 320, 8, 8), "bfloat16").contiguous(memory_format=mt.channels_last)
    b = cu(rnd(2, 640, 8, 8, seed=1), "bfloat16").contiguous(memory_format=mt.channels_last)
    c = mt.cat([a, b], dim=1)
    assert c.is_contiguous(mt.channels_last)
    np.testing.assert_array_equal(c.numpy(), np.concatenate([a.numpy(), b.numpy()], 1))
    up = mt.nn.functional.interpolate(b, scale_factor=2)
    assert up.is_contiguous(mt.channels_last)
    np.testing.assert_array_equal(up.numpy(), b.numpy().repeat(2, 2).repeat(2, 3))


@pytest.mark.parametrize("cols", [320, 640, 1280, 200])
def test_layer_norm_bf16(cols):
    x, w, b = rnd(333, cols, seed=4, scale=3.0) + 1.0, rnd(cols, seed=5), rnd(cols, seed=6)
    ref = oracle.layer_norm_f32(bf16_round(x), bf16_round(w), bf16_round(b))
    got = mt.layer_norm(cu(x, "bfloat16"), [cols], cu(w, "bfloat16"), cu(b, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)


def test_device_uniform_matches_host_generator():
    mt.manual_seed(7)
    host = mt.rand(1001).numpy()
    mt.manual_seed(7)
    dev = mt.empty(1001, device="cuda").uniform_(0.0, 1.0).numpy()
    np.testing.assert_array_equal(dev, host)
    after_dev = mt.rand(3).numpy()
    mt.manual_seed(7)
    mt.rand(1001)
    np.testing.assert_array_equal(after_dev, mt.rand(3).numpy())


def test_activations(golden):
    x = golden["silu.x"]
    check(mt.silu(cu(x)).numpy(), golden["silu.y"], 1e-5)
    check(mt.gelu(cu(x)).numpy(), golden["gelu.y"], 1e-5)
    check(mt.gelu(cu(x), approximate="tanh").numpy(), golden["gelu_tanh.y"], 1e-5)
    xb = bf16_round(x)
    check(mt.silu(cu(x, "bfloat16")).numpy(), oracle.silu_f32(xb), BF16_RTOL)


def test_softmax_layer_norm_group_norm(golden):
    check(mt.softmax(cu(golden["softmax.x"]), -1).numpy(), golden["softmax.y"], FP32_RTOL)
    x = rnd(6, 5000, seed=3)
    check(mt.softmax(cu(x), -1).numpy(), oracle.softmax_f32(x), FP32_RTOL)
    check(mt.softmax(cu(x.T.copy()), 0).numpy(), oracle.softmax_f32(x).T, FP32_RTOL)
    check(mt.layer_norm(cu(golden["layer_norm.x"]), [32], cu(golden["layer_norm.w"]), cu(golden["layer_norm.b"]))
          .numpy(), golden["layer_norm.y"], FP32_RTOL)
    x, w, b = rnd(300, 1280, seed=4), rnd(1280, seed=5), rnd(1280, seed=6)
    check(mt.layer_norm(cu(x), [1280], cu(w), cu(b)).numpy(), oracle.layer_norm_f32(x, w, b), FP32_RTOL)
    check(mt.group_norm(cu(golden["group_norm.x"]), 4, cu(golden["group_norm.w"]), cu(golden["group_norm.b"]))
          .numpy(), golden["group_norm.y"], FP32_RTOL)


@pytest.mark.parametrize("shape,G", [((2, 320, 16, 16), 32), ((3, 64, 9, 7), 8), ((1, 960, 8, 8), 32)])
@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
def test_group_norm_silu(shape, G, layout):
    x, w, b = rnd(*shape, seed=7, scale=2.0) + 0.5, rnd(shape[1], seed=8), rnd(shape[1], seed=9)
    ref = oracle.group_norm_f32(x, G, w, b)
    xt = cu(x)
    if layout == "channels_last":
        xt = xt.contiguous(memory_format=mt.channels_last)
    got = mt.group_norm(xt, G, cu(w), cu(b))
    check(got.numpy(), ref, FP32_RTOL)
    fused = mt.nn.GroupNorm(G, shape[1]).cuda()
    fused.weight.copy_(cu(w))
    fused.bias.copy_(cu(b))
    check(fused(xt, fuse_silu=True).numpy(), oracle.silu_f32(ref), FP32_RTOL)
    xb = bf16_round(x)
    gb = mt.group_norm(cu(x, "bfloat16").contiguous(memory_format=mt.channels_last), G, cu(w), cu(b), fuse_silu=True)
    check(gb.numpy(), oracle.silu_f32(oracle.group_norm_f32(xb, G, w, b)), BF16_RTOL)


@pytest.mark.parametrize("n,c,h,w,k", [(24, 320, 64, 64, 8), (16, 320, 50, 50, 10), (40, 1280, 16, 16, 20),
                                       (12, 640, 30, 30, 10), (80, 2560, 8, 8, 37)])
def test_group_norm_single_read(n, c, h, w, k):
    """Channels-last bf16 GroupNorm of a batch whose chunks fill the GPU once (k images here) runs
    as ONE cooperative launch (chunk in shared memory, one read and one write of the activation);
    the whole batch (n images) takes the three-launch path.  The two paths agree bit for bit
    (ragged last chunks, one lane per pixel at 2560 channels), so a sample's result never depends
    on the batch, and both are within the bf16 tolerance of the oracle (reference group_norm,
    tensor.cpp:18643-18963)."""
    x = rnd(n, c, h, w, seed=n + c, scale=1.5) + 0.3
    wt, bs = rnd(c, seed=1), rnd(c, seed=2)
    xd = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    lib = mt._lib.lib()
    got = mt.group_norm(xd, 32, cu(wt), cu(bs), fuse_silu=True).numpy()
    n0 = lib.mt_cuda_launch_count()
    part = mt.group_norm(xd[n - k:], 32, cu(wt), cu(bs), fuse_silu=True)
    if os.environ.get("MT_GN_FUSED", "1") != "0":
        assert lib.mt_cuda_launch_count() - n0 == 1  # statistics, affine and apply in one kernel
    np.testing.assert_array_equal(got[n - k:], part.numpy())
    ref = oracle.silu_f32(oracle.group_norm_f32(bf16_round(x[:2]), 32, wt, bs))
    check(got[:2], ref, BF16_RTOL)
    check(part.numpy()[-2:], oracle.silu_f32(oracle.group_norm_f32(bf16_round(x[-2:]), 32, wt, bs)), BF16_RTOL)


def test_group_norm_batch_independent():
    """An image's result does not depend on batch size or position (the multi-GPU sharding
    relies on it): bitwise equal."""
    x = cu(rnd(4, 320, 16, 16, seed=10), "bfloat16").contiguous(memory_format=mt.channels_last)
    full = mt.group_norm(x, 32, fuse_silu=True).numpy()
    part = mt.group_norm(x[2:], 32, fuse_silu=True).numpy()
    np.testing.assert_array_equal(full[2:], part)


# ---------------------------------------------------------------------------------------------
# GEMM family


def test_matmul_fp32_golden(golden):
    check(mt.matmul(cu(golden["matmul.a"]), cu(golden["matmul.b"])).numpy(), golden["matmul.y"], FP32_RTOL)
    check(mt.bmm(cu(golden["bmm.a"]), cu(golden["bmm.b"])).numpy(), golden["bmm.y"], FP32_RTOL)
    check(mt.addmm(cu(golden["addmm.i"]), cu(golden["addmm.a"]), cu(golden["addmm.b"]), beta=0.5, alpha=2.0).numpy(),
          golden["addmm.y"], FP32_RTOL)
    check(mt.linear(cu(golden["linear.x"]), cu(golden["linear.w"]), cu(golden["linear.b"])).numpy(),
          golden["linear.y"], FP32_RTOL)


@pytest.mark.parametrize("M,K,N", [(256, 320, 200), (130, 1000, 520), (1, 64, 3), (515, 48, 1280)])
def test_matmul_fp32_3xtf32(M, K, N):
    a, b = rnd(M, K, seed=M), rnd(K, N, seed=N)
    check(mt.matmul(cu(a), cu(b)).numpy(), oracle.matmul_f32(a, b), FP32_RTOL)
    # transposed views go through the operand packer
    check(mt.matmul(cu(a.T.copy()).t(), cu(b.T.copy()).t()).numpy(), oracle.matmul_f32(a, b), FP32_RTOL)


def test_batched_broadcast_matmul_fp32():
    a, b = rnd(2, 3, 33, 40), rnd(3, 40, 17, seed=1)
    ref = np.stack([[oracle.matmul_f32(a[i, j], b[j]) for j in range(3)] for i in range(2)])
    check(mt.matmul(cu(a), cu(b)).numpy(), ref, FP32_RTOL)
    check(mt.matmul(cu(a), cu(b[0])).numpy(), np.stack([[oracle.matmul_f32(a[i, j], b[0]) for j in range(3)]
                                                          for i in range(2)]), FP32_RTOL)
    v = rnd(40, seed=2)
    check(mt.matmul(cu(a[0, 0]), cu(v)).numpy(), oracle.matmul_f32(a[0, 0], v[:, None])[:, 0], FP32_RTOL)


@pytest.mark.parametrize("M,K,N", [(300, 320, 320), (1000, 320, 640), (257, 640, 1280), (128, 768, 320),
                                   (64, 320, 4), (4096, 320, 2560)])
def test_linear_bf16(M, K, N):
    x, w, b = rnd(M, K, seed=1), rnd(N, K, seed=2, scale=0.05), rnd(N, seed=3)
    ref = oracle.linear_f32(bf16_round(x), bf16_round(w), bf16_round(b))
    got = mt.linear(cu(x, "bfloat16"), cu(w, "bfloat16"), cu(b, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)


def test_linear_bf16_fused_epilogues():
    from mtorch_b200 import _lib
    from mtorch_b200.ops import linear

    M, K, F = 500, 320, 1280
    x, w, b, r = rnd(M, K), rnd(2 * F, K, seed=1, scale=0.05), rnd(2 * F, seed=2), rnd(M, F, seed=3)
    xb, wb, bb, rb = map(bf16_round, (x, w, b, r))
    # GEGLU: module order is [value rows; gate rows]; the kernel wants (64 value, 64 gate) groups
    h = oracle.linear_f32(xb, wb, bb)
    val, gate = h[:, :F], h[:, F:]
    ref = val * oracle.gelu_f32(gate) + rb
    perm = np.concatenate([np.concatenate([np.arange(g, g + 64), F + np.arange(g, g + 64)]) for g in range(0, F, 64)])
    got = linear(cu(x, "bfloat16"), cu(w[perm], "bfloat16"), cu(b[perm], "bfloat16"), epilogue=_lib.EPI_GEGLU,
                 residual=cu(r, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)
    got = linear(cu(x, "bfloat16"), cu(w[:F], "bfloat16"), None, epilogue=_lib.EPI_SILU).numpy()
    check(got, oracle.silu_f32(oracle.linear_f32(xb, wb[:F])), BF16_RTOL)
    # GELU epilogue over pre-activations spread across about +-8 (the 16-bit epilogue evaluates the
    # normal CDF as a clamped polynomial; fp32 keeps the erf of the reference at 1e-4)
    ws = rnd(F, K, seed=4, scale=0.15)
    pre = oracle.linear_f32(xb, bf16_round(ws))
    assert np.abs(pre).max() > 6
    got = linear(cu(x, "bfloat16"), cu(ws, "bfloat16"), None, epilogue=_lib.EPI_GELU).numpy()
    check(got, oracle.gelu_f32(pre), BF16_RTOL)
    got32 = linear(cu(x), cu(ws), None, epilogue=_lib.EPI_GELU).numpy()
    check(got32, oracle.gelu_f32(oracle.linear_f32(x, ws)), FP32_RTOL)


def test_baddbmm_fp32_golden(golden):
    """`baddbmm` (tensor.cpp:25557-25694): beta * input (broadcast over rows) + alpha * bmm, the
    reference's own output."""
    i, a, b = (cu(golden[f"baddbmm.{n}"]) for n in "iab")
    check(mt.baddbmm(i, a, b, beta=-0.75, alpha=1.5).numpy(), golden["baddbmm.y"], FP32_RTOL)


@pytest.mark.parametrize("B,M,K,N", [(16, 256, 40, 256), (4, 77, 64, 130)])
def test_baddbmm_bf16(B, M, K, N):
    i, a, b = rnd(B, M, N, seed=3), rnd(B, M, K, seed=4), rnd(B, K, N, seed=5)
    ref = oracle.baddbmm_f32(bf16_round(i), bf16_round(a), bf16_round(b), 0.5, 0.25)
    got = mt.baddbmm(cu(i, "bfloat16"), cu(a, "bfloat16"), cu(b, "bfloat16"), beta=0.5, alpha=0.25).numpy()
    check(got, ref, BF16_RTOL)


def test_bmm_bf16_attention_shapes():
    a, b = rnd(16, 256, 40), rnd(16, 40, 256, seed=1)
    ref = np.stack([oracle.matmul_f32(bf16_round(a[i]), bf16_round(b[i])) for i in range(16)])
    check(mt.bmm(cu(a, "bfloat16"), cu(b, "bfloat16")).numpy(), ref, BF16_RTOL)


def test_small_problem_tiling_is_batch_invariant():
    """Few-tile problems use narrower column tiles; results must not change with the batch."""
    x = cu(rnd(16384, 1280), "bfloat16")
    w = cu(rnd(1280, 1280, seed=1, scale=0.03), "bfloat16")
    np.testing.assert_array_equal(mt.linear(x, w).numpy()[:256], mt.linear(x[:256], w).numpy())
    xi = cu(rnd(32, 1280, 8, 8, seed=2), "bfloat16").contiguous(memory_format=mt.channels_last)
    wc = cu(rnd(1280, 1280, 3, 3, seed=3, scale=0.01), "bfloat16")
    full = mt.conv2d(xi, wc, None, 1, 1).numpy()
    np.testing.assert_array_equal(full[:2], mt.conv2d(xi[:2], wc, None, 1, 1).numpy())


@pytest.mark.parametrize("M,K,N,dtype,act", [
    (76000, 320, 320, "bfloat16", "none"),   # B-resident tiles (per-row residual loads); last tile 96 rows
    (40000, 320, 640, "bfloat16", "gelu"),   # residual map, several tiles per CTA (prefetched a tile ahead);
                                             # last tile 64 rows: two warps' rows all past M
    (5000, 640, 200, "float16", "none"),     # N = 200: partial 32-column chunk, chunks past N
    (300, 640, 1280, "bfloat16", "silu"),    # fewer tiles than CTAs
    (2000, 1280, 1280, "bfloat16", "none"),  # long K: per-row residual loads
])
def test_linear_residual_epilogue(M, K, N, dtype, act):
    """D = act(x W^T + b) + residual with the residual read through a tensor map into the output
    staging buffers (TMA-store epilogue), against the oracle on the same 16-bit inputs."""
    from mtorch_b200 import _lib

    x, w, b, r = rnd(M, K, seed=1), rnd(N, K, seed=2, scale=K ** -0.5), rnd(N, seed=3), rnd(M, N, seed=4)
    rd = bf16_round if dtype == "bfloat16" else (lambda a: mt.tensor(a).to("float16").numpy())  # noqa: E731
    pre = oracle.linear_f32(rd(x), rd(w), rd(b))
    f = {"none": lambda a: a, "gelu": oracle.gelu_f32, "silu": oracle.silu_f32}[act]
    epi = {"none": _lib.EPI_NONE, "gelu": _lib.EPI_GELU, "silu": _lib.EPI_SILU}[act]
    got = mt.ops.linear(cu(x, dtype), cu(w, dtype), cu(b, dtype), epilogue=epi, residual=cu(r, dtype)).numpy()
    check(got, f(pre) + rd(r), BF16_RTOL)


def test_gemm_residual_batched_and_pitched():
    """Batched GEMM with a per-batch residual, and a residual that is a column slice of a wider
    matrix (row pitch > N): both through the residual tensor map."""
    a, bm = rnd(3, 700, 256, seed=5), rnd(3, 256, 384, seed=6, scale=1 / 16)
    r = rnd(3, 700, 384, seed=7)
    got = mt.ops.gemm(cu(a, "bfloat16"), cu(bm, "bfloat16"), residual=cu(r, "bfloat16")).numpy()
    ref = np.stack([oracle.matmul_f32(bf16_round(a[i]), bf16_round(bm[i])) for i in range(3)]) + bf16_round(r)
    check(got, ref, BF16_RTOL)
    wide = cu(rnd(2000, 512, seed=8), "bfloat16")
    x, w = rnd(2000, 320, seed=9), rnd(320, 320, seed=10, scale=320 ** -0.5)
    got = mt.ops.linear(cu(x, "bfloat16"), cu(w, "bfloat16"), None, residual=wide[:, 64:384]).numpy()
    ref = oracle.linear_f32(bf16_round(x), bf16_round(w)) + wide.numpy()[:, 64:384]
    check(got, ref, BF16_RTOL)


def test_linear_batch_independent():
    x = cu(rnd(3000, 320), "bfloat16")
    w = cu(rnd(640, 320, seed=1, scale=0.05), "bfloat16")
    full = mt.linear(x, w).numpy()
    np.testing.assert_array_equal(full[1500:], mt.linear(x[1500:], w).numpy())


# ---------------------------------------------------------------------------------------------
# conv2d


@pytest.mark.parametrize("name", ["conv_p1", "conv_s2", "conv_d2", "conv_1x1", "conv_g4"])
def test_conv2d_fp32_golden(golden, name):
    s, p, d, g = (int(v) for v in golden[f"{name}.params"])
    got = mt.conv2d(cu(golden[f"{name}.x"]), cu(golden[f"{name}.w"]), cu(golden[f"{name}.b"]), s, p, d, g).numpy()
    check(got, golden[f"{name}.y"], FP32_RTOL)


@pytest.mark.parametrize("shape,K,k,pad,stride", [((2, 64, 16, 16), 64, 3, 1, 1), ((1, 96, 9, 11), 40, 3, 1, 1),
                                                  ((2, 32, 8, 8), 48, 1, 0, 1), ((2, 64, 16, 16), 64, 3, 1, 2),
                                                  ((1, 96, 9, 11), 40, 3, 1, 2)])
def test_conv2d_fp32_implicit(shape, K, k, pad, stride):
    x, w, b = rnd(*shape), rnd(K, shape[1], k, k, seed=1, scale=0.1), rnd(K, seed=2)
    ref = oracle.conv2d_f32(x, w, b, stride, pad)
    check(mt.conv2d(cu(x), cu(w), cu(b), stride, pad).numpy(), ref, FP32_RTOL)
    xl = cu(x).contiguous(memory_format=mt.channels_last)
    y = mt.conv2d(xl, cu(w), cu(b), stride, pad)
    assert y.is_contiguous(mt.channels_last)
    check(y.numpy(), ref, FP32_RTOL)


@pytest.mark.parametrize("shape,K,k,stride,pad", [((2, 320, 32, 32), 320, 3, 1, 1), ((2, 128, 8, 8), 256, 3, 1, 1),
                                                  ((1, 640, 16, 16), 1280, 1, 1, 0), ((2, 4, 32, 32), 320, 3, 1, 1),
                                                  ((2, 320, 16, 16), 320, 3, 2, 1), ((1, 320, 64, 64), 4, 3, 1, 1),
                                                  ((2, 320, 64, 64), 320, 3, 2, 1), ((1, 128, 15, 17), 64, 3, 2, 1),
                                                  ((2, 1280, 16, 16), 1280, 3, 2, 1), ((1, 64, 9, 9), 64, 1, 2, 0)])
def test_conv2d_bf16(shape, K, k, stride, pad):
    """Includes stride-2 implicit convolutions (the UNet's downsamplers, a ragged odd-sized input and a
    strided 1x1): the tensor map walks the input every other pixel."""
    x, w, b = rnd(*shape), rnd(K, shape[1], k, k, seed=1, scale=0.05), rnd(K, seed=2)
    ref = oracle.conv2d_f32(bf16_round(x), bf16_round(w), bf16_round(b), stride, pad)
    conv = mt.nn.Conv2d(shape[1], K, k, stride=stride, padding=pad).cuda().to("bfloat16")
    conv.weight.copy_(cu(w, "bfloat16"))
    conv.bias.copy_(cu(b, "bfloat16"))
    xl = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    check(conv(xl).numpy(), ref, BF16_RTOL)


def _up2(a):
    return a.repeat(2, 2).repeat(2, 3)


@pytest.mark.parametrize("shape,K", [((2, 320, 8, 8), 320), ((1, 640, 5, 7), 64), ((2, 1280, 4, 4), 1280),
                                     ((1, 64, 3, 9), 128)])
def test_conv2d_up2x_bf16(shape, K):
    """Fused nearest-2x upsample + 3x3 conv (four 2x2 parity convolutions of the source) against
    the oracle's conv of the explicitly upsampled input, and against the device's explicit pair."""
    from mtorch_b200 import ops
    x, w, b = rnd(*shape), rnd(K, shape[1], 3, 3, seed=1, scale=0.05), rnd(K, seed=2)
    ref = oracle.conv2d_f32(_up2(bf16_round(x)), bf16_round(w), bf16_round(b), 1, 1)
    xd = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    wd, bd = cu(w, "bfloat16"), cu(b, "bfloat16")
    got = ops.conv2d_up2x(xd, wd, bd)
    assert got.shape == (shape[0], K, 2 * shape[2], 2 * shape[3]) and got.is_contiguous(mt.channels_last)
    check(got.numpy(), ref, BF16_RTOL)
    check(ops.conv2d_up2x(xd, wd, bd, packed=ops.pack_conv_up2x_weight(wd)).numpy(), ref, BF16_RTOL)
    explicit = mt.conv2d(ops.interpolate_nearest2x(xd), wd, bd, 1, 1).numpy()
    check(got.numpy(), explicit, BF16_RTOL)


def test_conv2d_up2x_fp32_and_module():
    """fp32 (3xTF32) at the fp32 tolerance, NCHW input, and the UNet's Upsample module using it."""
    from mtorch_b200 import ops
    from mtorch_b200 import unet as U
    x, w, b = rnd(2, 64, 6, 5), rnd(32, 64, 3, 3, seed=1, scale=0.1), rnd(32, seed=2)
    ref = oracle.conv2d_f32(_up2(x), w, b, 1, 1)
    check(ops.conv2d_up2x(cu(x), cu(w), cu(b)).numpy(), ref, FP32_RTOL)
    up = U.Upsample(64, device="cuda")
    up.conv.weight.copy_(cu(rnd(64, 64, 3, 3, seed=3, scale=0.05), "float32"))
    up.conv.bias.copy_(cu(rnd(64, seed=4)))
    xm = cu(x).contiguous(memory_format=mt.channels_last)
    ref_m = oracle.conv2d_f32(_up2(x), up.conv.weight.numpy(), up.conv.bias.numpy(), 1, 1)
    check(up(xm).numpy(), ref_m, FP32_RTOL)
    check(up(xm).numpy(), ref_m, FP32_RTOL)  # second call: cached packed weights


def test_conv2d_bf16_resnet_epilogue():
    """Per-image bias (conv bias + time embedding) and the residual add fused in the epilogue."""
    N, C, H = 2, 320, 16
    x, w, r = rnd(N, C, H, H), rnd(C, C, 3, 3, seed=1, scale=0.05), rnd(N, C, H, H, seed=2)
    pb = rnd(N, C, seed=3)
    ref = oracle.conv2d_f32(bf16_round(x), bf16_round(w), None, 1, 1) + pb[:, :, None, None] + bf16_round(r)
    xl = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    rl = cu(r, "bfloat16").contiguous(memory_format=mt.channels_last)
    got = mt.conv2d(xl, cu(w, "bfloat16"), cu(pb), 1, 1, residual=rl, bias_batch_stride=C)
    check(got.numpy(), ref, BF16_RTOL)


# ---------------------------------------------------------------------------------------------
# attention


def test_sdpa_fp32_golden(golden):
    F = mt.nn.functional
    q, k, v = (cu(golden[f"sdpa_self.{n}"]) for n in "qkv")
    check(F.scaled_dot_product_attention(q, k, v).numpy(), golden["sdpa_self.y"], FP32_RTOL)
    check(F.scaled_dot_product_attention(q, k, v, is_causal=True).numpy(), golden["sdpa_causal.y"], FP32_RTOL)
    q, k, v = (cu(golden[f"sdpa_cross.{n}"]) for n in "qkv")
    check(F.scaled_dot_product_attention(q, k, v, scale=0.3).numpy(), golden["sdpa_cross.y"], FP32_RTOL)
    check(F.scaled_dot_product_attention(q, k, v, attn_mask=cu(golden["sdpa_fmask.m"])).numpy(),
          golden["sdpa_fmask.y"], FP32_RTOL)
    bm = mt.tensor(golden["sdpa_bmask.m"].astype(bool)).cuda()
    check(F.scaled_dot_product_attention(q, k, v, attn_mask=bm).numpy(), golden["sdpa_bmask.y"], FP32_RTOL)


@pytest.mark.parametrize("B,H,Sq,Sk,D", [(2, 8, 300, 300, 40), (2, 8, 256, 77, 40), (1, 8, 200, 200, 80),
                                         (1, 8, 64, 77, 160), (2, 8, 1024, 1024, 40), (2, 8, 100, 100, 40),
                                         (1, 4, 129, 130, 64), (1, 2, 256, 200, 128), (1, 2, 300, 257, 160)])
def test_sdpa_bf16(B, H, Sq, Sk, D):
    q, k, v = rnd(B, H, Sq, D), rnd(B, H, Sk, D, seed=1), rnd(B, H, Sk, D, seed=2)
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v))
    got = mt.scaled_dot_product_attention(cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)


@pytest.mark.parametrize("B,H,Sq,Sk,D", [(2, 12, 77, 77, 64), (1, 4, 300, 300, 64), (1, 4, 200, 330, 40),
                                         (1, 4, 330, 200, 80), (2, 2, 129, 129, 64)])
def test_sdpa_bf16_causal(B, H, Sq, Sk, D):
    """Causal attention on the tensor-core kernel (key j of query i hidden when j > i, the top-left
    alignment of the reference), with ragged query and key tiles and Sq != Sk both ways."""
    q, k, v = rnd(B, H, Sq, D), rnd(B, H, Sk, D, seed=1), rnd(B, H, Sk, D, seed=2)
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v), causal=True)
    got = mt.scaled_dot_product_attention(cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16"),
                                          is_causal=True).numpy()
    check(got, ref, BF16_RTOL)


@pytest.mark.parametrize("D,dtype", [(40, "bfloat16"), (64, "bfloat16"), (80, "bfloat16"), (80, "float16"),
                                     (72, "bfloat16"), (32, "bfloat16")])
def test_sdpa_bf16_growing_scores_rescale(D, dtype):
    """Later key tiles score much higher than earlier ones, so the running maximum grows by far more
    than the lazy-rescale threshold several times within a row.  Head dims 64 / 72 / 80 run the
    lazy kernel with one P buffer per query tile (72: row sum from a ones column of V's padding)."""
    B, H, S = 2, 4, 640
    q = rnd(B, H, S, D, scale=2.0)
    k = rnd(B, H, S, D, seed=1)
    k *= (1.0 + np.repeat(np.arange(S // 128), 128) * 1.5)[None, None, :, None].astype(np.float32)
    v = rnd(B, H, S, D, seed=2)
    rd = bf16_round if dtype == "bfloat16" else (lambda a: mt.tensor(a).to("float16").numpy())  # noqa: E731
    ref = oracle.sdpa_f32(rd(q), rd(k), rd(v))
    qd, kd, vd = cu(q, dtype), cu(k, dtype), cu(v, dtype)
    assert mt.ops.sdpa_path(qd, kd, vd) == "tc_lazy"
    check(mt.scaled_dot_product_attention(qd, kd, vd).numpy(), ref, BF16_RTOL)


@pytest.mark.parametrize("D", [40, 48, 80])
def test_sdpa_bf16_max_jumps_inside_key_tiles(D):
    """The score maximum jumps in the second half of key tiles (the P columns already written for
    the tile are rescaled) and the last key tile is ragged.  D 40 takes the row sum from the
    tensor core (a ones column in the padding of V); D 48 has no padding and sums on the SIMT side."""
    B, H, S = 2, 4, 600
    q = rnd(B, H, S, D, scale=2.0)
    k = rnd(B, H, S, D, seed=1)
    pos = np.arange(S)
    k *= (1.0 + (pos % 128 >= 64) * (pos // 128 + 1) * 1.2)[None, None, :, None].astype(np.float32)
    v = rnd(B, H, S, D, seed=2)
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v))
    got = mt.scaled_dot_product_attention(cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)


@pytest.mark.parametrize("Sq,Sk,D", [(1100, 300, 40), (1024, 77, 40), (1536, 1000, 48)])
def test_sdpa_bf16_ragged_long_queries(Sq, Sk, D):
    """Long query sequences with ragged query counts (a CTA's second query tile partly or wholly
    past the end), ragged and short key counts (cross-attention to 77 tokens) and head dim 48
    (row sum on the SIMT side)."""
    B, H = 2, 3
    q = rnd(B, H, Sq, D, scale=1.5)
    k = rnd(B, H, Sk, D, seed=1)
    v = rnd(B, H, Sk, D, seed=2)
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v))
    got = mt.scaled_dot_product_attention(cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16")).numpy()
    check(got, ref, BF16_RTOL)


def test_sdpa_fp32_strided_heads():
    """Q/K/V as head-split views of [B, S, H*D] projections (no copies)."""
    B, S, H, D = 2, 100, 8, 40
    x = rnd(B, S, 3 * H * D)
    t = cu(x)
    q, k, v = (t[..., i * H * D:(i + 1) * H * D].reshape(B, S, H, D).transpose(1, 2) for i in range(3))
    xs = x.reshape(B, S, 3, H, D).transpose(2, 0, 3, 1, 4)
    ref = oracle.sdpa_f32(xs[0], xs[1], xs[2])
    check(mt.scaled_dot_product_attention(q, k, v).numpy(), ref, FP32_RTOL)


@pytest.mark.parametrize("B,H,Sq,Sk,D", [(2, 2, 256, 256, 32), (2, 4, 100, 77, 32), (1, 2, 300, 129, 16),
                                         (1, 2, 200, 200, 96), (1, 2, 130, 300, 144), (1, 3, 260, 100, 24)])
def test_sdpa_bf16_padded_head_dims(B, H, Sq, Sk, D):
    """Head dims without their own kernel run on the next wider tcgen05 kernel (32, 128, 160), the
    extra columns zero-filled by TMA."""
    q, k, v = rnd(B, H, Sq, D), rnd(B, H, Sk, D, seed=1), rnd(B, H, Sk, D, seed=2)
    qd, kd, vd = cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16")
    lazy = Sq > 128 and D <= 80  # padded to 32 / 48 / 64 / 80
    assert mt.ops.sdpa_path(qd, kd, vd) == ("tc_short" if Sk <= 128 and D <= 128 else "tc_lazy" if lazy else "tc")
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v))
    check(mt.scaled_dot_product_attention(qd, kd, vd).numpy(), ref, BF16_RTOL)


def test_sdpa_path_of_unet_shapes():
    """The attention shapes of the SD-1.5 UNet (strided head views of the fused projections) run on
    the tensor-core kernels; fp32 calls and non-positive scales report the SIMT kernel."""
    def heads(t, n, s, h, d):
        p = t.stride(0)
        return t._view((n, h, s, d), (s * p, d, p, 1))

    n = 2
    for c, s in ((320, 4096), (640, 1024), (1280, 256), (1280, 64)):
        d = c // 8
        qkv = mt.empty(n * s, 3 * c, dtype="bfloat16", device="cuda")
        q, k, v = (heads(qkv[:, i * c:(i + 1) * c], n, s, 8, d) for i in range(3))
        want = "tc_lazy" if d <= 80 and s > 128 else "tc"
        assert mt.ops.sdpa_path(q, k, v) == want, (c, s)
        kv = mt.empty(n * 77, 2 * c, dtype="bfloat16", device="cuda")
        kc, vc = heads(kv[:, 0:c], n, 77, 8, d), heads(kv[:, c:2 * c], n, 77, 8, d)
        assert mt.ops.sdpa_path(q, kc, vc) == ("tc_short" if d <= 128 else "tc"), (c, s, "cross")
    q = mt.empty(1, 2, 64, 40, device="cuda")
    assert mt.ops.sdpa_path(q, q, q) == "simt"
    qb = q.to("bfloat16")
    mask = mt.zeros(64, 64, device="cuda")
    assert mt.ops.sdpa_path(qb, qb, qb, attn_mask=mask) == "tc"  # masks run on the general kernel
    assert mt.ops.sdpa_path(qb, qb, qb, scale=-1.0) == "simt"


@pytest.mark.parametrize("n,c1,c2,hw,silu", [(2, 1280, 1280, 8, True), (3, 640, 320, 16, True), (2, 320, 640, 32, False),
                                            (1, 64, 128, 12, True)])
def test_skip_concat_fused_consumers_bitwise(n, c1, c2, hw, silu):
    """The up-block skip connection: GroupNorm and the 1x1 shortcut conv read cat([a, b], dim=1)
    in place; both are bit-identical to the same kernels on the materialised concatenation, and
    within the bf16 tolerance of the oracle."""
    rng = np.random.default_rng(c1 + c2 + hw)
    a = cu(rng.standard_normal((n, c1, hw, hw)).astype(np.float32), "bfloat16").contiguous(memory_format=mt.channels_last)
    b = cu(rng.standard_normal((n, c2, hw, hw)).astype(np.float32) * 2, "bfloat16").contiguous(
        memory_format=mt.channels_last)
    C = c1 + c2
    w = cu(rng.standard_normal(C).astype(np.float32), "bfloat16")
    bias = cu(rng.standard_normal(C).astype(np.float32), "bfloat16")
    cat = mt.cat([a, b], dim=1)
    assert mt.ops.cat_fusable(a, b)
    got = mt.ops.group_norm_cat(a, b, 32, w, bias, 1e-5, fuse_silu=silu).numpy()
    np.testing.assert_array_equal(got, mt.group_norm(cat, 32, w, bias, 1e-5, fuse_silu=silu).numpy())
    ref = oracle.group_norm_f32(cat.numpy(), 32, w.numpy(), bias.numpy())
    check(got, oracle.silu_f32(ref) if silu else ref, BF16_RTOL)
    K = 320
    wc = cu(rng.standard_normal((K, C, 1, 1)).astype(np.float32) * C ** -0.5, "bfloat16")
    bc = cu(rng.standard_normal(K).astype(np.float32), "bfloat16")
    got = mt.ops.conv2d_cat(a, b, wc, bc).numpy()
    np.testing.assert_array_equal(got, mt.conv2d(cat, wc, bc).numpy())
    check(got, oracle.conv2d_f32(cat.numpy(), wc.numpy(), bc.numpy()), BF16_RTOL)
    w3 = cu(rng.standard_normal((K, C, 3, 3)).astype(np.float32) * (9 * C) ** -0.5, "bfloat16")
    np.testing.assert_array_equal(mt.ops.conv2d_cat(a, b, w3, None, 1, 1).numpy(), mt.conv2d(cat, w3, None, 1, 1).numpy())


@pytest.mark.parametrize("c,k,hw,stride", [(1280, 1280, 8, 1), (2560, 1280, 8, 1), (1280, 1280, 16, 1), (640, 640, 16, 1),
                                           (1280, 1280, 16, 2)])
def test_conv_split_k_deep_levels(c, k, hw, stride):
    """The 16x16 and 8x8 convolutions split their reduction (2 or 4 ways, chosen from the per-image
    shape only) and add the fp32 partial sums in a fixed order: within the bf16 tolerance of the
    oracle, with the per-image bias and residual epilogue, and bitwise independent of the batch."""
    rng = np.random.default_rng(c + hw)
    n = 3
    x = rng.standard_normal((n, c, hw, hw)).astype(np.float32)
    w = (rng.standard_normal((k, c, 3, 3)) * (9 * c) ** -0.5).astype(np.float32)
    bias = rng.standard_normal((n, k)).astype(np.float32)
    p = hw // stride
    res = rng.standard_normal((n, k, p, p)).astype(np.float32)
    xd = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    rd = cu(res, "bfloat16").contiguous(memory_format=mt.channels_last)
    wd = cu(w, "bfloat16")
    got = mt.ops.conv2d(xd, wd, cu(bias), stride, 1, bias_batch_stride=k, residual=rd).numpy()
    ref = np.stack([oracle.conv2d_f32(bf16_round(x)[i:i + 1], bf16_round(w), bias[i], stride, 1)[0] for i in range(n)])
    check(got, ref + bf16_round(res), BF16_RTOL)
    one = mt.ops.conv2d(xd[1:2], wd, cu(bias[1:2]), stride, 1, bias_batch_stride=k, residual=rd[1:2]).numpy()
    np.testing.assert_array_equal(one[0], got[1])


@pytest.mark.parametrize("dtype,groups", [("float32", 2), ("bfloat16", 4), ("bfloat16", 64)])
def test_conv2d_grouped(dtype, groups):
    """groups > 1 (tensor.cpp:26498-26543): one convolution per group, against the oracle's grouped
    loop; groups == channels is the depthwise case."""
    rng = np.random.default_rng(groups)
    x = rng.standard_normal((2, 64, 12, 12)).astype(np.float32)
    w = (rng.standard_normal((128, 64 // groups, 3, 3)) * 0.2).astype(np.float32)
    b = rng.standard_normal(128).astype(np.float32)
    rd = (lambda a: a) if dtype == "float32" else bf16_round  # noqa: E731
    ref = oracle.conv2d_f32(rd(x), rd(w), rd(b), 1, 1, 1, groups)
    got = mt.conv2d(cu(x, dtype), cu(w, dtype), cu(b, dtype), 1, 1, 1, groups)
    check(got.float().numpy(), ref, FP32_RTOL if dtype == "float32" else BF16_RTOL)
    m = mt.nn.Conv2d(64, 128, 3, padding=1, groups=groups, device="cuda", dtype=dtype)
    y = m(cu(x, dtype).contiguous(memory_format=mt.channels_last))
    assert tuple(y.shape) == (2, 128, 12, 12)


@pytest.mark.parametrize("kind,D,causal,bcast", [("bool", 40, False, False), ("float", 64, False, True),
                                                 ("float", 80, True, False), ("bool", 128, False, True),
                                                 ("bf16", 40, False, True)])
def test_sdpa_bf16_masked_tensor_core(kind, D, causal, bcast):
    """Boolean and additive masks (fp32 or bf16, full [B, H, Sq, Sk] or broadcast [Sq, Sk]) on the
    tcgen05 kernel, with ragged tiles, causal on top, and rows whose keys are all masked (NaN,
    as the reference's softmax over an empty set)."""
    B, H, Sq, Sk = 2, 3, 200, 150
    rng = np.random.default_rng(D)
    q, k, v = rnd(B, H, Sq, D), rnd(B, H, Sk, D, seed=1), rnd(B, H, Sk, D, seed=2)
    mshape = (Sq, Sk) if bcast else (B, H, Sq, Sk)
    if kind == "bool":
        m = rng.random(mshape) > 0.3
        m[..., 5, :] = False  # a fully masked query row
        md = mt.tensor(m).cuda()
    else:
        m = (rng.standard_normal(mshape) * 2).astype(np.float32)
        m[..., 7, 100:] = -np.inf
        md = cu(m, "bfloat16" if kind == "bf16" else None)
        m = md.float().numpy()
    qd, kd, vd = cu(q, "bfloat16"), cu(k, "bfloat16"), cu(v, "bfloat16")
    assert mt.ops.sdpa_path(qd, kd, vd, attn_mask=md, is_causal=causal) == "tc"
    ref = oracle.sdpa_f32(bf16_round(q), bf16_round(k), bf16_round(v), mask=m, causal=causal)
    got = mt.scaled_dot_product_attention(qd, kd, vd, attn_mask=md, is_causal=causal).numpy()
    nan = np.isnan(ref)
    assert (np.isnan(got) == nan).all()
    check(np.where(nan, 0, got), np.where(nan, 0, ref), BF16_RTOL)


@pytest.mark.parametrize("B,H,Sq,Sk,D,dtype", [(2, 8, 4096, 77, 40, "bfloat16"), (2, 8, 1024, 77, 80, "bfloat16"),
                                               (1, 3, 300, 128, 64, "bfloat16"), (3, 2, 100, 1, 40, "bfloat16"),
                                               (1, 4, 1000, 50, 128, "float16"), (2, 2, 700, 77, 16, "bfloat16"),
                                               (1, 2, 257, 120, 48, "float16"), (1, 2, 513, 80, 48, "float16"),
                                               (2, 3, 300, 64, 24, "bfloat16")])
def test_sdpa_short_keys(B, H, Sq, Sk, D, dtype):
    """At most 128 keys (cross-attention to the 77-token context): the persistent short-key
    kernel, K and V loaded once per CTA for several query-tile pairs; ragged query counts, one key,
    the ones-column row sum (head dim <= padded - 8) and the softmax-side row sum.  Up to 80 keys
    at padded head dims <= 48 use 80-column score tiles (two CTAs per SM)."""
    q, k, v = rnd(B, H, Sq, D, scale=1.5), rnd(B, H, Sk, D, seed=1), rnd(B, H, Sk, D, seed=2)
    qd, kd, vd = cu(q, dtype), cu(k, dtype), cu(v, dtype)
    assert mt.ops.sdpa_path(qd, kd, vd) == "tc_short"
    r = bf16_round if dtype == "bfloat16" else (lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32))
    ref = oracle.sdpa_f32(r(q), r(k), r(v))
    check(mt.scaled_dot_product_attention(qd, kd, vd).float().numpy(), ref, BF16_RTOL)
