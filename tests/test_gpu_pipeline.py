"""The ops around the UNet on the device, each against the oracle on the same inputs: the
sinusoidal timestep embedding, guidance + DDIM update with a device-resident timestep, the
embedding gather, quick GELU (unary and GEMM epilogue); the sampler (eager vs one CUDA graph per
step); and the CLIP text encoder and VAE decoder compositions at small widths.

Tolerances (north star): fp32 rtol 1e-4, bf16 rtol 2e-2 against the fp32 oracle, integer / index
work bit-exact.  The timestep embedding's cos / sin of arguments up to 999 rad amplify a one-ulp
difference in a frequency (device expf vs the host libm) by the argument, so its absolute tolerance
is 4 ulp of the argument: 4 * 2^-23 * |t * freq|."""
import numpy as np
import pytest

import oracle
import mtorch_b200 as mt
from mtorch_b200 import _lib as L
from mtorch_b200 import ops
from mtorch_b200 import unet as U

pytestmark = pytest.mark.gpu
RTOL = 1e-4


def check(got, ref, rtol=RTOL):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(ref, np.float64), rtol=rtol,
                               atol=rtol * np.abs(ref).max())


def npw(t):
    return t.numpy().astype(np.float32)


def cuda(a, dtype=None):
    return mt.tensor(a, dtype=dtype).cuda()


# ---- timestep embedding --------------------------------------------------------------------


@pytest.mark.parametrize("dim", [320, 64])
@pytest.mark.parametrize("tdtype", ["float32", "int64"])
def test_timestep_embedding_matches_oracle(dim, tdtype):
    ts = np.array([999, 981, 500, 21, 1, 0])
    got = ops.timestep_embedding(cuda(ts.astype(np.float32 if tdtype == "float32" else np.int64)), dim).numpy()
    ref = oracle.timestep_embedding_f32(ts.astype(np.float32), dim)
    half = dim // 2
    freq = np.exp(-np.log(10000.0) * np.arange(half) / half)
    arg = np.abs(ts[:, None] * freq[None])
    tol = 4 * 2.0 ** -23 * np.concatenate([arg, arg], 1) + 1e-6
    assert np.all(np.abs(got - ref) <= tol)


def test_timestep_embedding_broadcast_and_bf16():
    t = cuda(np.array([741], np.int64))
    one = ops.timestep_embedding(t, 320).numpy()
    many = ops.timestep_embedding(t, 320, batch=5).numpy()
    for r in range(5):
        np.testing.assert_array_equal(many[r], one[0])
    b = ops.timestep_embedding(t, 320, dtype="bfloat16", batch=3)
    assert b.dtype is mt.bfloat16
    check(npw(b)[0], one[0], 2e-2)
    with pytest.raises(RuntimeError):
        ops.timestep_embedding(t, 321)


# ---- guidance + DDIM with a device timestep ------------------------------------------------


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_ddim_indexed_matches_host_scalar_step(dtype):
    rng = np.random.default_rng(7)
    sched = U.DDIM(steps=50)
    ac = mt.tensor(sched.alphas_cumprod, dtype="float64").cuda()
    x = cuda(rng.standard_normal((3, 4, 8, 8)).astype(np.float32), dtype)
    e = cuda(rng.standard_normal((3, 4, 8, 8)).astype(np.float32), dtype)
    for t in (sched.timesteps[0], sched.timesteps[25], sched.timesteps[-1]):
        ref = sched.step(x, e, t).numpy()
        got = ops.ddim_step_indexed(x, e, ac, cuda(np.array([t], np.int64)), sched.interval).numpy()
        if dtype == "float32":
            np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)
        else:
            check(got, ref, 1e-2)


def test_cfg_ddim_matches_oracle_and_writes_both_copies():
    rng = np.random.default_rng(8)
    n = 2
    sched = U.DDIM(steps=50)
    ac = mt.tensor(sched.alphas_cumprod, dtype="float64").cuda()
    x = rng.standard_normal((n, 4, 8, 8)).astype(np.float32)
    eps = rng.standard_normal((2 * n, 4, 8, 8)).astype(np.float32)
    t = int(sched.timesteps[30])
    a_t, a_p = sched.alphas(t)
    ref = oracle.cfg_ddim_f32(x, eps, 7.5, a_t, a_p)
    buf = mt.empty(2 * n, 4, 8, 8, device="cuda")
    buf[0:n].copy_(cuda(x))
    got = ops.ddim_step_indexed(buf[0:n], cuda(eps), ac, cuda(np.array([t], np.int64)), sched.interval,
                                guidance_scale=7.5, out=buf, out_copies=2).numpy()
    check(got[:n], ref, 1e-5)
    np.testing.assert_array_equal(got[:n], got[n:])
    with pytest.raises(ValueError):
        ops.ddim_step_indexed(cuda(x), cuda(x), ac, cuda(np.array([t], np.int64)), sched.interval, guidance_scale=2.0)


# ---- embedding, quick GELU -----------------------------------------------------------------


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_embedding_gather_is_exact(dtype):
    rng = np.random.default_rng(9)
    w = rng.standard_normal((50, 24)).astype(np.float32)
    pw = rng.standard_normal((7, 24)).astype(np.float32)
    ids = np.array([[0, 49, -1, 17, 3, 3, -50], [9, 8, 7, 6, 5, 4, 3]], np.int64)
    pos = np.broadcast_to(np.arange(7), (2, 7)).copy()
    wt, pt = cuda(w, dtype), cuda(pw, dtype)
    wr, pr = npw(wt), npw(pt)  # the tables as stored (rounded to dtype)
    ref, bad = oracle.embedding_f32(wr, ids)
    assert bad == 0
    np.testing.assert_array_equal(npw(ops.embedding(mt.tensor(ids), wt)), npw(mt.tensor(ref, dtype=dtype)))
    ref2, _ = oracle.embedding_f32(wr, ids, pr, pos)
    got2 = ops.embedding(cuda(ids), wt, add_weight=pt, add_input=mt.tensor(pos))  # device ids, host positions
    np.testing.assert_array_equal(npw(got2), npw(mt.tensor(ref2, dtype=dtype)))


def test_embedding_out_of_range_raises_index_error():
    w = cuda(np.ones((5, 8), np.float32))
    with pytest.raises(IndexError):
        ops.embedding(mt.tensor(np.array([0, 5], np.int64)), w)
    with pytest.raises(IndexError):
        ops.embedding(cuda(np.array([1, -6], np.int64)), w)
    np.testing.assert_array_equal(ops.embedding(cuda(np.array([4, -5], np.int64)), w).numpy(), np.ones((2, 8)))


def test_quick_gelu_unary_and_gemm_epilogue():
    rng = np.random.default_rng(10)
    x = (rng.standard_normal(4099) * 4).astype(np.float32)
    check(ops.quick_gelu(cuda(x)).numpy(), oracle.quick_gelu_f32(x))
    check(npw(ops.quick_gelu(cuda(x, "bfloat16"))), oracle.quick_gelu_f32(npw(cuda(x, "bfloat16"))), 2e-2)
    a = rng.standard_normal((200, 96)).astype(np.float32)
    w = (rng.standard_normal((136, 96)) * 0.1).astype(np.float32)
    b = rng.standard_normal(136).astype(np.float32)
    ref = oracle.quick_gelu_f32(oracle.linear_f32(a, w, b))
    check(ops.linear(cuda(a), cuda(w), cuda(b), epilogue=L.EPI_QUICK_GELU).numpy(), ref)
    ab, wb, bb = cuda(a, "bfloat16"), cuda(w, "bfloat16"), cuda(b, "bfloat16")
    refb = oracle.quick_gelu_f32(oracle.linear_f32(npw(ab), npw(wb), npw(bb)))
    check(npw(ops.linear(ab, wb, bb, epilogue=L.EPI_QUICK_GELU)), refb, 2e-2)


# ---- sampler: guidance, device timestep, CUDA graph ------------------------------------------


def _tiny_unet():
    mt.manual_seed(0)
    return U.UNet(chans=(64, 128), attn=(True, False), layers=1, heads=2, ctx_dim=64, device="cuda",
                  dtype="bfloat16")


def test_sampler_graph_matches_eager_and_composition():
    net = _tiny_unet()
    rng = np.random.default_rng(11)
    n = 2
    lat = cuda(rng.standard_normal((n, 4, 16, 16)).astype(np.float32), "bfloat16")
    ctx = cuda(rng.standard_normal((n, 5, 64)).astype(np.float32), "bfloat16")
    unc = cuda(rng.standard_normal((n, 5, 64)).astype(np.float32), "bfloat16")
    sched = U.DDIM(steps=50)
    eager = U.Sampler(net, sched, ctx, uncond_ctx=unc, guidance_scale=7.5)(lat, steps=3).numpy()
    graphed = U.Sampler(net, sched, ctx, uncond_ctx=unc, guidance_scale=7.5, graph=True)
    g1 = graphed(lat, steps=3).numpy()
    np.testing.assert_array_equal(g1, eager)
    np.testing.assert_array_equal(graphed(lat, steps=3).numpy(), eager)  # replays restart from the latents
    # the same three steps composed from separate ops: cat, UNet, guidance by elementwise ops,
    # host-scalar DDIM step
    x = lat
    ctx2 = ops.cat([unc, ctx], dim=0)
    for t in sched.timesteps[:3]:
        te = ops.timestep_embedding(cuda(np.array([t], np.int64)), 64, dtype="bfloat16", batch=2 * n)
        e = net(ops.cat([x, x], dim=0), te, ctx2).float()
        eu, et = e[0:n], e[n:2 * n]
        guided = eu + (et - eu) * 7.5
        x = sched.step(x.float(), guided, t).to(dtype="bfloat16")
    check(eager.astype(np.float32), npw(x), 2e-2)


def test_sampler_without_guidance_matches_denoise_loop():
    net = _tiny_unet()
    rng = np.random.default_rng(12)
    lat = cuda(rng.standard_normal((2, 4, 16, 16)).astype(np.float32), "bfloat16")
    ctx = cuda(rng.standard_normal((2, 5, 64)).astype(np.float32), "bfloat16")
    sched = U.DDIM(steps=50)
    got = U.Sampler(net, sched, ctx, graph=True)(lat, steps=2).numpy().astype(np.float32)
    ref = npw(U.denoise(net, lat, ctx, sched, steps=2))  # host-built embedding, host-scalar steps
    check(got, ref, 2e-2)


# ---- CLIP text encoder, VAE decoder ----------------------------------------------------------


def test_clip_text_encoder_fp32_matches_oracle():
    from mtorch_b200.text_encoder import CLIPTextEncoder

    mt.manual_seed(5)
    enc = CLIPTextEncoder(vocab=100, positions=77, width=64, layers=2, heads=4, mlp=256, device="cuda")
    ids = (np.arange(2 * 77).reshape(2, 77) * 7 + 3) % 100
    got = enc(mt.tensor(ids)).numpy()
    n, s, c, H = 2, 77, 64, 4
    h, _ = oracle.embedding_f32(npw(enc.token_embedding), ids, npw(enc.position_embedding),
                                np.broadcast_to(np.arange(s), (n, s)))
    h = h.reshape(n * s, c)
    heads = lambda a: a.reshape(n, s, H, c // H).transpose(0, 2, 1, 3)  # noqa: E731
    for ly in enc.layers:
        y = oracle.layer_norm_f32(h, npw(ly.norm1.weight), npw(ly.norm1.bias))
        qkv = oracle.linear_f32(y, npw(ly.qkv.weight), npw(ly.qkv.bias))
        o = oracle.sdpa_f32(heads(qkv[:, :c]), heads(qkv[:, c:2 * c]), heads(qkv[:, 2 * c:]), causal=True)
        h = h + oracle.linear_f32(o.transpose(0, 2, 1, 3).reshape(n * s, c), npw(ly.out.weight), npw(ly.out.bias))
        y = oracle.layer_norm_f32(h, npw(ly.norm2.weight), npw(ly.norm2.bias))
        y = oracle.quick_gelu_f32(oracle.linear_f32(y, npw(ly.fc1.weight), npw(ly.fc1.bias)))
        h = h + oracle.linear_f32(y, npw(ly.fc2.weight), npw(ly.fc2.bias))
    ref = oracle.layer_norm_f32(h, npw(enc.final_norm.weight), npw(enc.final_norm.bias)).reshape(n, s, c)
    check(got, ref)


def test_clip_text_encoder_bf16_runs_and_is_batch_independent():
    from mtorch_b200.text_encoder import CLIPTextEncoder

    mt.manual_seed(6)
    enc = CLIPTextEncoder(vocab=1000, width=128, layers=2, heads=2, mlp=512, device="cuda", dtype="bfloat16")
    ids = (np.arange(3 * 77).reshape(3, 77) * 13) % 1000
    y = npw(enc(mt.tensor(ids)))
    assert y.shape == (3, 77, 128) and np.isfinite(y).all()
    np.testing.assert_array_equal(npw(enc(mt.tensor(ids[1:]))), y[1:])


def _up2x(a):
    return a.repeat(2, axis=2).repeat(2, axis=3)


def _vae_resnet_ref(blk, x):
    h = oracle.silu_f32(oracle.group_norm_f32(x, 32, npw(blk.norm1.weight), npw(blk.norm1.bias), eps=1e-6))
    h = oracle.conv2d_f32(h, npw(blk.conv1.weight), npw(blk.conv1.bias), 1, 1)
    h = oracle.silu_f32(oracle.group_norm_f32(h, 32, npw(blk.norm2.weight), npw(blk.norm2.bias), eps=1e-6))
    h = oracle.conv2d_f32(h, npw(blk.conv2.weight), npw(blk.conv2.bias), 1, 1)
    sc = x if blk.conv_shortcut is None else oracle.conv2d_f32(x, npw(blk.conv_shortcut.weight),
                                                               npw(blk.conv_shortcut.bias))
    return h + sc


def test_vae_decoder_fp32_matches_oracle():
    from mtorch_b200.vae import VAEDecoder, VAEResnetBlock

    mt.manual_seed(7)
    dec = VAEDecoder(chans=(32, 64), layers=1, device="cuda")
    rng = np.random.default_rng(13)
    z = rng.standard_normal((2, 4, 8, 8)).astype(np.float32)
    got = dec(cuda(z)).numpy()
    h = oracle.conv2d_f32(z, npw(dec.post_quant_conv.weight), npw(dec.post_quant_conv.bias))
    h = oracle.conv2d_f32(h, npw(dec.conv_in.weight), npw(dec.conv_in.bias), 1, 1)
    h = _vae_resnet_ref(dec.mid1, h)
    a = dec.mid_attn
    n, c, hh, ww = h.shape
    t = oracle.group_norm_f32(h, 32, npw(a.norm.weight), npw(a.norm.bias), eps=1e-6)
    t = t.transpose(0, 2, 3, 1).reshape(n, hh * ww, c)
    qkv = oracle.linear_f32(t.reshape(-1, c), npw(a.to_qkv.weight), npw(a.to_qkv.bias)).reshape(n, hh * ww, 3 * c)
    o = oracle.sdpa_f32(qkv[:, None, :, :c], qkv[:, None, :, c:2 * c], qkv[:, None, :, 2 * c:])[:, 0]
    o = oracle.linear_f32(o.reshape(-1, c), npw(a.to_out.weight), npw(a.to_out.bias)).reshape(n, hh, ww, c)
    h = h + o.transpose(0, 3, 1, 2)
    h = _vae_resnet_ref(dec.mid2, h)
    for m in dec.up:
        if isinstance(m, VAEResnetBlock):
            h = _vae_resnet_ref(m, h)
        else:
            h = oracle.conv2d_f32(_up2x(h), npw(m.conv.weight), npw(m.conv.bias), 1, 1)
    h = oracle.silu_f32(oracle.group_norm_f32(h, 32, npw(dec.norm_out.weight), npw(dec.norm_out.bias), eps=1e-6))
    ref = oracle.conv2d_f32(h, npw(dec.conv_out.weight), npw(dec.conv_out.bias), 1, 1)
    assert got.shape == (2, 3, 16, 16)
    check(got, ref)


def test_vae_decoder_bf16_batch_independent():
    from mtorch_b200.vae import VAEDecoder

    mt.manual_seed(8)
    dec = VAEDecoder(chans=(32, 64, 64), layers=1, device="cuda", dtype="bfloat16")
    z = cuda(np.random.default_rng(14).standard_normal((3, 4, 16, 16)).astype(np.float32), "bfloat16")
    y = npw(dec(z))
    assert y.shape == (3, 3, 64, 64) and np.isfinite(y).all()
    np.testing.assert_array_equal(npw(dec(z[1:])), y[1:])
