"""Pins the C oracle restatement (oracle/mtorch_oracle.c) against golden outputs of the
reference mtorch itself (tests/golden/reference_ops.npz, made by tests/golden/make_golden.py)."""
import numpy as np
import pytest

import oracle


def close(a, b, rtol=1e-6, atol=1e-6):
    np.testing.assert_allclose(a, b, rtol=rtol, atol=atol)


def test_matmul(golden):
    close(oracle.matmul_f32(golden["matmul.a"], golden["matmul.b"]), golden["matmul.y"], 0, 0)


def test_bmm(golden):
    a, b = golden["bmm.a"], golden["bmm.b"]
    close(np.stack([oracle.matmul_f32(a[i], b[i]) for i in range(a.shape[0])]), golden["bmm.y"], 0, 0)


def test_addmm(golden):
    close(oracle.addmm_f32(golden["addmm.i"], golden["addmm.a"], golden["addmm.b"], 0.5, 2.0), golden["addmm.y"],
          1e-6, 1e-6)


def test_baddbmm(golden):
    i, a, b = golden["baddbmm.i"], golden["baddbmm.a"], golden["baddbmm.b"]
    close(oracle.baddbmm_f32(i, a, b, -0.75, 1.5), golden["baddbmm.y"], 0, 0)


def test_linear(golden):
    close(oracle.linear_f32(golden["linear.x"], golden["linear.w"], golden["linear.b"]), golden["linear.y"], 0, 0)


@pytest.mark.parametrize("name", ["conv_p1", "conv_s2", "conv_d2", "conv_1x1", "conv_g4"])
def test_conv(golden, name):
    s, p, d, g = golden[f"{name}.params"]
    y = oracle.conv2d_f32(golden[f"{name}.x"], golden[f"{name}.w"], golden[f"{name}.b"], int(s), int(p), int(d), int(g))
    close(y, golden[f"{name}.y"], 0, 0)


def test_sdpa(golden):
    q, k, v = golden["sdpa_self.q"], golden["sdpa_self.k"], golden["sdpa_self.v"]
    close(oracle.sdpa_f32(q, k, v), golden["sdpa_self.y"], 1e-6, 1e-7)
    close(oracle.sdpa_f32(q, k, v, causal=True), golden["sdpa_causal.y"], 1e-6, 1e-7)
    q, k, v = golden["sdpa_cross.q"], golden["sdpa_cross.k"], golden["sdpa_cross.v"]
    close(oracle.sdpa_f32(q, k, v, scale=0.3), golden["sdpa_cross.y"], 1e-6, 1e-7)
    close(oracle.sdpa_f32(q, k, v, mask=golden["sdpa_fmask.m"]), golden["sdpa_fmask.y"], 1e-6, 1e-7)
    close(oracle.sdpa_f32(q, k, v, mask=golden["sdpa_bmask.m"].astype(bool)), golden["sdpa_bmask.y"], 1e-6, 1e-7)


def test_norms_and_activations(golden):
    close(oracle.softmax_f32(golden["softmax.x"]), golden["softmax.y"], 1e-6, 1e-7)
    close(oracle.group_norm_f32(golden["group_norm.x"], 4, golden["group_norm.w"], golden["group_norm.b"]),
          golden["group_norm.y"], 1e-6, 1e-6)
    close(oracle.layer_norm_f32(golden["layer_norm.x"], golden["layer_norm.w"], golden["layer_norm.b"]),
          golden["layer_norm.y"], 1e-6, 1e-6)
    close(oracle.silu_f32(golden["silu.x"]), golden["silu.y"], 1e-6, 1e-7)
    close(oracle.gelu_f32(golden["gelu.x"]), golden["gelu.y"], 1e-6, 1e-7)
    close(oracle.gelu_f32(golden["gelu_tanh.x"], "tanh"), golden["gelu_tanh.y"], 1e-6, 1e-7)


def test_pipeline_ops(golden):
    """Timestep embedding, quick GELU, embedding gather + add, and guidance + DDIM step."""
    close(oracle.timestep_embedding_f32(golden["tsemb.t"], 320), golden["tsemb.y"], 0, 2e-6)
    close(oracle.quick_gelu_f32(golden["quick_gelu.x"]), golden["quick_gelu.y"], 1e-6, 1e-7)
    y, bad = oracle.embedding_f32(golden["embedding.w"], golden["embedding.ids"], golden["embedding.pw"],
                                  golden["embedding.pos"])
    assert bad == 0
    close(y, golden["embedding.y"], 0, 0)
    a_t, a_prev = (float(v) for v in golden["cfg_ddim.a"])
    close(oracle.cfg_ddim_f32(golden["cfg_ddim.x"], golden["cfg_ddim.eps"], 7.5, a_t, a_prev), golden["cfg_ddim.y"],
          1e-6, 1e-6)


def test_reference_live_if_built():
    """When the reference is built here, the oracle matches it on a fresh case too."""
    m = oracle.ref()
    if m is None:
        pytest.skip("reference not built in this environment")
    m.manual_seed(99)
    x, w, b = m.randn(1, 5, 6, 6), m.randn(7, 5, 3, 3), m.randn(7)
    y = m.nn.functional.conv2d(x, w, b, padding=1).numpy()
    close(oracle.conv2d_f32(x.numpy(), w.numpy(), b.numpy(), 1, 1), y, 0, 0)


def test_oracle_unet_matches_reference_unet():
    """The whole-UNet oracle composition (oracle/unet.py over the C restatement), with parameters
    and inputs from mtorch_b200's host generator, reproduces the reference's own UNet forward and
    DDIM step (tests/golden/reference_unet.npz) bit for bit."""
    from pathlib import Path

    import mtorch_b200 as mt
    from oracle import unet as OU

    g = np.load(Path(__file__).resolve().parent / "golden" / "reference_unet.npz")
    cfg = OU.GOLDEN_CFG
    mt.manual_seed(cfg["param_seed"])
    P = OU.make_params(cfg, lambda s: mt.randn(*s).numpy(), OU.NumpyOps)
    assert [n for n, _ in OU.param_spec(cfg)] == list(g["param_names"])
    ck = np.array([float(np.abs(P[n]).astype(np.float64).sum()) for n in g["param_names"]])
    np.testing.assert_array_equal(ck, g["param_checksum"])
    mt.manual_seed(cfg["input_seed"])
    x, ctx, temb = OU.make_inputs(cfg, lambda s: mt.randn(*s).numpy())
    for k, v in (("x", x), ("ctx", ctx), ("temb", temb)):
        np.testing.assert_array_equal(v, g[k])
    eps = OU.unet_forward(P, x, temb, ctx, cfg, OU.NumpyOps)
    np.testing.assert_array_equal(eps, g["eps"])
    np.testing.assert_array_equal(OU.ddim_step(x, eps, cfg["timestep"], OU.NumpyOps), g["x_next"])
