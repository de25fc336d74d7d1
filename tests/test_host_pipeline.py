"""Host-side logic of the workloads around the UNet (no GPU): FLOP models, argument checks that
run before any device work, and the DDIM schedule tables the device kernels index."""
import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import ops
from mtorch_b200 import unet as U
from mtorch_b200.text_encoder import clip_text_flops
from mtorch_b200.vae import vae_decoder_flops


def test_flop_models_match_hand_counts():
    # SD-1.5 VAE decoder at a 64x64 latent: about 1.26 T multiply-adds
    assert abs(vae_decoder_flops() / 2.5145e12 - 1) < 1e-3
    # CLIP ViT-L/14 text tower, 77 tokens: per layer 4 projections + two 77x77 products
    per_layer = 2 * 77 * 768 * (4 * 768 + 2 * 3072) + 4 * 77 * 77 * 768
    assert clip_text_flops() == 12 * per_layer


def test_sampler_guidance_arguments_go_together():
    ctx = mt.zeros(2, 77, 768)
    with pytest.raises(ValueError):
        U.Sampler(None, U.DDIM(), ctx, guidance_scale=7.5)
    with pytest.raises(ValueError):
        U.Sampler(None, U.DDIM(), ctx, uncond_ctx=ctx)


def test_host_embedding_ids_are_range_checked_before_the_copy():
    ids = mt.tensor(np.array([[0, 3], [7, 2]], np.int64))
    with pytest.raises(IndexError):
        ops._ids_on_device(ids, 7, mt.device("cuda"))
    with pytest.raises(ValueError):
        ops._ids_on_device(mt.tensor(np.array([0.5], np.float32)), 7, mt.device("cuda"))


def test_ddim_schedule_is_the_reference_scaled_linear_one():
    s = U.DDIM(steps=50)
    betas = np.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 1000) ** 2
    np.testing.assert_allclose(s.alphas_cumprod, np.cumprod(1 - betas), rtol=1e-12)
    assert s.interval == 20 and s.timesteps[0] == 980 and s.timesteps[-1] == 0
    # the device kernel clamps t - interval at 0, as alphas() does
    assert s.alphas(0) == (s.alphas_cumprod[0], s.alphas_cumprod[0])
