"""The reference-side binding (mtorch_b200.compat): the REFERENCE mtorch package, with the `cuda`
device installed, runs its own public API on this library's kernels.

* The reference's own nn modules (Conv2d, GroupNorm, Linear) and functional calls, moved with
  `Module.to('cuda')` / `Tensor.to('cuda')`, give the reference's CPU results (fp32, rtol 1e-4).
* The whole-UNet composition of oracle/unet.py, written against the reference's public API
  (`mtorch.nn.functional.*`, `mtorch.cat`, tensor methods), run through the patched reference
  module on device tensors, reproduces the reference's own UNet output
  (tests/golden/reference_unet.npz) at rtol 1e-4.

Needs the reference built into oracle/_ref (test infrastructure; skipped where it is absent).
"""
import numpy as np
import pytest

import mtorch_b200 as mt
import oracle
from mtorch_b200.tensor import Tensor
from oracle import unet as OU
from tests.conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    m = oracle.ref()
    if m is None:
        pytest.skip("the reference is not built into oracle/_ref")
    from mtorch_b200 import compat

    return compat.install(m)


def scale_err(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return np.abs(got - want).max() / np.abs(want).max()


def test_reference_modules_on_the_device(ref):
    m, F = ref, ref.nn.functional
    m.manual_seed(0)
    conv = m.nn.Conv2d(32, 64, 3, padding=1)
    gn = m.nn.GroupNorm(8, 64)
    lin = m.nn.Linear(64, 48)
    x = m.randn(2, 32, 8, 8)
    q, k, v = m.randn(1, 2, 100, 40), m.randn(1, 2, 77, 40), m.randn(1, 2, 77, 40)

    def run(x, q, k, v):
        h = F.silu(gn(conv(x)))
        t = lin(h.permute(0, 2, 3, 1).reshape(2 * 64, 64))
        return t, F.scaled_dot_product_attention(q, k, v)

    want_t, want_a = run(x, q, k, v)  # the reference's CPU path
    for mod in (conv, gn, lin):
        mod.to("cuda")
    assert isinstance(conv.weight, Tensor) and conv.weight.device.type == "cuda"
    xd = x.to("cuda")
    assert isinstance(xd, Tensor)
    got_t, got_a = run(xd, q.cuda(), k.cuda(), v.cuda())
    assert got_t.device.type == "cuda"
    e1, e2 = scale_err(got_t.numpy(), want_t.numpy()), scale_err(got_a.numpy(), want_a.numpy())
    print(f"reference modules on cuda: conv/GN/SiLU/linear {e1:.2e}, SDPA {e2:.2e}")
    assert e1 <= 1e-4 and e2 <= 1e-4
    # a seeded device factory draws from the reference's own generator
    m.manual_seed(5)
    a = m.randn(3, 4)
    m.manual_seed(5)
    np.testing.assert_array_equal(m.randn(3, 4, device="cuda").numpy(), a.numpy())
    # device ops the library does not have raise instead of falling back
    with pytest.raises(NotImplementedError):
        F.interpolate(xd, scale_factor=3, mode="nearest")


def test_reference_api_unet_on_the_device(ref):
    g = np.load(ROOT / "tests" / "golden" / "reference_unet.npz")
    cfg = OU.GOLDEN_CFG
    # the golden's parameters, drawn with this package's generator (bit-identical to the reference's)
    mt.manual_seed(cfg["param_seed"])
    P = OU.make_params(cfg, lambda s: mt.randn(*s).numpy(), OU.NumpyOps)
    Pd = {k: mt.tensor(v).cuda() for k, v in P.items()}
    x, ctx, temb = (mt.tensor(g[k]).cuda() for k in ("x", "ctx", "temb"))
    eps = OU.unet_forward(Pd, x, temb, ctx, cfg, OU.ReferenceOps(ref))
    assert isinstance(eps, Tensor) and eps.device.type == "cuda"
    e = scale_err(eps.numpy(), g["eps"])
    print(f"reference-API UNet on cuda vs the reference's own output: {e:.2e}")
    assert e <= 1e-4
