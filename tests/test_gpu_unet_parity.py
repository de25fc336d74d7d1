"""Whole-UNet parity: the device UNet (the model bench.py times, at SD-1.5 channel widths 320/640,
head dims 40 and 80) plus one DDIM step, against

* fp32: the REFERENCE mtorch's own output for the same parameters and inputs
  (tests/golden/reference_unet.npz, made by tests/golden/make_golden_unet.py), rtol 1e-4;
* bf16 and fp16: the oracle composition (oracle/unet.py, bit-identical to the reference golden in
  fp32, see test_oracle_pins.py) evaluated in fp32 on the same rounded parameters and inputs,
  rtol 2e-2.

Parameters are drawn from mtorch's seeded generator in the reference's draw order, so the module
holds exactly the values the reference used.  Errors are measured against the output's scale
(atol = rtol * max|ref|): the error of a K-term dot product is bounded by sum |a_i b_i|, not by
|sum a_i b_i|, so an elementwise relative bound is not meaningful where the output cancels.  The
max elementwise relative error over |ref| > 1e-2 * max|ref| is printed beside it.
"""
import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import unet as U
from oracle import unet as OU
from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
CFG = OU.GOLDEN_CFG


def errors(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.abs(ref).max()
    d = np.abs(got - ref)
    big = np.abs(ref) > 1e-2 * scale
    return d.max() / scale, (d[big] / np.abs(ref[big])).max()


def check(name, got, ref, rtol):
    assert got.shape == ref.shape, (got.shape, ref.shape)
    e_scale, e_rel = errors(got, ref)
    print(f"{name}: max|d|/max|ref| = {e_scale:.3e}, max rel (|ref| > 1e-2 max) = {e_rel:.3e}")
    assert e_scale <= rtol, f"{name}: {e_scale:.3e} > {rtol}"


def build_unet(dtype):
    mt.manual_seed(0)
    net = U.UNet(in_ch=CFG["in_ch"], out_ch=CFG["out_ch"], chans=CFG["chans"], attn=CFG["attn"],
                 layers=CFG["layers"], heads=CFG["heads"], ctx_dim=CFG["ctx_dim"], device="cuda", dtype=dtype)
    names = [n for n, _ in net.named_parameters()]
    spec = OU.param_spec(CFG)
    assert names == [n for n, _ in spec], "UNet parameter layout differs from the oracle's"
    mt.manual_seed(CFG["param_seed"])
    P = OU.make_params(CFG, lambda s: mt.randn(*s).numpy(), OU.NumpyOps)
    params = dict(net.named_parameters())
    for n, shape in spec:
        assert tuple(params[n].shape) == shape, n
        params[n].copy_(mt.tensor(P[n]).to(dtype).cuda())
    return net, P


@pytest.fixture(scope="module")
def golden():
    return np.load(ROOT / "tests" / "golden" / "reference_unet.npz")


def run_device(net, x, temb, ctx, dtype):
    xd = mt.tensor(x).to(dtype).cuda()
    eps = net(xd, mt.tensor(temb).to(dtype).cuda(), mt.tensor(ctx).to(dtype).cuda())
    sched = U.DDIM(steps=50)
    x_next = sched.step(xd, eps, CFG["timestep"])
    return eps.float().numpy(), x_next.float().numpy()


def test_unet_fp32_matches_reference(golden):
    net, P = build_unet("float32")
    ck = np.array([float(np.abs(P[n]).astype(np.float64).sum()) for n in golden["param_names"]])
    np.testing.assert_array_equal(ck, golden["param_checksum"])  # same parameters as the reference
    eps, x_next = run_device(net, golden["x"], golden["temb"], golden["ctx"], "float32")
    check("fp32 eps", eps, golden["eps"], 1e-4)
    check("fp32 x_next", x_next, golden["x_next"], 1e-4)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_unet_16bit_matches_oracle(golden, dtype):
    """bf16 (the bench's dtype) and fp16 (the reference's own SD dtype) device UNets."""
    net, P = build_unet(dtype)
    rb = lambda a: mt.tensor(np.asarray(a, np.float32)).to(dtype).float().numpy()  # noqa: E731
    Pb = {k: rb(v) for k, v in P.items()}
    x, ctx, temb = rb(golden["x"]), rb(golden["ctx"]), rb(golden["temb"])
    ref_eps = OU.unet_forward(Pb, x, temb, ctx, CFG, OU.NumpyOps)
    ref_next = OU.ddim_step(x, ref_eps, CFG["timestep"], OU.NumpyOps)
    eps, x_next = run_device(net, x, temb, ctx, dtype)
    check(f"{dtype} eps", eps, ref_eps, 2e-2)
    check(f"{dtype} x_next", x_next, ref_next, 2e-2)

