"""Generates tests/golden/reference_unet.npz: a whole UNet forward + one DDIM step computed by the
REFERENCE mtorch (its own portable CPU code, built from the reference sources by
oracle/build_ref.py), through its public API, in the composition of oracle/unet.py.

Parameters and inputs come from mtorch.manual_seed + mtorch.randn in param_spec order (scaled by
powers of two), so mtorch_b200's bit-identical host generator rebuilds them on any machine and the
fixture holds only the inputs and outputs.  Run here (where the reference tree exists):

    python tests/golden/make_golden_unet.py
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build_ref  # noqa: E402
from oracle import unet as OU  # noqa: E402

build_ref.build()
sys.path.insert(0, str(build_ref.OUT))
import mtorch  # noqa: E402

cfg = OU.GOLDEN_CFG
ops = OU.ReferenceOps(mtorch)
mtorch.manual_seed(cfg["param_seed"])
P = OU.make_params(cfg, lambda shape: mtorch.randn(*shape), ops)
mtorch.manual_seed(cfg["input_seed"])
x, ctx, temb = OU.make_inputs(cfg, lambda shape: mtorch.randn(*shape))
t0 = time.time()
eps = OU.unet_forward(P, x, mtorch.tensor(temb.tolist()), ctx, cfg, ops)
x_next = OU.ddim_step(x, eps, cfg["timestep"], ops)
dt = time.time() - t0
spec = OU.param_spec(cfg)
out = dict(x=x.numpy(), ctx=ctx.numpy(), temb=temb, eps=eps.numpy(), x_next=x_next.numpy(),
           param_names=np.array([n for n, _ in spec]), param_checksum=np.array(
               [float(np.abs(P[n].numpy()).astype(np.float64).sum()) for n, _ in spec]))
np.savez_compressed(ROOT / "tests" / "golden" / "reference_unet.npz", **out)
print(f"reference UNet forward + DDIM step: {dt:.1f} s; eps max {np.abs(out['eps']).max():.3f}")
