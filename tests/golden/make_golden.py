"""Generates tests/golden/reference_ops.npz by running the REFERENCE mtorch (its own portable CPU
code, built from the reference sources by oracle/build_ref.py) on small seeded inputs.

Inputs come from mtorch.manual_seed + mtorch.randn/rand in a fixed order, so the fixture also
pins the seeded generator.  Run here (where the reference tree exists):

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import build_ref  # noqa: E402

build_ref.build()
sys.path.insert(0, str(build_ref.OUT))
import mtorch  # noqa: E402

F = mtorch.nn.functional
out: dict[str, np.ndarray] = {}


def rec(name, **arrays):
    for k, v in arrays.items():
        out[f"{name}.{k}"] = np.asarray(v.numpy() if hasattr(v, "numpy") else v)


mtorch.manual_seed(0)
rec("rng", randn=mtorch.randn(7), rand=mtorch.rand(5), randn_odd=mtorch.randn(3), randn_after=mtorch.randn(4))

mtorch.manual_seed(1)
a, b = mtorch.randn(33, 47), mtorch.randn(47, 29)
rec("matmul", a=a, b=b, y=mtorch.matmul(a, b))

mtorch.manual_seed(2)
a, b = mtorch.randn(3, 20, 24), mtorch.randn(3, 24, 18)
rec("bmm", a=a, b=b, y=mtorch.bmm(a, b))

mtorch.manual_seed(3)
i, a, b = mtorch.randn(16, 12), mtorch.randn(16, 40), mtorch.randn(40, 12)
rec("addmm", i=i, a=a, b=b, y=mtorch.addmm(i, a, b, beta=0.5, alpha=2.0))

mtorch.manual_seed(40)
i, a, b = mtorch.randn(3, 1, 14), mtorch.randn(3, 18, 33), mtorch.randn(3, 33, 14)
rec("baddbmm", i=i, a=a, b=b, y=mtorch.baddbmm(i, a, b, beta=-0.75, alpha=1.5))

mtorch.manual_seed(4)
x, w, bias = mtorch.randn(3, 17, 40), mtorch.randn(24, 40), mtorch.randn(24)
rec("linear", x=x, w=w, b=bias, y=F.linear(x, w, bias))

conv_cases = {
    "conv_p1": dict(shape=(2, 8, 9, 9), w=(6, 8, 3, 3), stride=1, padding=1, dilation=1, groups=1),
    "conv_s2": dict(shape=(1, 4, 10, 10), w=(5, 4, 3, 3), stride=2, padding=1, dilation=1, groups=1),
    "conv_d2": dict(shape=(1, 3, 11, 11), w=(4, 3, 3, 3), stride=1, padding=2, dilation=2, groups=1),
    "conv_1x1": dict(shape=(2, 16, 5, 7), w=(8, 16, 1, 1), stride=1, padding=0, dilation=1, groups=1),
    "conv_g4": dict(shape=(2, 8, 7, 7), w=(12, 2, 3, 3), stride=1, padding=1, dilation=1, groups=4),
}
for seed, (name, c) in enumerate(conv_cases.items(), start=10):
    mtorch.manual_seed(seed)
    x, w, bias = mtorch.randn(*c["shape"]), mtorch.randn(*c["w"]), mtorch.randn(c["w"][0])
    y = F.conv2d(x, w, bias, stride=c["stride"], padding=c["padding"], dilation=c["dilation"], groups=c["groups"])
    rec(name, x=x, w=w, b=bias, y=y, params=np.array([c["stride"], c["padding"], c["dilation"], c["groups"]]))

mtorch.manual_seed(20)
q, k, v = mtorch.randn(2, 3, 17, 8), mtorch.randn(2, 3, 17, 8), mtorch.randn(2, 3, 17, 8)
rec("sdpa_self", q=q, k=k, v=v, y=F.scaled_dot_product_attention(q, k, v))
rec("sdpa_causal", q=q, k=k, v=v, y=F.scaled_dot_product_attention(q, k, v, is_causal=True))
mtorch.manual_seed(21)
q, k, v = mtorch.randn(2, 2, 9, 16), mtorch.randn(2, 2, 5, 16), mtorch.randn(2, 2, 5, 12)
rec("sdpa_cross", q=q, k=k, v=v, y=F.scaled_dot_product_attention(q, k, v, scale=0.3))
fm = mtorch.randn(9, 5)
rec("sdpa_fmask", q=q, k=k, v=v, m=fm, y=F.scaled_dot_product_attention(q, k, v, attn_mask=fm))
bm_np = (np.arange(45).reshape(9, 5) % 3 != 1)
bm = mtorch.tensor(bm_np.tolist(), dtype=mtorch.bool)
rec("sdpa_bmask", q=q, k=k, v=v, m=bm_np, y=F.scaled_dot_product_attention(q, k, v, attn_mask=bm))

mtorch.manual_seed(30)
x = mtorch.randn(7, 33)
rec("softmax", x=x, y=F.softmax(x, dim=-1))
x, w, bias = mtorch.randn(2, 8, 5, 5), mtorch.randn(8), mtorch.randn(8)
rec("group_norm", x=x, w=w, b=bias, y=F.group_norm(x, 4, w, bias, eps=1e-5))
x, w, bias = mtorch.randn(5, 32), mtorch.randn(32), mtorch.randn(32)
rec("layer_norm", x=x, w=w, b=bias, y=F.layer_norm(x, [32], w, bias, eps=1e-5))
x = mtorch.randn(257) * 3.0
rec("silu", x=x, y=F.silu(x))
rec("gelu", x=x, y=F.gelu(x))
rec("gelu_tanh", x=x, y=F.gelu(x, approximate="tanh"))

# Scheduler / text-encoder ops around the UNet (appended after the cases above so their seeded
# inputs are unchanged).  Each follows the reference's own scenario code in
# tests/compat/benchmarking.py, written against the public API.
t = mtorch.tensor([999.0, 500.0, 1.0, 0.0], dtype=mtorch.float32)
exponent = -mtorch.log(mtorch.tensor(10000.0, dtype=mtorch.float32)) * mtorch.arange(0, 160, dtype=mtorch.float32) / 160
args = t.reshape(-1, 1) * mtorch.exp(exponent).reshape(1, -1)  # 6016-6021, 6035
rec("tsemb", t=t, y=mtorch.cat([mtorch.cos(args), mtorch.sin(args)], dim=-1))  # 6036

mtorch.manual_seed(40)
x = mtorch.randn(300) * 3.0
rec("quick_gelu", x=x, y=x * mtorch.sigmoid(x * 1.702))  # 7714

mtorch.manual_seed(41)
w, pw = mtorch.randn(11, 6), mtorch.randn(4, 6)
ids = mtorch.tensor([[0, 3, -1, 10], [5, 5, 2, -11]], dtype=mtorch.long)
pos = mtorch.tensor([[0, 1, 2, 3], [0, 1, 2, 3]], dtype=mtorch.long)
rec("embedding", w=w, pw=pw, ids=ids, pos=pos, y=F.embedding(ids, w) + F.embedding(pos, pw))  # 5235-5236

mtorch.manual_seed(42)
uncond, text, cur = mtorch.randn(2, 4, 3, 3), mtorch.randn(2, 4, 3, 3), mtorch.randn(2, 4, 3, 3)
noise = uncond + (text - uncond) * 7.5  # 5847-5850
betas = mtorch.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 16, dtype=mtorch.float32) ** 2  # 6138-6141
alphas_cumprod = mtorch.cumprod(1.0 - betas, dim=0)
a_t, a_prev = alphas_cumprod[10], alphas_cumprod[6]
pred_original = ((cur - (1.0 - a_t).sqrt() * noise) / a_t.sqrt()).clamp(-1.0, 1.0)  # 6158-6164
pred_epsilon = (cur - a_t.sqrt() * pred_original) / (1.0 - a_t).sqrt()
step = a_prev.sqrt() * pred_original + (1.0 - a_prev).sqrt() * pred_epsilon
rec("cfg_ddim", x=cur, eps=mtorch.cat([uncond, text], dim=0), a=mtorch.stack([a_t, a_prev]), y=step)

path = Path(__file__).resolve().parent / "reference_ops.npz"
np.savez_compressed(path, **out)
print(f"wrote {path} ({len(out)} arrays)")
