"""The CTA-pair GEMM variant (clusters of two CTAs, tcgen05 cta_group::2 MMAs of 256 rows, each
CTA staging half of the B columns) is opt-in through MT_GEMM_PAIR=1, read once per process, so
its parity checks run in a child process with the variable set: 16-bit GEMMs with 160- and
256-wide column tiles, a GEGLU projection (128-wide), odd row-tile counts (the last pair has one
real tile), and implicit-GEMM convolutions at stride 1 (160-wide) and 2 (128-wide), against the oracle at the bf16
tolerance (rtol 2e-2 against fp32 on the same bf16-rounded inputs)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

CHILD = r'''
import numpy as np
import oracle
import mtorch_b200 as mt
from mtorch_b200 import _lib as L, ops

R = 2e-2
def check(got, ref):
    np.testing.assert_allclose(got, ref, rtol=R, atol=R * np.abs(ref).max())
def bf(a):
    return mt.tensor(a, dtype="bfloat16").numpy()
rng = np.random.default_rng(0)
# enough row tiles that no narrower column tile is chosen; odd row-tile counts included
for M, N, K in [(20000, 256, 128), (20001, 320, 128), (19100, 160, 64)]:
    a = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    got = ops.linear(mt.tensor(a, dtype="bfloat16").cuda(), mt.tensor(w, dtype="bfloat16").cuda(),
                     mt.tensor(b, dtype="bfloat16").cuda()).numpy()
    check(got, oracle.linear_f32(bf(a), bf(w), bf(b)))
a = rng.standard_normal((512, 320)).astype(np.float32)
w = (rng.standard_normal((2560, 320)) * 0.05).astype(np.float32)
wi = w.reshape(2, 20, 64, 320).transpose(1, 0, 2, 3).reshape(2560, 320)
h = oracle.linear_f32(bf(a), bf(w))
ref = h[:, :1280] * oracle.gelu_f32(h[:, 1280:])
got = ops.linear(mt.tensor(a, dtype="bfloat16").cuda(), mt.tensor(wi, dtype="bfloat16").cuda(),
                 epilogue=L.EPI_GEGLU).numpy()
check(got, ref)
for N, C, H, K, s in [(5, 64, 48, 320, 1), (8, 64, 64, 512, 2)]:
    x = rng.standard_normal((N, C, H, H)).astype(np.float32)
    w = (rng.standard_normal((K, C, 3, 3)) * 0.03).astype(np.float32)
    xc = mt.tensor(x, dtype="bfloat16").cuda().contiguous(memory_format=mt.channels_last)
    got = mt.conv2d(xc, mt.tensor(w, dtype="bfloat16").cuda(), None, s, 1).numpy()
    check(got, oracle.conv2d_f32(bf(x), bf(w), None, s, 1))
print("pair-ok")
'''


def test_pair_variant_parity():
    env = dict(os.environ, MT_GEMM_PAIR="1")
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "pair-ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
