"""The persistent norm kernels against the kernels they replace, on the same inputs.

`gn_partial_cl_bf16x8_persist_kernel` (GroupNorm statistics, one CTA walking several
(image, chunk) items) sums every slot in the same order as `gn_partial_cl_bf16x8_kernel` (one
item per CTA), so GroupNorm outputs must be bitwise equal with either (`MT_GN_PERSIST=0`
selects the old kernel).  `layer_norm_bf16_persist_kernel` evaluates the same per-row sequence
as `layer_norm_bf16_sub_kernel` (`MT_LN_PERSIST=0`); its outputs are checked to within one
bf16 rounding step.  The switches are read once per process, so each variant runs in its own
child process.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import mtorch_b200 as mt

def cu(a, dtype=None):
    t = mt.tensor(np.asarray(a, np.float32))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()

out = {}
rng = np.random.default_rng(7)
# GroupNorm + SiLU, channels-last bf16: one source and the two-source skip concatenation
for n, c, hw in [(12, 320, 64), (6, 640, 32), (5, 1280, 16), (9, 960, 20)]:
    x = (rng.standard_normal((n, c, hw, hw)) * 1.3 + 0.2).astype(np.float32)
    w = rng.standard_normal(c).astype(np.float32)
    b = rng.standard_normal(c).astype(np.float32)
    xd = cu(x, "bfloat16").contiguous(memory_format=mt.channels_last)
    out[f"gn_{n}_{c}_{hw}"] = mt.group_norm(xd, 32, cu(w), cu(b), fuse_silu=True).numpy()
    c1 = c // 128 * 64  # both halves multiples of 64 channels (the skip concatenation's layout)
    x1 = cu(x[:, :c1], "bfloat16").contiguous(memory_format=mt.channels_last)
    x2 = cu(x[:, c1:], "bfloat16").contiguous(memory_format=mt.channels_last)
    out[f"gncat_{n}_{c}_{hw}"] = mt.ops.group_norm_cat(x1, x2, 32, cu(w, "bfloat16"), cu(b, "bfloat16"),
                                                       fuse_silu=True).numpy()
# LayerNorm over the UNet's widths (rows not a multiple of a CTA's row group)
for rows, cols in [(4099, 320), (1027, 640), (515, 1280)]:
    x = (rng.standard_normal((rows, cols)) * 2.0 - 0.5).astype(np.float32)
    w = rng.standard_normal(cols).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    out[f"ln_{rows}_{cols}"] = mt.layer_norm(cu(x, "bfloat16"), [cols], cu(w, "bfloat16"), cu(b, "bfloat16")).numpy()
np.savez(sys.argv[2], **out)
"""


def _run(tmp_path, name, env_extra):
    path = tmp_path / f"{name}.npz"
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(path)], env=env, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    return dict(np.load(path))


def test_persistent_norm_kernels_match_replaced_kernels(tmp_path):
    new = _run(tmp_path, "persist", {"MT_GN_PERSIST": "1", "MT_LN_PERSIST": "1"})
    old = _run(tmp_path, "plain", {"MT_GN_PERSIST": "0", "MT_LN_PERSIST": "0"})
    assert new.keys() == old.keys()
    for k in new:
        if k.startswith("gn"):
            np.testing.assert_array_equal(new[k], old[k], err_msg=k)
        else:
            # one bf16 step (2^-8 relative) at most
            np.testing.assert_allclose(new[k], old[k], rtol=2.0 ** -7, atol=1e-6, err_msg=k)
