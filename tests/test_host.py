"""Host-side logic that needs no GPU: the C ABI library exports every header symbol, the seeded
generator is bit-identical to mtorch's, tensor metadata / views, dtype parsing, error paths."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import mtorch_b200 as mt
from mtorch_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "mtorch_cuda.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mt_(?:cuda|rng)_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) <= set(_lib.SIGNATURES), set(syms) - set(_lib.SIGNATURES)


def test_no_gpu_calls_are_safe():
    lib = _lib.lib()
    assert lib.mt_cuda_device_count() >= 0
    assert lib.mt_cuda_gemm(None, None, 0, None) == _lib.MT_ERR_INVALID
    assert b"null descriptor" in lib.mt_cuda_last_error_string()


def test_workspace_queries_without_gpu():
    d = _lib.GemmDesc()
    d.M, d.N, d.K, d.batch = 64, 64, 64, 1
    d.dtype = d.out_dtype = _lib.MT_F32
    d.A = d.B = d.D = 16
    d.lda = d.ldb = d.ldd = 64
    d.b_trans = 0
    ws = _lib.lib().mt_cuda_gemm_workspace_size(ctypes.byref(d))
    # fp32 needs lo parts of A and B, and B is transposed: 3 x 64*64*4 bytes at least
    assert ws >= 3 * 64 * 64 * 4
    d.dtype = d.out_dtype = _lib.MT_BF16
    d.b_trans = 1
    assert _lib.lib().mt_cuda_gemm_workspace_size(ctypes.byref(d)) == 0


def test_rng_matches_reference_golden(golden):
    mt.manual_seed(0)
    np.testing.assert_array_equal(mt.randn(7).numpy(), golden["rng.randn"])
    np.testing.assert_array_equal(mt.rand(5).numpy(), golden["rng.rand"])
    np.testing.assert_array_equal(mt.randn(3).numpy(), golden["rng.randn_odd"])
    np.testing.assert_array_equal(mt.randn(4).numpy(), golden["rng.randn_after"])  # uses the spare normal
    mt.manual_seed(1)
    np.testing.assert_array_equal(mt.randn(33, 47).numpy(), golden["matmul.a"])


def test_views_are_metadata():
    x = mt.tensor(np.arange(24, dtype=np.float32).reshape(2, 3, 4))
    assert x.permute(2, 0, 1).shape == (4, 2, 3)
    assert x.permute(2, 0, 1).stride() == (1, 12, 4)
    np.testing.assert_array_equal(x.transpose(0, 2).numpy(), np.arange(24).reshape(2, 3, 4).transpose(2, 1, 0))
    np.testing.assert_array_equal(x[:, 1:, ::2].numpy(), np.arange(24).reshape(2, 3, 4)[:, 1:, ::2])
    np.testing.assert_array_equal(x[..., 1].numpy(), np.arange(24).reshape(2, 3, 4)[..., 1])
    a, b = x.chunk(2, dim=-1)
    np.testing.assert_array_equal(b.numpy(), np.arange(24).reshape(2, 3, 4)[..., 2:])
    assert x.unsqueeze(1).shape == (2, 1, 3, 4)
    assert x[None].expand(5, 2, 3, 4).stride()[0] == 0


def test_dtype_parsing_bf16_is_not_fp16():
    assert mt.tensor([1.0]).to("bfloat16").dtype is mt.bfloat16
    assert mt.tensor([1.0]).to(dtype="torch.bfloat16").dtype is mt.bfloat16
    with pytest.raises(TypeError):
        mt.tensor([1.0]).to(dtype="complex64")


def test_bf16_round_trip_rounds_to_nearest_even():
    v = np.array([1.0, 1.00390625, 1.01171875, -3.1415926, 65504.0], np.float32)
    got = mt.tensor(v).to("bfloat16").numpy()
    import torch

    np.testing.assert_array_equal(got, torch.tensor(v).to(torch.bfloat16).float().numpy())


def test_cpu_compute_raises_not_silently_falls_back():
    x = mt.randn(4, 4)
    with pytest.raises(NotImplementedError):
        mt.matmul(x, x)
    with pytest.raises(NotImplementedError):
        _ = x + x


def test_mps_raises_like_reference():
    with pytest.raises(NotImplementedError):
        mt.device("mps")


def test_module_init_is_seeded_and_deterministic():
    mt.manual_seed(5)
    a = mt.nn.Linear(16, 8).weight.numpy()
    mt.manual_seed(5)
    b = mt.nn.Linear(16, 8).weight.numpy()
    np.testing.assert_array_equal(a, b)
    bound = np.sqrt(3.0) * np.sqrt(2.0 / 6.0) / np.sqrt(16)
    assert np.abs(a).max() <= bound


def test_reference_binding_installs_and_leaves_the_cpu_path_alone():
    """mtorch_b200.compat.install patches the reference package in place: `cuda` becomes a device
    name its Module.to accepts, the functional ops dispatch on device tensors, and calls on the
    reference's own CPU tensors still run the reference's code (same results as before)."""
    import oracle

    m = oracle.ref()
    if m is None:
        pytest.skip("the reference is not built into oracle/_ref")
    F = m.nn.functional
    m.manual_seed(3)
    x, w = m.randn(1, 4, 5, 5), m.randn(6, 4, 3, 3)
    before = F.conv2d(x, w, None, 1, 1).numpy()
    from mtorch_b200 import compat

    compat.install(m)
    compat.install(m)  # idempotent
    assert "cuda" in m._DEVICE_NAMES
    assert m.nn.functional.conv2d.__mtorch_b200_reference__ is not None
    np.testing.assert_array_equal(F.conv2d(x, w, None, 1, 1).numpy(), before)
    np.testing.assert_array_equal(m.cat([x, x], dim=1).numpy()[:, 4:], x.numpy())
