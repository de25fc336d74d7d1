"""ctypes binding of ``libmtorch_cuda.so`` (declared in ``include/mtorch_cuda.h``).

Loading is lazy and LOUD: if the library is missing, ``lib()`` raises instead of letting any
caller fall back to another implementation.  The struct layouts below mirror the header exactly.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libmtorch_cuda.so"

MT_F32, MT_BF16, MT_F16, MT_F64, MT_I32, MT_I64, MT_BOOL = range(7)
MT_OK, MT_ERR_INVALID, MT_ERR_UNSUPPORTED, MT_ERR_LAUNCH, MT_ERR_TIMEOUT, MT_ERR_WORKSPACE = range(6)
UNARY = {"silu": 0, "gelu": 1, "gelu_tanh": 2, "neg": 3, "exp": 4, "sigmoid": 5, "relu": 6, "quick_gelu": 7}
BINARY = {"add": 0, "sub": 1, "mul": 2, "div": 3}
EPI_NONE, EPI_GELU, EPI_SILU, EPI_GEGLU, EPI_QUICK_GELU = range(5)
SDPA_PATH_TC_LAZY, SDPA_PATH_TC, SDPA_PATH_SIMT, SDPA_PATH_TC_SHORT = 1, 2, 3, 4

I64 = C.c_int64
I64_4 = I64 * 4
VP = C.c_void_p


class GemmDesc(C.Structure):
    _fields_ = [
        ("M", I64), ("N", I64), ("K", I64), ("batch", I64),
        ("dtype", C.c_int), ("out_dtype", C.c_int),
        ("A", VP), ("lda", I64), ("stride_a", I64), ("a_trans", C.c_int),
        ("B", VP), ("ldb", I64), ("stride_b", I64), ("b_trans", C.c_int),
        ("D", VP), ("ldd", I64), ("stride_d", I64),
        ("C", VP), ("ldc", I64), ("stride_c", I64),
        ("bias", VP), ("bias_dtype", C.c_int), ("bias_batch_stride", I64),
        ("residual", VP), ("ldr", I64), ("stride_r", I64),
        ("alpha", C.c_float), ("beta", C.c_float),
        ("epilogue", C.c_int),
        ("A_lo", VP), ("B_lo", VP),
    ]


class Conv2dDesc(C.Structure):
    _fields_ = [
        ("N", I64), ("C", I64), ("H", I64), ("W", I64), ("K", I64), ("R", I64), ("S", I64), ("P", I64), ("Q", I64),
        ("stride_h", C.c_int), ("stride_w", C.c_int), ("pad_h", C.c_int), ("pad_w", C.c_int),
        ("dil_h", C.c_int), ("dil_w", C.c_int), ("groups", C.c_int),
        ("dtype", C.c_int), ("out_dtype", C.c_int),
        ("x", VP), ("x_strides", I64_4),
        ("w", VP),
        ("w_packed", C.c_int), ("w_lo", VP),
        ("bias", VP), ("bias_dtype", C.c_int), ("bias_batch_stride", I64),
        ("residual", VP), ("res_strides", I64_4),
        ("y", VP), ("y_strides", I64_4),
        ("epilogue", C.c_int),
    ]


class SdpaDesc(C.Structure):
    _fields_ = [
        ("B", I64), ("H", I64), ("Hkv", I64), ("Sq", I64), ("Sk", I64), ("D", I64), ("Dv", I64),
        ("dtype", C.c_int),
        ("q", VP), ("q_strides", I64_4),
        ("k", VP), ("k_strides", I64_4),
        ("v", VP), ("v_strides", I64_4),
        ("o", VP), ("o_strides", I64_4),
        ("mask", VP), ("mask_kind", C.c_int), ("mask_dtype", C.c_int), ("mask_strides", I64_4),
        ("causal", C.c_int),
        ("scale", C.c_double),
    ]


class RngState(C.Structure):
    _fields_ = [("state", C.c_uint64), ("has_spare", C.c_int32), ("spare", C.c_double)]


# (name, restype, argtypes) for every symbol the header declares.
_P64 = C.POINTER(I64)
SIGNATURES = {
    "mt_cuda_last_error_string": (C.c_char_p, []),
    "mt_cuda_device_count": (C.c_int, []),
    "mt_cuda_set_device": (C.c_int, [C.c_int]),
    "mt_cuda_synchronize": (C.c_int, [VP]),
    "mt_cuda_device_status": (C.c_int, [C.c_int]),
    "mt_cuda_selftest_wait_timeout": (C.c_int, [C.c_longlong, VP]),
    "mt_cuda_launch_count": (C.c_uint64, []),
    "mt_cuda_memcpy":(C.c_int, [VP, VP, C.c_size_t, C.c_int, VP]),
    "mt_cuda_memset": (C.c_int, [VP, C.c_int, C.c_size_t, VP]),
    "mt_cuda_malloc": (C.c_int, [C.POINTER(VP), C.c_size_t]),
    "mt_cuda_free": (C.c_int, [VP]),
    "mt_cuda_memory_stats": (C.c_int, [C.c_int, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "mt_cuda_empty_cache": (C.c_int, []),
    "mt_cuda_host_alloc": (C.c_int, [C.POINTER(VP), C.c_size_t]),
    "mt_cuda_host_free": (C.c_int, [VP]),
    "mt_cuda_stream_create": (C.c_int, [C.POINTER(VP)]),
    "mt_cuda_stream_destroy": (C.c_int, [VP]),
    "mt_cuda_library_stream": (C.c_int, [C.c_int, C.POINTER(VP)]),
    "mt_cuda_event_create": (C.c_int, [C.POINTER(VP)]),
    "mt_cuda_event_destroy": (C.c_int, [VP]),
    "mt_cuda_event_record": (C.c_int, [VP, VP]),
    "mt_cuda_event_synchronize": (C.c_int, [VP]),
    "mt_cuda_event_elapsed_ms": (C.c_int, [VP, VP, C.POINTER(C.c_float)]),
    "mt_cuda_graph_begin": (C.c_int, [VP]),
    "mt_cuda_graph_end": (C.c_int, [VP, C.POINTER(VP)]),
    "mt_cuda_graph_launch": (C.c_int, [VP, VP]),
    "mt_cuda_graph_destroy": (C.c_int, [VP]),
    "mt_nccl_available": (C.c_int, []),
    "mt_nccl_unique_id": (C.c_int, [VP, C.c_size_t]),
    "mt_nccl_comm_init": (C.c_int, [C.POINTER(VP), VP, C.c_size_t, C.c_int, C.c_int]),
    "mt_nccl_all_gather": (C.c_int, [VP, VP, C.c_size_t, VP, VP]),
    "mt_nccl_comm_destroy": (C.c_int, [VP]),
    "mt_cuda_copy_strided": (C.c_int, [VP, C.c_int, _P64, VP, C.c_int, _P64, _P64, C.c_int, VP]),
    "mt_cuda_fill_uniform": (C.c_int, [VP, C.c_int, I64, C.c_uint64, C.c_double, C.c_double, VP]),
    "mt_cuda_fill": (C.c_int, [VP, C.c_int, I64, C.c_double, VP]),
    "mt_cuda_unary": (C.c_int, [C.c_int, VP, C.c_int, VP, C.c_int, I64, VP]),
    "mt_cuda_binary": (C.c_int, [C.c_int, VP, C.c_int, _P64, VP, C.c_int, _P64, VP, C.c_int, _P64, C.c_double,
                                 _P64, C.c_int, VP]),
    "mt_cuda_axpby": (C.c_int, [VP, C.c_int, VP, C.c_int, C.c_double, VP, C.c_int, C.c_double, VP, C.c_int,
                                C.c_double, I64, VP]),
    "mt_cuda_ddim_step": (C.c_int, [VP, VP, VP, C.c_int, C.c_int, I64, C.c_double, C.c_double, C.c_int, VP]),
    "mt_cuda_ddim_step_indexed": (C.c_int, [VP, I64, VP, VP, C.c_int, C.c_int, I64, VP, I64, VP, I64, C.c_int,
                                            C.c_double, C.c_int, VP]),
    "mt_cuda_timestep_embedding": (C.c_int, [VP, C.c_int, VP, C.c_int, I64, I64, I64, C.c_double, C.c_int, VP]),
    "mt_cuda_embedding": (C.c_int, [VP, C.c_int, VP, C.c_int, I64, I64, VP, I64, VP, C.c_int, I64, VP, VP, VP]),
    "mt_cuda_softmax":(C.c_int, [VP, C.c_int, VP, C.c_int, I64, I64, I64, C.c_int, VP]),
    "mt_cuda_layer_norm": (C.c_int, [VP, C.c_int, VP, C.c_int, VP, VP, C.c_int, I64, I64, C.c_double, VP]),
    "mt_cuda_group_norm_workspace_size": (C.c_size_t, [I64, I64, I64, I64]),
    "mt_cuda_group_norm_cat": (C.c_int, [VP, C.c_int, _P64, VP, _P64, I64, VP, _P64, C.c_int, VP, VP, C.c_int, I64,
                                         I64, I64, I64, C.c_double, C.c_int, VP, C.c_size_t, VP]),
    "mt_cuda_group_norm": (C.c_int, [VP, C.c_int, _P64, VP, C.c_int, _P64, VP, VP, C.c_int, I64, I64, I64, I64,
                                     C.c_double, C.c_int, VP, C.c_size_t, VP]),
    "mt_cuda_group_norm_noalloc": (C.c_int, [VP, C.c_int, _P64, VP, C.c_int, _P64, VP, VP, C.c_int, I64, I64, I64,
                                             I64, C.c_double, C.c_int, VP]),
    "mt_cuda_gemm_workspace_size":(C.c_size_t, [C.POINTER(GemmDesc)]),
    "mt_cuda_gemm": (C.c_int, [C.POINTER(GemmDesc), VP, C.c_size_t, VP]),
    "mt_cuda_conv2d_workspace_size": (C.c_size_t, [C.POINTER(Conv2dDesc)]),
    "mt_cuda_conv2d": (C.c_int, [C.POINTER(Conv2dDesc), VP, C.c_size_t, VP]),
    "mt_cuda_conv2d_cat_workspace_size": (C.c_size_t, [C.POINTER(Conv2dDesc), VP, _P64, I64]),
    "mt_cuda_conv2d_cat": (C.c_int, [C.POINTER(Conv2dDesc), VP, _P64, I64, VP, C.c_size_t, VP]),
    "mt_cuda_conv2d_packed_channels": (I64, [I64, I64, I64, C.c_int]),
    "mt_cuda_conv2d_pack_weight": (C.c_int, [VP, VP, VP, C.c_int, I64, I64, I64, I64, VP]),
    "mt_cuda_conv2d_up2x_workspace_size": (C.c_size_t, [C.POINTER(Conv2dDesc)]),
    "mt_cuda_conv2d_up2x": (C.c_int, [C.POINTER(Conv2dDesc), VP, C.c_size_t, VP]),
    "mt_cuda_conv2d_up2x_packed_elems": (I64, [I64, I64, C.c_int]),
    "mt_cuda_conv2d_up2x_pack_weight": (C.c_int, [VP, VP, VP, C.c_int, I64, I64, VP]),
    "mt_cuda_sdpa_workspace_size": (C.c_size_t, [C.POINTER(SdpaDesc)]),
    "mt_cuda_sdpa": (C.c_int, [C.POINTER(SdpaDesc), VP, C.c_size_t, VP]),
    "mt_cuda_sdpa_path": (C.c_int, [C.POINTER(SdpaDesc)]),
    "mt_rng_seed": (None, [C.POINTER(RngState), C.c_uint64]),
    "mt_rng_fill_normal": (None, [C.POINTER(RngState), VP, C.c_int, I64, C.c_double, C.c_double]),
    "mt_rng_fill_uniform": (None, [C.POINTER(RngState), VP, C.c_int, I64, C.c_double, C.c_double]),
}

_LIB = None


class CudaError(RuntimeError):
    pass


def lib():
    """The loaded kernel library; raises if it has not been built (no fallback exists)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"mtorch_b200 kernel library not built ({LIB_PATH}); run `python mtorch_b200/build.py` "
                "or __graft_entry__.build()")
        L = C.CDLL(os.fspath(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def check(rc: int, what: str = "") -> None:
    if rc != MT_OK:
        msg = lib().mt_cuda_last_error_string().decode(errors="replace")
        if rc == MT_ERR_UNSUPPORTED:
            raise NotImplementedError(f"{what}: {msg}")
        if rc == MT_ERR_INVALID:
            raise ValueError(f"{what}: {msg}")
        raise CudaError(f"{what}: {msg} (status {rc})")


def arr64(values) -> C.Array:
    vals = list(values)
    return (I64 * max(1, len(vals)))(*vals)
