"""Device op functions: the `cuda` branch of the reference's hot-path ops.

Each function validates arguments the way the reference does (same error types), computes
strides / broadcast metadata on the host and calls exactly one C-ABI entry point of
``libmtorch_cuda.so`` (plus metadata-only views).  CPU tensors raise NotImplementedError:
compute on the host is mtorch's own CPU backend, never a silent fallback here.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib as L
from .tensor import (Tensor, _new, _require_cuda, _broadcast_shape, bfloat16, float16, float32, float64, int32, int64,
                     tensor, to_dtype, workspace, zeros, _contig_strides)


def _lib():
    return L.lib()


def _same_dtype(*ts, what):
    d = ts[0].dtype
    for t in ts[1:]:
        if t is not None and t.dtype is not d:
            raise RuntimeError(f"{what}: expected all tensors to have the same dtype, got {d.name} and {t.dtype.name}")
    if not d.is_floating_point or d.name == "float64":
        raise NotImplementedError(f"{what}: dtype {d.name} is not supported on the cuda device")


# ---------------------------------------------------------------------------------------------
# GEMM family: matmul / bmm / addmm / baddbmm / linear (tensor.cpp:24896-25694, 31401-31694)


def _mat_layout(t: Tensor):
    """(ptr-owner tensor, leading dim, trans) for a 2-D [R, C] view, copying if neither axis is
    unit-stride."""
    sr, sc = t._strides[-2], t._strides[-1]
    R, Cc = t._shape[-2], t._shape[-1]
    if sc == 1 or Cc == 1:
        return t, max(sr, Cc) if R > 1 else max(Cc, 1), 0
    if sr == 1 or R == 1:
        return t, max(sc, R), 1
    t = t.contiguous()
    return t, Cc, 0


def gemm(a: Tensor, b: Tensor, *, out: Tensor | None = None, bias: Tensor | None = None, bias_batch_stride=0,
         residual: Tensor | None = None, C_in: Tensor | None = None, alpha=1.0, beta=0.0, epilogue=L.EPI_NONE,
         out_dtype=None, a_lo=None, b_lo=None) -> Tensor:
    """Batched D = alpha * a @ b + beta * C_in + bias (act) + residual.  a: [batch?, M, K],
    b: [batch?, K, N] (either may be 2-D and is then broadcast); all on one cuda device."""
    _require_cuda(a, b)
    batch = max(a._shape[0] if a.dim() == 3 else 1, b._shape[0] if b.dim() == 3 else 1)
    M, K = a._shape[-2], a._shape[-1]
    K2, N = b._shape[-2], b._shape[-1]
    if K != K2:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({M}x{K} and {K2}x{N})")
    odt = out_dtype or a.dtype
    n_out = N // 2 if epilogue == L.EPI_GEGLU else N
    if out is None:
        out = _new((batch, M, n_out) if (a.dim() == 3 or b.dim() == 3) else (M, n_out), odt, a.device)
    if K == 0:
        out.zero_()
        if bias is not None:
            out.add_(bias)
        return out
    a_t, lda, at = _mat_layout(a)
    b_t, ldb, bt_stored = _mat_layout(b)
    # _mat_layout's trans flag: 0 = [rows, cols] row-major.  For B, [K, N] row-major is b_trans=0;
    # unit stride along K ([N, K] storage) is b_trans=1.
    d = L.GemmDesc()
    d.M, d.N, d.K, d.batch = M, N, K, batch
    d.dtype, d.out_dtype = a.dtype.code, odt.code
    d.A, d.lda, d.stride_a, d.a_trans = a_t.data_ptr(), lda, (a_t._strides[0] if a_t.dim() == 3 and a_t._shape[0] > 1 else 0), at
    d.B, d.ldb, d.stride_b, d.b_trans = b_t.data_ptr(), ldb, (b_t._strides[0] if b_t.dim() == 3 and b_t._shape[0] > 1 else 0), bt_stored
    d.D, d.ldd = out.data_ptr(), out._strides[-2]
    d.stride_d = out._strides[0] if out.dim() == 3 else 0
    if C_in is not None and beta != 0.0:
        Ce = C_in.expand(out.shape) if C_in.dim() <= out.dim() else C_in
        if Ce._strides[-1] != 1:
            Ce = Ce.contiguous()
        d.C, d.ldc, d.stride_c = Ce.data_ptr(), Ce._strides[-2], (Ce._strides[0] if Ce.dim() == 3 else 0)
    if bias is not None:
        bias = bias if bias._strides[-1] == 1 else bias.contiguous()
        d.bias, d.bias_dtype, d.bias_batch_stride = bias.data_ptr(), bias.dtype.code, bias_batch_stride
    if residual is not None:
        r = residual if residual._strides[-1] == 1 else residual.contiguous()
        d.residual, d.ldr, d.stride_r = r.data_ptr(), r._strides[-2], (r._strides[0] if r.dim() == 3 else 0)
    d.alpha, d.beta, d.epilogue = float(alpha), float(beta), int(epilogue)
    if a_lo is not None:
        d.A_lo = a_lo.data_ptr()
    if b_lo is not None:
        d.B_lo = b_lo.data_ptr()
    lib = _lib()
    need = lib.mt_cuda_gemm_workspace_size(C.byref(d))
    ws, wsb = workspace(need, a._idx())
    L.check(lib.mt_cuda_gemm(C.byref(d), ws, wsb, a._stream()), "gemm")
    out._mark_modified()
    return out


def matmul(a: Tensor, b: Tensor) -> Tensor:
    """`matmul` (tensor.cpp:24896-25064): dot / mv / vm / mm / broadcast batched mm."""
    _require_cuda(a, b)
    _same_dtype(a, b, what="matmul")
    if a.dim() == 0 or b.dim() == 0:
        raise RuntimeError("both arguments to matmul need to be at least 1D")
    squeeze_m = a.dim() == 1
    squeeze_n = b.dim() == 1
    if squeeze_m:
        a = a.unsqueeze(0)
    if squeeze_n:
        b = b.unsqueeze(-1)
    batch_shape = _broadcast_shape(a._shape[:-2], b._shape[:-2])
    M, K, N = a._shape[-2], a._shape[-1], b._shape[-1]
    if not batch_shape:
        out = gemm(a, b)
    elif b.dim() == 2 and a.is_contiguous():
        # fold the batch into M (one large GEMM)
        out = gemm(a.reshape(-1, K), b).reshape(batch_shape + (M, N))
    else:
        nb = math.prod(batch_shape)
        a3 = _fold_batch(a, batch_shape)
        b3 = _fold_batch(b, batch_shape)
        out = gemm(a3, b3).reshape(batch_shape + (M, N))
    if squeeze_n:
        out = out.squeeze(-1)
    if squeeze_m:
        out = out.squeeze(-2)
    return out


def _fold_batch(t: Tensor, batch_shape) -> Tensor:
    """[*batch, R, C] (broadcast to batch_shape) -> [nb, R, C] with one batch stride (0 if the
    tensor is broadcast over the whole batch)."""
    R, Cc = t._shape[-2], t._shape[-1]
    nb = math.prod(batch_shape)
    if t.dim() == 2 or all(s == 1 for s in t._shape[:-2]):
        t2 = t.reshape(R, Cc) if t.dim() > 2 else t
        return t2._view((nb, R, Cc), (0,) + t2._strides)
    e = t.expand(tuple(batch_shape) + (R, Cc))
    # collapsible batch dims?
    bs = e._strides[:-2]
    ok = all(bs[i] == bs[i + 1] * batch_shape[i + 1] for i in range(len(bs) - 1)) and 0 not in bs
    if ok:
        return e._view((nb, R, Cc), (bs[-1],) + e._strides[-2:])
    return e.contiguous().reshape(nb, R, Cc)


def mm(a, b):
    if a.dim() != 2 or b.dim() != 2:
        raise RuntimeError("mm: expected 2D tensors")
    return matmul(a, b)


def bmm(a: Tensor, b: Tensor) -> Tensor:
    """`bmm` (tensor.cpp:25066-25182)."""
    if a.dim() != 3 or b.dim() != 3:
        raise RuntimeError("batch1 and batch2 must be 3D tensors")
    if a._shape[0] != b._shape[0]:
        raise RuntimeError("batch1 and batch2 must have same number of batches")
    _require_cuda(a, b)
    _same_dtype(a, b, what="bmm")
    return gemm(a, b)


def addmm(inp: Tensor, m1: Tensor, m2: Tensor, beta=1.0, alpha=1.0) -> Tensor:
    """`addmm` (tensor.cpp:25184-25366): beta * input + alpha * (m1 @ m2)."""
    _require_cuda(inp, m1, m2)
    _same_dtype(m1, m2, inp, what="addmm")
    M, N = m1._shape[0], m2._shape[1]
    return gemm(m1, m2, C_in=inp.expand((M, N)), alpha=alpha, beta=beta)


def baddbmm(inp: Tensor, b1: Tensor, b2: Tensor, beta=1.0, alpha=1.0) -> Tensor:
    """`baddbmm` (tensor.cpp:25557-25694)."""
    _require_cuda(inp, b1, b2)
    _same_dtype(b1, b2, inp, what="baddbmm")
    shape = (b1._shape[0], b1._shape[1], b2._shape[2])
    return gemm(b1, b2, C_in=inp.expand(shape), alpha=alpha, beta=beta)


def linear(x: Tensor, w: Tensor, bias: Tensor | None = None, *, epilogue=L.EPI_NONE, residual=None,
           w_lo=None) -> Tensor:
    """`linear` (tensor.cpp:31401-31694): y = x @ w^T + bias over any leading dims."""
    _require_cuda(x, w, bias)
    _same_dtype(x, w, what="linear")
    K = x._shape[-1]
    if w._shape[-1] != K:
        raise RuntimeError(f"mat1 and mat2 shapes cannot be multiplied ({math.prod(x._shape[:-1])}x{K} and "
                           f"{w._shape[1]}x{w._shape[0]})")
    lead = x._shape[:-1]
    x2 = x.reshape(-1, K) if x.dim() != 2 else x
    wt = w.transpose(0, 1)  # [K, N] view over [N, K] storage: unit stride along K -> b_trans
    res2 = residual.reshape(-1, residual._shape[-1]) if residual is not None else None
    y = gemm(x2, wt, bias=bias, residual=res2, epilogue=epilogue, b_lo=w_lo)
    return y.reshape(lead + (y._shape[-1],))


# ---------------------------------------------------------------------------------------------
# conv2d (tensor.cpp:26490-27528)


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def conv2d(x: Tensor, w: Tensor, bias: Tensor | None = None, stride=1, padding=0, dilation=1, groups=1, *,
           residual: Tensor | None = None, bias_batch_stride=0, packed=None, epilogue=L.EPI_NONE,
           out_channels_last=None) -> Tensor:
    _require_cuda(x, w, bias, residual)
    _same_dtype(x, w, what="conv2d")
    unbatched = x.dim() == 3
    if unbatched:
        x = x.unsqueeze(0)
    if x.dim() != 4 or w.dim() != 4:
        raise RuntimeError("conv2d: expected 3D (unbatched) or 4D (batched) input and 4D weight")
    N, Cin, H, W = x._shape
    K, Cg, R, S = w._shape
    if Cg * groups != Cin:
        raise RuntimeError(f"Given groups={groups}, weight of size {tuple(w._shape)}, expected input{tuple(x._shape)} "
                           f"to have {Cg * groups} channels, but got {Cin} channels instead")
    sh, sw = _pair(stride)
    dh, dw = _pair(dilation)
    if isinstance(padding, str):
        if padding == "valid":
            ph = pw = 0
        elif padding == "same":
            if (sh, sw) != (1, 1):
                raise ValueError("padding='same' is not supported for strided convolutions")
            ph, pw = dh * (R - 1) // 2, dw * (S - 1) // 2
            if (dh * (R - 1)) % 2 or (dw * (S - 1)) % 2:
                raise NotImplementedError("asymmetric 'same' padding is not supported on the cuda device")
        else:
            raise ValueError(f"Invalid padding string '{padding}'")
    else:
        ph, pw = _pair(padding)
    P = (H + 2 * ph - dh * (R - 1) - 1) // sh + 1
    Q = (W + 2 * pw - dw * (S - 1) - 1) // sw + 1
    if P <= 0 or Q <= 0:
        raise RuntimeError("conv2d: output size is too small")
    cl = x.is_contiguous("channels_last") and not x.is_contiguous() if out_channels_last is None else out_channels_last
    y = _new((N, K, P, Q), x.dtype, x.device, channels_last=cl)
    d = L.Conv2dDesc()
    d.N, d.C, d.H, d.W, d.K, d.R, d.S, d.P, d.Q = N, Cin, H, W, K, R, S, P, Q
    d.stride_h, d.stride_w, d.pad_h, d.pad_w, d.dil_h, d.dil_w, d.groups = sh, sw, ph, pw, dh, dw, groups
    d.dtype = d.out_dtype = x.dtype.code
    d.x = x.data_ptr()
    d.x_strides[:] = list(x._strides)
    if packed is not None:
        d.w, d.w_packed = packed[0].data_ptr(), 1
        d.w_lo = packed[1].data_ptr() if packed[1] is not None else None
    else:
        wc = w.contiguous()
        d.w, d.w_packed = wc.data_ptr(), 0
    if bias is not None:
        bias = bias.contiguous()
        d.bias, d.bias_dtype, d.bias_batch_stride = bias.data_ptr(), bias.dtype.code, bias_batch_stride
    if residual is not None:
        d.residual = residual.data_ptr()
        d.res_strides[:] = list(residual.expand(y.shape)._strides)
    d.y = y.data_ptr()
    d.y_strides[:] = list(y._strides)
    d.epilogue = int(epilogue)
    lib = _lib()
    need = lib.mt_cuda_conv2d_workspace_size(C.byref(d))
    ws, wsb = workspace(need, x._idx())
    L.check(lib.mt_cuda_conv2d(C.byref(d), ws, wsb, x._stream()), "conv2d")
    return y.squeeze(0) if unbatched else y


def cat_fusable(a: Tensor, b: Tensor) -> bool:
    """Whether `group_norm_cat` / `conv2d_cat` read the channel concatenation [a | b] in place: bf16
    cuda tensors [N, C, H, W] of equal N, H, W, dense channels-last, channel counts multiples of 64."""
    return (a.device.type == "cuda" and b.device.type == "cuda" and a.dim() == 4 and b.dim() == 4 and
            a.dtype is bfloat16 and b.dtype is bfloat16 and a._shape[0] == b._shape[0] and
            a._shape[2:] == b._shape[2:] and a._shape[1] % 64 == 0 and b._shape[1] % 64 == 0 and
            a.is_contiguous("channels_last") and b.is_contiguous("channels_last"))


def group_norm_cat(a: Tensor, b: Tensor, num_groups: int, weight=None, bias=None, eps=1e-5, *,
                   fuse_silu=False) -> Tensor:
    """group_norm(cat([a, b], dim=1)) without forming the concatenation (bit-identical to it);
    inputs as `cat_fusable` describes, output channels-last."""
    _require_cuda(a, b, weight, bias)
    if not cat_fusable(a, b):
        raise NotImplementedError("group_norm_cat: inputs must satisfy cat_fusable")
    N, C1 = a._shape[0], a._shape[1]
    Cc = C1 + b._shape[1]
    if Cc % num_groups:
        raise RuntimeError(f"Expected number of channels in input to be divisible by num_groups, but got {Cc} "
                           f"channels and num_groups={num_groups}")
    HW = a._shape[2] * a._shape[3]
    out = _new((N, Cc) + a._shape[2:], a.dtype, a.device, channels_last=True)
    wbd = (weight if weight is not None else bias).dtype.code if (weight is not None or bias is not None) else L.MT_F32
    lib = _lib()
    need = lib.mt_cuda_group_norm_workspace_size(N, Cc, HW, num_groups)
    ws, wsb = workspace(need, a._idx())
    L.check(lib.mt_cuda_group_norm_cat(out.data_ptr(), out.dtype.code, L.arr64(_nchw_view_strides(out)), a.data_ptr(),
                                       L.arr64(_nchw_view_strides(a)), C1, b.data_ptr(),
                                       L.arr64(_nchw_view_strides(b)), a.dtype.code,
                                       weight.data_ptr() if weight is not None else None,
                                       bias.data_ptr() if bias is not None else None, wbd, N, Cc, HW, num_groups,
                                       float(eps), 1 if fuse_silu else 0, ws, wsb, a._stream()), "group_norm_cat")
    return out


def conv2d_cat(a: Tensor, b: Tensor, w: Tensor, bias: Tensor | None = None, stride=1, padding=0, *,
               residual: Tensor | None = None, packed=None) -> Tensor:
    """conv2d(cat([a, b], dim=1), w, bias, stride, padding) without forming the concatenation
    (bit-identical to it); inputs as `cat_fusable` describes, output channels-last."""
    _require_cuda(a, b, w, bias, residual)
    _same_dtype(a, b, w, what="conv2d_cat")
    if not cat_fusable(a, b):
        raise NotImplementedError("conv2d_cat: inputs must satisfy cat_fusable")
    N, C1, H, W = a._shape
    Cin = C1 + b._shape[1]
    K, Cg, R, S = w._shape
    if Cg != Cin:
        raise RuntimeError(f"conv2d_cat: weight of size {tuple(w._shape)} expects {Cg} input channels, got {Cin}")
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    P = (H + 2 * ph - (R - 1) - 1) // sh + 1
    Q = (W + 2 * pw - (S - 1) - 1) // sw + 1
    y = _new((N, K, P, Q), a.dtype, a.device, channels_last=True)
    d = L.Conv2dDesc()
    d.N, d.C, d.H, d.W, d.K, d.R, d.S, d.P, d.Q = N, Cin, H, W, K, R, S, P, Q
    d.stride_h, d.stride_w, d.pad_h, d.pad_w, d.dil_h, d.dil_w, d.groups = sh, sw, ph, pw, 1, 1, 1
    d.dtype = d.out_dtype = a.dtype.code
    d.x = a.data_ptr()
    d.x_strides[:] = list(a._strides)
    if packed is not None:
        d.w, d.w_packed = packed[0].data_ptr(), 1
    else:
        wc = w.contiguous()
        d.w, d.w_packed = wc.data_ptr(), 0
    if bias is not None:
        bias = bias.contiguous()
        d.bias, d.bias_dtype = bias.data_ptr(), bias.dtype.code
    if residual is not None:
        d.residual = residual.data_ptr()
        d.res_strides[:] = list(residual.expand(y.shape)._strides)
    d.y = y.data_ptr()
    d.y_strides[:] = list(y._strides)
    lib = _lib()
    bst = L.arr64(list(b._strides))
    need = lib.mt_cuda_conv2d_cat_workspace_size(C.byref(d), b.data_ptr(), bst, C1)
    ws, wsb = workspace(need, a._idx())
    L.check(lib.mt_cuda_conv2d_cat(C.byref(d), b.data_ptr(), bst, C1, ws, wsb, a._stream()), "conv2d_cat")
    return y


def pack_conv_weight(w: Tensor):
    """[K, C, R, S] -> ([K, R, S, Cp] packed, tf32 low part or None) for the implicit-GEMM path."""
    _require_cuda(w)
    K, Cin, R, S = w._shape
    Cp = _lib().mt_cuda_conv2d_packed_channels(Cin, R, S, w.dtype.code)
    wp = _new((K, R * S * Cp), w.dtype, w.device)
    lo = _new((K, R * S * Cp), float32, w.device) if w.dtype is float32 else None
    wc = w.contiguous()
    L.check(_lib().mt_cuda_conv2d_pack_weight(wp.data_ptr(), lo.data_ptr() if lo is not None else None,
                                              wc.data_ptr(), w.dtype.code, K, Cin, R, S, w._stream()), "pack weight")
    return wp, lo


def conv2d_up2x_supported(x: Tensor, w: Tensor) -> bool:
    """Whether `conv2d_up2x` takes this input: a 3x3 weight and channels filling whole 128-byte
    chunks (64 for bf16/f16, 32 for fp32)."""
    per = 128 // x.dtype.itemsize
    return (x.dim() == 4 and w.dim() == 4 and tuple(w._shape[2:]) == (3, 3) and x._shape[1] % per == 0
            and x.dtype is w.dtype)


def conv2d_up2x(x: Tensor, w: Tensor, bias: Tensor | None = None, *, packed=None) -> Tensor:
    """conv2d(interpolate(x, scale_factor=2, mode="nearest"), w, bias, stride=1, padding=1) for a
    3x3 weight, without forming the upsampled tensor (the SD UNet up-block pair,
    tensor.cpp:10897 + 26490-27528): four 2x2 convolutions of the source, one per output parity,
    with the 3x3 taps summed per parity.  Output [N, K, 2H, 2W] channels-last.  `packed`: the
    result of `pack_conv_up2x_weight(w)`."""
    _require_cuda(x, w, bias)
    _same_dtype(x, w, what="conv2d")
    if not conv2d_up2x_supported(x, w):
        raise NotImplementedError("conv2d_up2x: needs a 3x3 weight and channels filling 128-byte chunks")
    N, Cin, H, W = x._shape
    K = w._shape[0]
    if w._shape[1] != Cin:
        raise RuntimeError(f"conv2d_up2x: weight expects {w._shape[1]} input channels, got {Cin}")
    y = _new((N, K, 2 * H, 2 * W), x.dtype, x.device, channels_last=True)
    d = L.Conv2dDesc()
    d.N, d.C, d.H, d.W, d.K, d.R, d.S, d.P, d.Q = N, Cin, H, W, K, 3, 3, 2 * H, 2 * W
    d.stride_h, d.stride_w, d.pad_h, d.pad_w, d.dil_h, d.dil_w, d.groups = 1, 1, 1, 1, 1, 1, 1
    d.dtype = d.out_dtype = x.dtype.code
    d.x = x.data_ptr()
    d.x_strides[:] = list(x._strides)
    if packed is not None:
        d.w, d.w_packed = packed[0].data_ptr(), 1
        d.w_lo = packed[1].data_ptr() if packed[1] is not None else None
    else:
        wc = w.contiguous()
        d.w, d.w_packed = wc.data_ptr(), 0
    if bias is not None:
        bias = bias.contiguous()
        d.bias, d.bias_dtype, d.bias_batch_stride = bias.data_ptr(), bias.dtype.code, 0
    d.y = y.data_ptr()
    d.y_strides[:] = list(y._strides)
    d.epilogue = int(L.EPI_NONE)
    lib = _lib()
    need = lib.mt_cuda_conv2d_up2x_workspace_size(C.byref(d))
    ws, wsb = workspace(need, x._idx())
    L.check(lib.mt_cuda_conv2d_up2x(C.byref(d), ws, wsb, x._stream()), "conv2d_up2x")
    return y


def pack_conv_up2x_weight(w: Tensor):
    """[K, C, 3, 3] -> (per-parity 2x2 weights [4, K, 2, 2, Cp], tf32 low part or None)."""
    _require_cuda(w)
    K, Cin = w._shape[0], w._shape[1]
    n = _lib().mt_cuda_conv2d_up2x_packed_elems(K, Cin, w.dtype.code)
    wp = _new((n,), w.dtype, w.device)
    lo = _new((n,), float32, w.device) if w.dtype is float32 else None
    wc = w.contiguous()
    L.check(_lib().mt_cuda_conv2d_up2x_pack_weight(wp.data_ptr(), lo.data_ptr() if lo is not None else None,
                                                   wc.data_ptr(), w.dtype.code, K, Cin, w._stream()),
            "pack up2x weight")
    return wp, lo


# ---------------------------------------------------------------------------------------------
# attention (tensor.cpp:30930-31324)


def _sdpa_desc(q, k, v, out, attn_mask, is_causal, scale, enable_gqa):
    """The mt_sdpa_desc of an SDPA call (shapes already checked by the caller)."""
    lead = q._shape[:-2]
    Lq, E = q._shape[-2], q._shape[-1]
    Sk, Ev = k._shape[-2], v._shape[-1]

    def as4(t):
        if t.dim() == 4:
            return t
        if t.dim() == 2:
            return t._view((1, 1) + t._shape, (0, 0) + t._strides)
        if t.dim() == 3:
            return t._view((t._shape[0], 1) + t._shape[1:], (t._strides[0], 0) + t._strides[1:])
        # fold extra leading dims
        return t.reshape((-1, t._shape[-3]) + t._shape[-2:])

    q4, k4, v4, o4 = as4(q), as4(k), as4(v), as4(out)
    B, H = q4._shape[0], q4._shape[1]
    Hkv = k4._shape[1]
    if k4._shape[0] != B and k4._shape[0] == 1:
        k4 = k4.expand((B,) + k4._shape[1:])
        v4 = v4.expand((B,) + v4._shape[1:])
    if Hkv != H:
        if not enable_gqa and Hkv != 1:
            raise ValueError("scaled_dot_product_attention key/value heads must match query heads unless enable_gqa")
        if H % Hkv:
            raise ValueError("number of heads in key/value must divide number of heads in query")
    d = L.SdpaDesc()
    d.B, d.H, d.Hkv, d.Sq, d.Sk, d.D, d.Dv = B, H, Hkv, Lq, Sk, E, Ev
    d.dtype = q.dtype.code
    d.q, d.k, d.v, d.o = q4.data_ptr(), k4.data_ptr(), v4.data_ptr(), o4.data_ptr()
    d.q_strides[:], d.k_strides[:], d.v_strides[:], d.o_strides[:] = (list(q4._strides), list(k4._strides),
                                                                      list(v4._strides), list(o4._strides))
    if attn_mask is not None:
        m = attn_mask
        if m.dtype.name == "bool":
            d.mask_kind = 1
        else:
            d.mask_kind = 2
            d.mask_dtype = m.dtype.code
        me = m.expand(_broadcast_shape(m._shape, (B, H, Lq, Sk)))
        if me.dim() != 4:
            me = me.reshape(B, H, Lq, Sk)
        d.mask = me.data_ptr()
        d.mask_strides[:] = list(me._strides)
    d.causal = 1 if is_causal else 0
    d.scale = float(scale) if scale is not None else 1.0 / math.sqrt(E)
    return d


def sdpa_path(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None = None, is_causal=False, scale=None,
              enable_gqa=False) -> str:
    """Which device kernel scaled_dot_product_attention runs for these arguments: "tc_lazy" (the
    tcgen05 kernel with the output in TMEM), "tc" (the general tcgen05 kernel), "tc_short" (the
    tcgen05 kernel for at most 128 keys) or "simt" (the fp32 SIMT kernel).  Nothing is launched."""
    _require_cuda(q, k, v, attn_mask)
    out = _new(q._shape[:-2] + (q._shape[-2], v._shape[-1]), q.dtype, q.device)
    d = _sdpa_desc(q, k, v, out, attn_mask, is_causal, scale, enable_gqa)
    code = _lib().mt_cuda_sdpa_path(C.byref(d))
    if code == 0:
        raise ValueError("sdpa_path: invalid arguments")
    return {L.SDPA_PATH_TC_LAZY: "tc_lazy", L.SDPA_PATH_TC: "tc", L.SDPA_PATH_SIMT: "simt",
            L.SDPA_PATH_TC_SHORT: "tc_short"}[code]


def scaled_dot_product_attention(q: Tensor, k: Tensor, v: Tensor, attn_mask: Tensor | None = None, dropout_p=0.0,
                                 is_causal=False, scale=None, enable_gqa=False, *, out: Tensor | None = None) -> Tensor:
    """`scaled_dot_product_attention` (tensor.cpp:30930-31324).  `out` (optional) may be any
    strided view of the right shape, e.g. a heads-merged [B, S, H, D] buffer seen as
    [B, H, S, D], so the next projection reads it without a copy."""
    _require_cuda(q, k, v, attn_mask)
    if q.dtype is not k.dtype or q.dtype is not v.dtype:
        raise ValueError("scaled_dot_product_attention query, key, and value must have the same dtype")
    if not (0.0 <= dropout_p <= 1.0):
        raise ValueError("scaled_dot_product_attention dropout_p must be between 0 and 1")
    if dropout_p not in (0.0, 1.0):
        raise ValueError("scaled_dot_product_attention dropout_p is only supported when it is 0 or 1")
    if q.dim() < 2:
        raise ValueError("scaled_dot_product_attention expects query with at least 2 dims")
    lead = q._shape[:-2]
    Lq, E = q._shape[-2], q._shape[-1]
    Sk, Ev = k._shape[-2], v._shape[-1]
    if out is None:
        out = _new(lead + (Lq, Ev), q.dtype, q.device)
    elif tuple(out.shape) != lead + (Lq, Ev):
        raise RuntimeError(f"sdpa: out has shape {tuple(out.shape)}, expected {lead + (Lq, Ev)}")
    if dropout_p == 1.0:
        return out.zero_()

    d = _sdpa_desc(q, k, v, out, attn_mask, is_causal, scale, enable_gqa)
    lib = _lib()
    need = lib.mt_cuda_sdpa_workspace_size(C.byref(d))
    ws, wsb = workspace(need, q._idx())
    L.check(lib.mt_cuda_sdpa(C.byref(d), ws, wsb, q._stream()), "scaled_dot_product_attention")
    return out


# ---------------------------------------------------------------------------------------------
# softmax / norms / activations


def softmax(x: Tensor, dim=-1, dtype=None) -> Tensor:
    """`softmax` (tensor.cpp:15145-15213)."""
    _require_cuda(x)
    odt = to_dtype(dtype) if dtype is not None else x.dtype
    dim = dim % x.dim()
    if dim != x.dim() - 1:
        perm = list(range(x.dim()))
        perm[dim], perm[-1] = perm[-1], perm[dim]
        return softmax(x.permute(perm), -1, dtype).permute(perm).contiguous()
    xc = x.contiguous()
    out = _new(x._shape, odt, x.device)
    cols = x._shape[-1] if x.dim() else 1
    rows = xc.numel() // max(cols, 1)
    L.check(_lib().mt_cuda_softmax(out.data_ptr(), odt.code, xc.data_ptr(), xc.dtype.code, rows, cols, cols, 0,
                                   x._stream()), "softmax")
    return out


def log_softmax(x: Tensor, dim=-1, dtype=None) -> Tensor:
    _require_cuda(x)
    odt = to_dtype(dtype) if dtype is not None else x.dtype
    dim = dim % x.dim()
    if dim != x.dim() - 1:
        perm = list(range(x.dim()))
        perm[dim], perm[-1] = perm[-1], perm[dim]
        return log_softmax(x.permute(perm), -1, dtype).permute(perm).contiguous()
    xc = x.contiguous()
    out = _new(x._shape, odt, x.device)
    cols = x._shape[-1]
    L.check(_lib().mt_cuda_softmax(out.data_ptr(), odt.code, xc.data_ptr(), xc.dtype.code, xc.numel() // cols, cols,
                                   cols, 1, x._stream()), "log_softmax")
    return out


def layer_norm(x: Tensor, normalized_shape, weight=None, bias=None, eps=1e-5) -> Tensor:
    """`layer_norm` (tensor.cpp:17386-17714)."""
    _require_cuda(x, weight, bias)
    ns = (normalized_shape,) if isinstance(normalized_shape, int) else tuple(normalized_shape)
    if tuple(x._shape[-len(ns):]) != ns:
        raise RuntimeError(f"Given normalized_shape={list(ns)}, expected input with shape [*, {', '.join(map(str, ns))}]")
    cols = math.prod(ns)
    xc = x.contiguous()
    out = _new(x._shape, x.dtype, x.device)
    wbd = (weight or bias).dtype.code if (weight is not None or bias is not None) else L.MT_F32
    wp = weight.contiguous().data_ptr() if weight is not None else None
    bp = bias.contiguous().data_ptr() if bias is not None else None
    L.check(_lib().mt_cuda_layer_norm(out.data_ptr(), out.dtype.code, xc.data_ptr(), xc.dtype.code, wp, bp, wbd,
                                      xc.numel() // max(cols, 1), cols, float(eps), x._stream()), "layer_norm")
    return out


def _nchw_view_strides(x: Tensor):
    """(sn, sc, shw) if the spatial dims of x collapse to one stride, else None."""
    sp_shape, sp_str = x._shape[2:], x._strides[2:]
    for i in range(len(sp_shape) - 1):
        if sp_shape[i + 1] != 1 and sp_str[i] != sp_str[i + 1] * sp_shape[i + 1]:
            return None
    shw = sp_str[-1] if sp_shape else 1
    return (x._strides[0], x._strides[1], shw)


def group_norm(x: Tensor, num_groups: int, weight=None, bias=None, eps=1e-5, *, fuse_silu=False) -> Tensor:
    """`group_norm` (tensor.cpp:18643-18963); `fuse_silu` adds the SD ResNet SiLU."""
    _require_cuda(x, weight, bias)
    if x.dim() < 2:
        raise RuntimeError("group_norm expects input with at least 2 dims")
    N, Cc = x._shape[0], x._shape[1]
    if Cc % num_groups:
        raise RuntimeError(f"Expected number of channels in input to be divisible by num_groups, but got input of "
                           f"shape {list(x._shape)} and num_groups={num_groups}")
    HW = math.prod(x._shape[2:])
    xs = _nchw_view_strides(x)
    if xs is None or not ((xs[1] == 1 and xs[2] == Cc) or (xs[2] == 1 and xs[1] == HW)):
        x = x.contiguous()
        xs = _nchw_view_strides(x)
    cl = x.dim() == 4 and x.is_contiguous("channels_last") and not x.is_contiguous()
    out = _new(x._shape, x.dtype, x.device, channels_last=cl)
    ys = _nchw_view_strides(out)
    wbd = (weight if weight is not None else bias).dtype.code if (weight is not None or bias is not None) else L.MT_F32
    lib = _lib()
    need = lib.mt_cuda_group_norm_workspace_size(N, Cc, HW, num_groups)
    ws, wsb = workspace(need, x._idx())
    L.check(lib.mt_cuda_group_norm(out.data_ptr(), out.dtype.code, L.arr64(ys), x.data_ptr(), x.dtype.code,
                                   L.arr64(xs), weight.data_ptr() if weight is not None else None,
                                   bias.data_ptr() if bias is not None else None, wbd, N, Cc, HW, num_groups,
                                   float(eps), 1 if fuse_silu else 0, ws, wsb, x._stream()), "group_norm")
    return out


def _unary(x: Tensor, op: str) -> Tensor:
    _require_cuda(x)
    cl = x.dim() == 4 and x.is_contiguous("channels_last")
    xc = x if (x.is_contiguous() or cl) else x.contiguous()
    out = _new(x._shape, x.dtype, x.device, channels_last=cl and not x.is_contiguous())
    L.check(_lib().mt_cuda_unary(L.UNARY[op], out.data_ptr(), out.dtype.code, xc.data_ptr(), xc.dtype.code,
                                 xc.numel(), x._stream()), op)
    return out


def silu(x: Tensor) -> Tensor:
    """`silu` (tensor.cpp:16480-16600)."""
    return _unary(x, "silu")


def gelu(x: Tensor, approximate="none") -> Tensor:
    """`gelu` (tensor.cpp:17207-17290)."""
    if approximate not in ("none", "tanh"):
        raise ValueError("gelu approximate must be 'none' or 'tanh'")
    return _unary(x, "gelu" if approximate == "none" else "gelu_tanh")


def sigmoid(x):
    return _unary(x, "sigmoid")


def relu(x):
    return _unary(x, "relu")


def exp(x):
    return _unary(x, "exp")


def quick_gelu(x):
    """CLIP's x * sigmoid(1.702 x) in one pass (the reference composes it from mul and sigmoid,
    tests/compat/benchmarking.py:7714)."""
    return _unary(x, "quick_gelu")


def _ids_on_device(ids: Tensor, rows: int, dev) -> Tensor:
    """int64 ids on `dev`.  Host ids are range-checked on the host (the reference's
    normalized_dim_index raises std::out_of_range -> IndexError) before the copy."""
    if ids.dtype not in (int32, int64):
        raise ValueError("embedding indices must have integer dtype")
    if ids.device.type != "cpu" and ids.dtype is int64:
        return ids.contiguous()
    a = ids.numpy().astype(np.int64)  # host ids, or device int32 ids widened on the host
    if a.size and (a.min() < -rows or a.max() >= rows):
        raise IndexError("index out of range in embedding")
    return tensor(a).to(dev)


def embedding(input: Tensor, weight: Tensor, padding_idx=None, max_norm=None, norm_type=2.0,
              scale_grad_by_freq=False, sparse=False, *, add_weight: Tensor | None = None,
              add_input: Tensor | None = None) -> Tensor:
    """`embedding` (tensor.cpp:31748-31800): rows of `weight` [rows, dim] selected by `input`.
    `add_weight` / `add_input` (keyword-only, an extension) add a second gathered table in the same
    pass — CLIP's token + position embedding.  Ids may live on the host (checked there) or on the
    device (an out-of-range id is counted by the kernel and raises IndexError after a sync)."""
    _require_cuda(weight)
    if weight.dim() != 2:
        raise ValueError("embedding weight must be 2-D")
    if max_norm is not None:
        raise NotImplementedError("embedding max_norm renormalisation is not implemented on the cuda device")
    rows, dim = weight._shape
    if padding_idx is not None:
        p = padding_idx + rows if padding_idx < 0 else padding_idx
        if not 0 <= p < rows:
            raise IndexError("embedding padding_idx is out of bounds")
    dev = weight.device
    ids = _ids_on_device(input, rows, dev)
    w = weight.contiguous()
    out = _new(tuple(input._shape) + (dim,), weight.dtype, dev)
    add = add_ids = None
    add_rows = 0
    if add_weight is not None:
        _require_cuda(add_weight)
        if add_weight.dim() != 2 or add_weight._shape[1] != dim:
            raise ValueError("embedding: add_weight must be [rows, dim] with the same dim")
        if add_input is None or tuple(add_input.shape) != tuple(input.shape):
            raise ValueError("embedding: add_input must have the shape of input")
        add = add_weight.contiguous()
        add_rows = add._shape[0]
        add_ids = _ids_on_device(add_input, add_rows, dev)
    device_ids = (input.device.type != "cpu" and input.dtype is int64) or (
        add_input is not None and add_input.device.type != "cpu" and add_input.dtype is int64)
    counter = zeros(1, dtype=int32, device=dev) if device_ids else None
    L.check(_lib().mt_cuda_embedding(out.data_ptr(), out.dtype.code, w.data_ptr(), w.dtype.code, rows, dim,
                                     ids.data_ptr(), ids.numel(), add.data_ptr() if add is not None else None,
                                     add.dtype.code if add is not None else 0, add_rows,
                                     add_ids.data_ptr() if add_ids is not None else None,
                                     counter.data_ptr() if counter is not None else None, weight._stream()),
            "embedding")
    if counter is not None and int(counter.item()) != 0:
        raise IndexError("index out of range in embedding")
    return out


def timestep_embedding(timesteps: Tensor, dim: int, dtype=None, flip_sin_to_cos=True, max_period=10000.0,
                       batch: int | None = None) -> Tensor:
    """Sinusoidal timestep embedding [n, dim] on the device, fp32 math in the reference's order
    (tests/compat/benchmarking.py:6011-6036): freq_j = exp(-ln(max_period) * j / (dim/2)),
    [cos(t freq) | sin(t freq)].  `timesteps` is a device tensor of n values, or one value
    broadcast over `batch` rows (so a captured graph can read the step's timestep from memory)."""
    _require_cuda(timesteps)
    t = timesteps.contiguous()
    if batch is None:
        n, stride = t.numel(), 1
    else:
        if t.numel() != 1:
            raise ValueError("timestep_embedding: batch= needs a single timestep")
        n, stride = int(batch), 0
    out = _new((n, dim), to_dtype(dtype) if dtype is not None else float32, t.device)
    L.check(_lib().mt_cuda_timestep_embedding(out.data_ptr(), out.dtype.code, t.data_ptr(), t.dtype.code, stride, n,
                                              dim, float(max_period), 1 if flip_sin_to_cos else 0, t._stream()),
            "timestep_embedding")
    return out


def ddim_step_indexed(x: Tensor, eps: Tensor, alphas_cumprod: Tensor, timestep: Tensor, interval: int, clip=True,
                      guidance_scale: float | None = None, out: Tensor | None = None, out_copies: int = 1) -> Tensor:
    """DDIM update reading the timestep from device memory (one graph serves every step), with
    classifier-free guidance folded in when `guidance_scale` is given: `eps` is then the model
    output for the doubled batch [uncond; text] (tests/compat/benchmarking.py:5847-5850,
    6148-6168).  `out` receives `out_copies` (1 or 2) stacked copies of the updated latents; 2
    writes the next step's doubled model input directly.  `out` may alias `x`'s storage."""
    _require_cuda(x, eps, alphas_cumprod, timestep)
    if alphas_cumprod.dtype is not float64 or timestep.dtype is not int64:
        raise ValueError("ddim_step_indexed: alphas_cumprod must be float64 and timestep int64")
    n = x.numel()
    cfg = guidance_scale is not None
    if eps.numel() != (2 * n if cfg else n):
        raise ValueError(f"ddim_step_indexed: eps has {eps.numel()} values, expected {(2 if cfg else 1) * n}")
    if x.is_contiguous() is False or eps.is_contiguous() is False:
        raise ValueError("ddim_step_indexed: x and eps must be contiguous")
    if out is None:
        out = _new((out_copies * x._shape[0],) + tuple(x._shape[1:]), x.dtype, x.device)
    if out.numel() != out_copies * n or not out.is_contiguous():
        raise ValueError("ddim_step_indexed: out must be contiguous with out_copies * x.numel() values")
    L.check(_lib().mt_cuda_ddim_step_indexed(out.data_ptr(), out_copies, x.data_ptr(), eps.data_ptr(), x.dtype.code,
                                             eps.dtype.code, n, alphas_cumprod.data_ptr(), alphas_cumprod.numel(),
                                             timestep.data_ptr(), int(interval), 1 if cfg else 0,
                                             float(guidance_scale) if cfg else 0.0, 1 if clip else 0, x._stream()),
            "ddim_step_indexed")
    return out


# ---------------------------------------------------------------------------------------------
# cat / interpolate (copies through mt_cuda_copy_strided)


def _copy_into(dst: Tensor, src: Tensor):
    L.check(_lib().mt_cuda_copy_strided(dst.data_ptr(), dst.dtype.code, L.arr64(dst._strides), src.data_ptr(),
                                        src.dtype.code, L.arr64(src._strides), L.arr64(dst._shape), dst.dim(),
                                        dst._stream()), "copy")


def cat(tensors, dim=0) -> Tensor:
    """`cat` (tensor.cpp:32141)."""
    ts = [t for t in tensors if not (t.dim() == 1 and t.numel() == 0)]
    _require_cuda(*ts)
    ref = ts[0]
    dim = dim % ref.dim()
    shape = list(ref._shape)
    shape[dim] = sum(t._shape[dim] for t in ts)
    cl = ref.dim() == 4 and all(t.is_contiguous("channels_last") and not t.is_contiguous() for t in ts)
    out = _new(shape, ref.dtype, ref.device, channels_last=cl)
    off = 0
    for t in ts:
        _copy_into(out.narrow(dim, off, t._shape[dim]), t)
        off += t._shape[dim]
    return out


def interpolate_nearest2x(x: Tensor) -> Tensor:
    """Nearest-neighbour 2x upsample of [N, C, H, W] (interpolate, tensor.cpp:10897): a broadcast
    view [N, C, H, 2, W, 2] copied once into the output (layout follows the input)."""
    _require_cuda(x)
    N, Cc, H, W = x._shape
    cl = x.is_contiguous("channels_last") and not x.is_contiguous()
    out = _new((N, Cc, 2 * H, 2 * W), x.dtype, x.device, channels_last=cl)
    sn, sc, sh, sw = x._strides
    src = x._view((N, Cc, H, 2, W, 2), (sn, sc, sh, 0, sw, 0))
    on, oc, oh, ow = out._strides
    dst = out._view((N, Cc, H, 2, W, 2), (on, oc, 2 * oh, oh, 2 * ow, ow))
    _copy_into(dst, src)
    return out


def ddim_step(x: Tensor, eps: Tensor, alpha_t: float, alpha_prev: float, clip=True, out: Tensor | None = None):
    """One DDIM latent update (the reference's scheduler scenario, tests/compat/benchmarking.py:
    6148-6168) as a single fused kernel."""
    _require_cuda(x, eps)
    xc, ec = x.contiguous(), eps.contiguous()
    if out is None:
        out = _new(x._shape, x.dtype, x.device)
    L.check(_lib().mt_cuda_ddim_step(out.data_ptr(), xc.data_ptr(), ec.data_ptr(), x.dtype.code, ec.dtype.code,
                                     x.numel(), float(alpha_t), float(alpha_prev), 1 if clip else 0, x._stream()),
            "ddim_step")
    return out
