"""CPU oracle for the device path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
package, and only as the checker; the product (``mtorch_b200``) never does.

* ``oracle.ref`` gives the reference mtorch itself (built from the reference sources into
  ``oracle/_ref`` by ``build_ref.py``) when it is available;
* the ``*_f32`` functions below are the C restatement in ``mtorch_oracle.c`` (compiled to
  ``oracle/_build/liboracle.so`` by ``build()``), numpy in / numpy out.
"""
from __future__ import annotations

import ctypes as C
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SO = HERE / "_build" / "liboracle.so"
_L = None


def build() -> Path:
    src = HERE / "mtorch_oracle.c"
    if not SO.exists() or SO.stat().st_mtime < src.stat().st_mtime:
        SO.parent.mkdir(exist_ok=True)
        tmp = SO.with_suffix(".tmp")
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-ffp-contract=off", str(src), "-o", str(tmp), "-lm"])
        tmp.replace(SO)
    return SO


def _lib():
    global _L
    if _L is None:
        build()
        _L = C.CDLL(str(SO))
    return _L


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


I = C.c_int64


def matmul_f32(A, B):
    A, B = _f(A), _f(B)
    M, K = A.shape
    N = B.shape[1]
    out = np.empty((M, N), np.float32)
    _lib().oracle_matmul_f32(_p(A), _p(B), _p(out), I(M), I(K), I(N))
    return out


def addmm_f32(inp, A, B, beta=1.0, alpha=1.0):
    A, B = _f(A), _f(B)
    M, K = A.shape
    N = B.shape[1]
    inp = _f(np.broadcast_to(inp, (M, N)))
    out = np.empty((M, N), np.float32)
    _lib().oracle_addmm_f32(_p(inp), _p(A), _p(B), _p(out), I(M), I(K), I(N), C.c_double(beta), C.c_double(alpha))
    return out


def baddbmm_f32(inp, A, B, beta=1.0, alpha=1.0):
    """A [b, M, K] @ B [b, K, N], input broadcast to [b, M, N]."""
    A, B = _f(A), _f(B)
    nb, M, K = A.shape
    N = B.shape[2]
    inp = _f(np.broadcast_to(inp, (nb, M, N)))
    out = np.empty((nb, M, N), np.float32)
    for k in range(nb):
        _lib().oracle_baddbmm_f32(_p(inp[k]), _p(_f(A[k])), _p(_f(B[k])), _p(out[k]), I(M), I(K), I(N),
                                  C.c_double(beta), C.c_double(alpha))
    return out


def linear_f32(X, W, b=None):
    X, W = _f(X), _f(W)
    lead = X.shape[:-1]
    K = X.shape[-1]
    N = W.shape[0]
    X2 = X.reshape(-1, K)
    out = np.empty((X2.shape[0], N), np.float32)
    bb = _f(b) if b is not None else None
    _lib().oracle_linear_f32(_p(X2), _p(W), _p(bb), _p(out), I(X2.shape[0]), I(K), I(N))
    return out.reshape(lead + (N,))


def conv2d_f32(x, w, b=None, stride=1, padding=0, dilation=1, groups=1):
    x, w = _f(x), _f(w)
    sh, sw = (stride, stride) if isinstance(stride, int) else stride
    ph, pw = (padding, padding) if isinstance(padding, int) else padding
    dh, dw = (dilation, dilation) if isinstance(dilation, int) else dilation
    N, Cc, H, W = x.shape
    K, _, R, S = w.shape
    P = (H + 2 * ph - dh * (R - 1) - 1) // sh + 1
    Q = (W + 2 * pw - dw * (S - 1) - 1) // sw + 1
    out = np.empty((N, K, P, Q), np.float32)
    bb = _f(b) if b is not None else None
    _lib().oracle_conv2d_f32(_p(x), _p(w), _p(bb), _p(out), I(N), I(Cc), I(H), I(W), I(K), I(R), I(S), I(sh), I(sw),
                             I(ph), I(pw), I(dh), I(dw), I(groups))
    return out


def sdpa_f32(q, k, v, mask=None, causal=False, scale=None):
    """q [..., Lq, D], k [..., Sk, D], v [..., Sk, Dv]; mask broadcastable to [..., Lq, Sk]."""
    q, k, v = _f(q), _f(k), _f(v)
    lead = q.shape[:-2]
    Lq, D = q.shape[-2:]
    Sk, Dv = v.shape[-2:]
    P = int(np.prod(lead)) if lead else 1
    k = _f(np.broadcast_to(k, lead + k.shape[-2:]))
    v = _f(np.broadcast_to(v, lead + v.shape[-2:]))
    out = np.empty(lead + (Lq, Dv), np.float32)
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    mp, kind, ps = None, 0, 0
    if mask is not None:
        m = np.broadcast_to(mask, lead + (Lq, Sk))
        if m.dtype == np.bool_:
            mp, kind = np.ascontiguousarray(m.astype(np.uint8)), 1
        else:
            mp, kind = _f(m), 2
        ps = Lq * Sk
    _lib().oracle_sdpa_f32(_p(q), _p(k), _p(v), _p(out), I(P), I(Lq), I(Sk), I(D), I(Dv), C.c_double(scale), _p(mp),
                           C.c_int(kind), I(ps), C.c_int(1 if causal else 0))
    return out


def softmax_f32(x):
    x = _f(x)
    out = np.empty_like(x)
    cols = x.shape[-1]
    _lib().oracle_softmax_f32(_p(x), _p(out), I(x.size // cols), I(cols))
    return out


def layer_norm_f32(x, w=None, b=None, eps=1e-5):
    x = _f(x)
    out = np.empty_like(x)
    cols = x.shape[-1] if w is None else int(np.prod(np.shape(w)))
    _lib().oracle_layer_norm_f32(_p(x), _p(_f(w) if w is not None else None), _p(_f(b) if b is not None else None),
                                 _p(out), I(x.size // cols), I(cols), C.c_double(eps))
    return out


def group_norm_f32(x, G, w=None, b=None, eps=1e-5):
    x = _f(x)
    N, Cc = x.shape[:2]
    HW = int(np.prod(x.shape[2:]))
    out = np.empty_like(x)
    _lib().oracle_group_norm_f32(_p(x), _p(_f(w) if w is not None else None), _p(_f(b) if b is not None else None),
                                 _p(out), I(N), I(Cc), I(HW), I(G), C.c_double(eps))
    return out


def silu_f32(x):
    x = _f(x)
    out = np.empty_like(x)
    _lib().oracle_silu_f32(_p(x), _p(out), I(x.size))
    return out


def gelu_f32(x, approximate="none"):
    x = _f(x)
    out = np.empty_like(x)
    _lib().oracle_gelu_f32(_p(x), _p(out), I(x.size), C.c_int(1 if approximate == "tanh" else 0))
    return out


def quick_gelu_f32(x):
    x = _f(x)
    out = np.empty_like(x)
    _lib().oracle_quick_gelu_f32(_p(x), _p(out), I(x.size))
    return out


def timestep_embedding_f32(t, dim, max_period=10000.0, flip=True):
    t = _f(t).reshape(-1)
    out = np.empty((t.size, dim), np.float32)
    _lib().oracle_timestep_embedding_f32(_p(t), _p(out), I(t.size), I(dim), C.c_double(max_period),
                                         C.c_int(1 if flip else 0))
    return out


def embedding_f32(w, ids, add=None, add_ids=None):
    """Returns (rows [*ids.shape, dim], number of out-of-range ids)."""
    w = _f(w)
    ids = np.ascontiguousarray(ids, np.int64)
    dim = w.shape[1]
    out = np.empty(ids.shape + (dim,), np.float32)
    a = _f(add) if add is not None else None
    ai = np.ascontiguousarray(add_ids, np.int64) if add_ids is not None else None
    f = _lib().oracle_embedding_f32
    f.restype = C.c_int64
    bad = f(_p(w), I(w.shape[0]), I(dim), _p(ids), I(ids.size), _p(a), I(a.shape[0] if a is not None else 0), _p(ai),
            _p(out))
    return out, int(bad)


def cfg_ddim_f32(x, eps, g, a_t, a_prev, clip=True):
    """eps = [uncond; text] stacked on the first axis (2n rows for n latents)."""
    x, eps = _f(x), _f(eps)
    out = np.empty_like(x)
    _lib().oracle_cfg_ddim_f32(_p(x), _p(eps), _p(out), I(x.size), C.c_double(g), C.c_double(a_t),
                               C.c_double(a_prev), C.c_int(1 if clip else 0))
    return out


def ref():
    """The reference mtorch module (built CPU implementation) or None when not built here."""
    from . import build_ref

    if not build_ref.available():
        return None
    p = str(build_ref.OUT)
    if p not in sys.path:
        sys.path.insert(0, p)
    import mtorch  # noqa: E402

    return mtorch
