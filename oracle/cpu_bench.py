"""Reference-CPU timing of the SD-1.5 UNet step — TEST/BENCH INFRASTRUCTURE ONLY (used by
bench.py's reference arm and its cpu_baseline leg; never by the product).

The reference's own portable CPU code (built from its sources into oracle/_ref by build_ref.py;
the C restatement of oracle/mtorch_oracle.c, "port", when that build is absent) runs EVERY op of
one sample's UNet forward — conv2d, linear, scaled_dot_product_attention, group_norm, layer_norm,
silu, gelu, add, mul, cat, interpolate — at the model's full channel widths and key lengths, on a
1/R slice of each op's output rows (output pixels of a conv, query rows of an attention, token rows
of a linear / layer norm, pixels of a group norm or elementwise op; at least one).  Every one of
these ops costs the same per output row whatever the number of rows, so one sampled step is 1/R
of one sample's UNet forward, and a C5 step (64 samples) is 64 * R sampled steps.

The ops are spread over P worker processes (the reference is single-threaded), statically
balanced by their FLOPs; a step's time is the wall time from the start signal to the last
worker's reply.  This module does not import mtorch_b200, so the timed processes load only the
reference (or the oracle) library.
"""
from __future__ import annotations

import math
import multiprocessing as mp
import time

import numpy as np

CHANS = (320, 640, 1280, 1280)
ATTN = (True, True, True, False)
HEADS = 8
CTX_LEN, CTX_DIM, TDIM = 77, 768, 1280


def resnet_ops(cin, cout, h):
    """Ops of one sample's SD ResNet block at h x h: GN + SiLU, conv3x3, time-embedding linear and
    add, GN + SiLU, conv3x3, (1x1 shortcut), residual add."""
    hw = h * h
    ops = [("gn", cin, hw), ("ew", cin * hw), ("conv", cin, cout, 3, 1, h, h), ("lin", 1, TDIM, cout),
           ("ew", cout * hw), ("gn", cout, hw), ("ew", cout * hw), ("conv", cout, cout, 3, 1, h, h)]
    if cin != cout:
        ops.append(("conv", cin, cout, 1, 1, h, h))
    ops.append(("ew", cout * hw))
    return ops


def transformer_ops(c, h):
    """Ops of one sample's SD spatial transformer at h x h with c channels: GN, proj_in, self-
    attention (LN, QKV, SDPA, out + residual), cross-attention to the 77x768 context, GEGLU FFN,
    proj_out + residual."""
    s = h * h
    d = c // HEADS
    return [("gn", c, s), ("lin", s, c, c), ("ln", s, c), ("lin", s, c, 3 * c), ("attn", HEADS, s, s, d),
            ("lin", s, c, c), ("ew", s * c), ("ln", s, c), ("lin", s, c, c), ("lin", CTX_LEN, CTX_DIM, 2 * c),
            ("attn", HEADS, s, CTX_LEN, d), ("lin", s, c, c), ("ew", s * c), ("ln", s, c),
            ("lin", s, c, 8 * c), ("ew", s * 4 * c), ("ew", s * 4 * c), ("lin", s, 4 * c, c), ("ew", s * c),
            ("lin", s, c, c), ("ew", s * c)]


def unet_ops(size=64):
    """The op list of one sample's SD-1.5 UNet forward (fp32, unfused, in the reference's op
    order).  Each entry: (kind, dims...) with
      conv  (cin, cout, k, stride, P, Q)        output P x Q
      attn  (heads, Sq, Sk, D)
      lin   (rows, in, out)
      gn    (C, HW)      ln (rows, C)      ew (elements)      up (C, H, W) nearest 2x"""
    ops = []
    ops.extend([("lin", 1, CHANS[0], TDIM), ("ew", TDIM), ("lin", 1, TDIM, TDIM), ("ew", TDIM)])
    h = size
    ops.append(("conv", 4, CHANS[0], 3, 1, h, h))
    c, skip = CHANS[0], [CHANS[0]]
    for lvl, co in enumerate(CHANS):
        for _ in range(2):
            ops.extend(resnet_ops(c, co, h))
            c = co
            if ATTN[lvl]:
                ops.extend(transformer_ops(c, h))
            skip.append(c)
        if lvl != len(CHANS) - 1:
            h //= 2
            ops.append(("conv", c, c, 3, 2, h, h))
            skip.append(c)
    ops.extend(resnet_ops(c, c, h))
    ops.extend(transformer_ops(c, h))
    ops.extend(resnet_ops(c, c, h))
    for lvl, co in reversed(list(enumerate(CHANS))):
        for _ in range(3):
            cin = c + skip.pop()
            ops.append(("ew", cin * h * h))  # cat
            ops.extend(resnet_ops(cin, co, h))
            c = co
            if ATTN[lvl]:
                ops.extend(transformer_ops(c, h))
        if lvl != 0:
            ops.append(("up", c, h, h))
            h *= 2
            ops.append(("conv", c, c, 3, 1, h, h))
    ops.extend([("gn", c, h * h), ("ew", c * h * h), ("conv", c, 4, 3, 1, h, h)])
    return ops


def op_flops(op) -> float:
    k = op[0]
    if k == "conv":
        _, ci, co, r, _, p, q = op
        return 2.0 * ci * co * r * r * p * q
    if k == "attn":
        _, hh, sq, sk, d = op
        return 4.0 * hh * sq * sk * d
    if k == "lin":
        _, rows, i, o = op
        return 2.0 * rows * i * o
    if k == "mm":
        _, m, kk, n = op
        return 2.0 * m * kk * n
    return 0.0


def _rows(n, r):
    return max(1, n // r)


class _Ref:
    """Sampled ops on the reference mtorch."""

    def __init__(self, m):
        self.m, self.F = m, m.nn.functional

    def randn(self, *shape):
        return self.m.randn(*shape) * 0.05

    def prepare(self, op, r):
        k = op[0]
        if k == "conv":
            _, ci, co, kk, st, p, q = op
            n = _rows(p * q, r)
            qc = min(q, n)
            pr = max(1, n // qc)
            x = self.randn(1, ci, (pr - 1) * st + kk, (qc - 1) * st + kk)
            w, b = self.randn(co, ci, kk, kk), self.randn(co)
            return lambda: self.F.conv2d(x, w, b, st, 0)
        if k == "attn":
            _, hh, sq, sk, d = op
            q, kt, v = self.randn(1, hh, _rows(sq, r), d), self.randn(1, hh, sk, d), self.randn(1, hh, sk, d)
            return lambda: self.F.scaled_dot_product_attention(q, kt, v)
        if k == "lin":
            _, rows, i, o = op
            x, w, b = self.randn(_rows(rows, r), i), self.randn(o, i), self.randn(o)
            return lambda: self.F.linear(x, w, b)
        if k == "mm":
            _, m, kk, n = op
            a, b2 = self.randn(_rows(m, r), kk), self.randn(kk, n)
            return lambda: self.m.matmul(a, b2)
        if k == "gn":
            _, c, hw = op
            x, w, b = self.randn(1, c, _rows(hw, r), 1), self.randn(c), self.randn(c)
            return lambda: self.F.group_norm(x, 32, w, b, 1e-5)
        if k == "ln":
            _, rows, c = op
            x, w, b = self.randn(_rows(rows, r), c), self.randn(c), self.randn(c)
            return lambda: self.F.layer_norm(x, [c], w, b, 1e-5)
        if k == "up":
            _, c, h, w_ = op
            x = self.randn(1, c, 1, _rows(h * w_, r))
            return lambda: self.F.interpolate(x, scale_factor=2, mode="nearest")
        x, y = self.randn(_rows(op[1], r)), self.randn(_rows(op[1], r))
        return lambda: x + y


class _Port:
    """Sampled ops on the C restatement (when the reference build is absent)."""

    def __init__(self, oracle):
        self.o = oracle
        self.rng = np.random.default_rng(0)

    def randn(self, *shape):
        return (self.rng.standard_normal(shape) * 0.05).astype(np.float32)

    def prepare(self, op, r):
        o, k = self.o, op[0]
        if k == "conv":
            _, ci, co, kk, st, p, q = op
            n = _rows(p * q, r)
            qc = min(q, n)
            pr = max(1, n // qc)
            x = self.randn(1, ci, (pr - 1) * st + kk, (qc - 1) * st + kk)
            w, b = self.randn(co, ci, kk, kk), self.randn(co)
            return lambda: o.conv2d_f32(x, w, b, st, 0)
        if k == "attn":
            _, hh, sq, sk, d = op
            q, kt, v = self.randn(1, hh, _rows(sq, r), d), self.randn(1, hh, sk, d), self.randn(1, hh, sk, d)
            return lambda: o.sdpa_f32(q, kt, v)
        if k == "lin":
            _, rows, i, oo = op
            x, w, b = self.randn(_rows(rows, r), i), self.randn(oo, i), self.randn(oo)
            return lambda: o.linear_f32(x, w, b)
        if k == "mm":
            _, m, kk, n = op
            a, b2 = self.randn(_rows(m, r), kk), self.randn(kk, n)
            return lambda: o.matmul_f32(a, b2)
        if k == "gn":
            _, c, hw = op
            x = self.randn(1, c, _rows(hw, r), 1)
            return lambda: o.group_norm_f32(x, 32)
        if k == "ln":
            _, rows, c = op
            x = self.randn(_rows(rows, r), c)
            return lambda: o.layer_norm_f32(x)
        if k == "up":
            _, c, h, w_ = op
            x = self.randn(1, c, 1, _rows(h * w_, r))
            return lambda: x.repeat(2, axis=2).repeat(2, axis=3)
        x = self.randn(_rows(op[1], r))
        return lambda: o.silu_f32(x + x)


def _worker(conn, ops, r):
    import oracle

    m = oracle.ref()
    runner = _Ref(m) if m is not None else _Port(oracle)
    fns = [runner.prepare(op, r) for op in ops]
    conn.send(("ready", "reference" if m is not None else "port"))
    while True:
        msg = conn.recv()
        if msg == "stop":
            break
        t0 = time.perf_counter()
        for f in fns:
            f()
        conn.send(("done", time.perf_counter() - t0))


class SampledOps:
    """P worker processes, each owning a FLOP-balanced share of a sampled op list (one sample's ops;
    every op on 1/r of its output rows)."""

    def __init__(self, ops, processes: int, r: int):
        self.r, self.processes = r, max(1, processes)
        self.nops = len(ops)
        self.full_flops = sum(op_flops(o) for o in ops)
        shares: list[list] = [[] for _ in range(self.processes)]
        load = [0.0] * self.processes
        # longest-processing-time-first; memory-bound ops weighted by their element count
        cost = lambda o: op_flops(o) or 50.0 * (o[1] * (o[2] if o[0] in ("gn", "ln") else 1))  # noqa: E731
        for op in sorted(ops, key=cost, reverse=True):
            i = min(range(self.processes), key=load.__getitem__)
            shares[i].append(op)
            load[i] += cost(op)
        ctx = mp.get_context("spawn")
        self.conns, self.procs = [], []
        for share in shares:
            a, b = ctx.Pipe()
            p = ctx.Process(target=_worker, args=(b, share, r), daemon=True)
            p.start()
            self.conns.append(a)
            self.procs.append(p)
        kinds = {c.recv()[1] for c in self.conns}
        self.kind = "reference" if kinds == {"reference"} else "port"

    def step(self) -> float:
        """Wall seconds of one sampled step (all workers run their ops once)."""
        t0 = time.perf_counter()
        for c in self.conns:
            c.send("run")
        for c in self.conns:
            c.recv()
        return time.perf_counter() - t0

    def close(self):
        for c in self.conns:
            c.send("stop")
        for p in self.procs:
            p.join(timeout=10)

    def describe(self, what="one sample's SD-1.5 UNet forward", unit="a C5 step (64 samples) = 64") -> str:
        return (f"every op of {what} (fp32; {self.nops} ops: conv2d, linear, sdpa, group/layer norm, silu/gelu, "
                f"add/mul/cat, interpolate) at full widths on 1/{self.r} of each op's output rows, spread over "
                f"{self.processes} single-threaded processes; {unit} x {self.r} sampled steps")


class SampledUNet(SampledOps):
    """The sampled op list of one sample's SD-1.5 UNet forward."""

    def __init__(self, processes: int, r: int, size: int = 64):
        super().__init__(unet_ops(size), processes, r)


def config_ops(name: str):
    """One run of a BASELINE configuration as a list of ops: C1 the 2048^2 fp32 matmul, C2 the SD
    ResNet block (GN -> SiLU -> conv3x3 -> GN -> SiLU -> conv3x3 + residual) on [2, 320, 64, 64],
    C3 the attention block (self-attention over 4096 tokens, cross-attention to 77 projected context
    tokens, GEGLU FFN) on [2, 4096, 320]."""
    if name == "c1":
        return [("mm", 2048, 2048, 2048)]
    if name == "c2":
        one = [("gn", 320, 4096), ("ew", 320 * 4096), ("conv", 320, 320, 3, 1, 64, 64), ("gn", 320, 4096),
               ("ew", 320 * 4096), ("conv", 320, 320, 3, 1, 64, 64), ("ew", 320 * 4096)]
        return one * 2
    if name == "c3":
        return transformer_ops(320, 64)[2:-2] * 2  # without GroupNorm / proj_in and proj_out / residual
    raise ValueError(name)


class FullRun(SampledOps):
    """A whole configuration on all host cores: every op cut into r row slices (each slice the
    reference's own op on 1/r of the rows), the slices spread over the processes, so one step
    computes the full configuration."""

    def __init__(self, name: str, processes: int, r: int = 32):
        super().__init__(config_ops(name) * r, processes, r)
        self.name = name


def default_r(cores: int) -> int:
    """Sampling factor so that one sampled step takes a few seconds on `cores` host cores
    (about 1300 core-seconds per unsampled sample on the reference's portable path)."""
    return 1 << max(0, round(math.log2(max(1.0, 1300.0 / (3.0 * max(1, cores))))))
