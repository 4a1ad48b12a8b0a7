"""Device timing of the two single-op workloads of the benchmark plan through
the C ABI, on the reference's NCHW layout with device-resident buffers:

* conv3x3 (N=2, 32 -> 32, 64x64, stride 1, pad 1): forward + dX + dW + db,
  0.453 GFLOP (ConvLayerGPU.forward/backward, ConvGPU.swift:57-81);
* the ResNet block (N=8, C=128, 128x128): GroupNorm(32, eps 1e-6) + SiLU ->
  conv3x3 -> GroupNorm + SiLU -> conv3x3 + identity, forward and backward,
  231.9 GFLOP of convs (ResidualBlockGPU, ResidualBlock.swift:30-47).

Each repetition is one session (yl_session_begin / yl_session_end, device
time between its events) after a 256 MB write that evicts L2, so no
repetition starts with its inputs cached.  Every C-ABI call includes its
NCHW <-> NHWC conversions, as a caller of the reference's API would see.
"""
from __future__ import annotations

import ctypes as C
import statistics

import numpy as np

from ._lib import LAYOUT_NCHW, ConvDesc, call
from .session import Context, GPUTensor

CONV1 = dict(n=2, c=32, oc=32, h=64, w=64)
BLOCK = dict(n=8, c=128, h=128, w=128, groups=32, eps=1e-6)
CONV1_FLOPS = 3 * 2.0 * 2 * 32 * 32 * 9 * 64 * 64
BLOCK_FLOPS = 6 * 2.0 * 8 * 128 * 128 * 9 * 128 * 128


def _dev(ctx, a):
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    return GPUTensor(ctx, 1, a.size, a)


def _p(t):
    return C.c_void_p(t.ptr) if t is not None else None


class _Timer:
    """Per-repetition device time of `fn` with L2 evicted before each."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self.flush = GPUTensor(ctx, 1, 64 * 1024 * 1024)  # 256 MB > 126 MB L2

    def median_ms(self, fn, reps: int, warmup: int = 3) -> float:
        for _ in range(warmup):
            fn()
        out = []
        ms = C.c_double()
        for _ in range(reps):
            call("yl_zero_fill", self.ctx.handle, _p(self.flush), self.flush.n)
            call("yl_session_begin", self.ctx.handle)
            fn()
            call("yl_session_end", self.ctx.handle, 60.0, C.byref(ms))
            out.append(ms.value)
        return statistics.median(out)


def conv1_gpu_ms(ctx: Context | None = None, reps: int = 20) -> float:
    ctx = ctx or Context.shared()
    d = CONV1
    rng = np.random.default_rng(0)
    x = _dev(ctx, rng.standard_normal((d["n"], d["c"], d["h"], d["w"])))
    bound = np.sqrt(6.0 / (d["c"] * 9))
    w = _dev(ctx, rng.uniform(-bound, bound, (d["oc"], d["c"], 3, 3)))
    b = _dev(ctx, np.zeros(d["oc"]))
    dy = _dev(ctx, rng.standard_normal((d["n"], d["oc"], d["h"], d["w"])))
    y, dx = GPUTensor(ctx, 1, dy.n), GPUTensor(ctx, 1, x.n)
    dw, db = GPUTensor(ctx, 1, w.n), GPUTensor(ctx, 1, d["oc"])
    desc = ConvDesc(d["n"], d["c"], d["h"], d["w"], d["oc"], 3, 1, 1, 0, 0, 0, LAYOUT_NCHW)

    def step():
        h = ctx.handle
        call("yl_conv2d_fwd", h, C.byref(desc), _p(x), _p(w), _p(b), None, _p(y))
        call("yl_conv2d_bwd_data", h, C.byref(desc), _p(dy), _p(w), _p(dx))
        call("yl_conv2d_bwd_filter", h, C.byref(desc), _p(x), _p(dy), _p(dw), _p(db))

    return _Timer(ctx).median_ms(step, reps)


def block_gpu_ms(ctx: Context | None = None, reps: int = 10) -> float:
    ctx = ctx or Context.shared()
    d = BLOCK
    n, c, h, w, g, eps = d["n"], d["c"], d["h"], d["w"], d["groups"], d["eps"]
    rng = np.random.default_rng(0)
    e = n * c * h * w
    x = _dev(ctx, rng.standard_normal(e))
    dy = _dev(ctx, rng.standard_normal(e))
    gam = [_dev(ctx, 1 + 0.02 * rng.standard_normal(c)) for _ in range(2)]
    bet = [_dev(ctx, 0.02 * rng.standard_normal(c)) for _ in range(2)]
    bound = np.sqrt(6.0 / (c * 9))
    wt = [_dev(ctx, rng.uniform(-bound, bound, (c, c, 3, 3))) for _ in range(2)]
    cb = [_dev(ctx, np.zeros(c)) for _ in range(2)]
    h1, c1, h2, y, dh2, dc1, dh1, dx = (GPUTensor(ctx, 1, e) for _ in range(8))
    stats = [GPUTensor(ctx, 1, n * g) for _ in range(4)]
    dws = [GPUTensor(ctx, 1, c * c * 9) for _ in range(2)]
    dbs = [GPUTensor(ctx, 1, c) for _ in range(6)]
    desc = ConvDesc(n, c, h, w, c, 3, 1, 1, 0, 0, 0, LAYOUT_NCHW)

    def gn_f(src, i, out):
        call("yl_groupnorm_silu_fwd", ctx.handle, _p(src), n, c, h, w, LAYOUT_NCHW, g, eps, 0,
             _p(gam[i]), _p(bet[i]), 1, _p(out), _p(stats[2 * i]), _p(stats[2 * i + 1]))

    def gn_b(src, dout, i, addend, out):
        call("yl_groupnorm_silu_bwd", ctx.handle, _p(src), _p(dout), n, c, h, w, LAYOUT_NCHW, g,
             eps, 0, _p(gam[i]), _p(bet[i]), 1, None, None, _p(addend), _p(out),
             _p(dbs[2 + 2 * i]), _p(dbs[3 + 2 * i]))

    def step():
        hd = ctx.handle
        gn_f(x, 0, h1)
        call("yl_conv2d_fwd", hd, C.byref(desc), _p(h1), _p(wt[0]), _p(cb[0]), None, _p(c1))
        gn_f(c1, 1, h2)
        call("yl_conv2d_fwd", hd, C.byref(desc), _p(h2), _p(wt[1]), _p(cb[1]), _p(x), _p(y))
        call("yl_conv2d_bwd_data", hd, C.byref(desc), _p(dy), _p(wt[1]), _p(dh2))
        call("yl_conv2d_bwd_filter", hd, C.byref(desc), _p(h2), _p(dy), _p(dws[1]), _p(dbs[1]))
        gn_b(c1, dh2, 1, None, dc1)
        call("yl_conv2d_bwd_data", hd, C.byref(desc), _p(dc1), _p(wt[0]), _p(dh1))
        call("yl_conv2d_bwd_filter", hd, C.byref(desc), _p(h1), _p(dc1), _p(dws[0]), _p(dbs[0]))
        gn_b(x, dh1, 0, dy, dx)

    return _Timer(ctx).median_ms(step, reps)
