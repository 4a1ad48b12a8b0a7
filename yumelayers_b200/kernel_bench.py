"""Per-kernel timing of the conv and GroupNorm kernels on the workload's layer
shapes (the B200 counterpart of the reference's profileConv, Diagnostics.swift:
124-201).  Prints one JSON line per shape.

    python -m yumelayers_b200.kernel_bench [--shapes vae|unet|epilogue|small] [--reps R] [--only NAME]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import sys

from ._lib import ConvProfile, call
from .session import Context

# (name, n, c, h, w, oc, k, stride, up): the distinct conv shapes of one batch-8
# VAE step at 480x856 (up = 1: the input is the half-resolution source).
VAE_SHAPES = [
    ("full_128_128", 8, 128, 480, 856, 128, 3, 1, 0),
    ("full_in_4_128", 8, 4, 480, 856, 128, 3, 1, 0),
    ("full_out_128_4", 8, 128, 480, 856, 4, 3, 1, 0),
    ("down1_128_s2", 8, 128, 480, 856, 128, 3, 2, 0),
    ("half_128_256", 8, 128, 240, 428, 256, 3, 1, 0),
    ("half_256_256", 8, 256, 240, 428, 256, 3, 1, 0),
    ("half_skip_128_256", 8, 128, 240, 428, 256, 1, 1, 0),
    ("quarter_256_256", 8, 256, 120, 214, 256, 3, 1, 0),
    ("up3_256_128", 8, 256, 240, 428, 128, 3, 1, 1),
    ("up2_256_256", 8, 256, 120, 214, 256, 3, 1, 1),
]
# the motion U-Net's 3x3 convs on batch-8 latents of 60x107 (and its two
# down-sampled levels)
UNET_SHAPES = [
    ("u60_96_128", 8, 96, 60, 107, 128, 3, 1, 0),
    ("u60_128_128", 8, 128, 60, 107, 128, 3, 1, 0),
    ("u30_256_256", 8, 256, 30, 54, 256, 3, 1, 0),
    ("u15_384_384", 8, 384, 15, 27, 384, 3, 1, 0),
    ("u30_512_256", 8, 512, 30, 54, 256, 3, 1, 0),
]
# pointwise GEMMs whose time is the epilogue's (one or two 32-channel k-blocks)
EPILOGUE_SHAPES = [
    ("pw_32_128", 8, 32, 480, 856, 128, 1, 1, 0),
    ("pw_64_128", 8, 64, 480, 856, 128, 1, 1, 0),
]
SMALL_SHAPES = [
    ("small_128_128", 8, 128, 192, 192, 128, 3, 1, 0),
    ("small_256_256", 8, 256, 96, 192, 256, 3, 1, 0),
    ("mid_128_128", 2, 128, 480, 856, 128, 3, 1, 0),
]


def _sobel(ctx, reps: int) -> None:
    """Device time of yl_sobel_edge_loss on 8 NCHW RGB frames of 480x856
    (reads recon + target, writes the gradient: 36 B per pixel)."""
    import numpy as np
    from .session import GPUTensor
    n, h, w = 8, 480, 856
    rng = np.random.default_rng(0)
    r = GPUTensor(ctx, 1, n * 3 * h * w, rng.uniform(0, 1, n * 3 * h * w).astype(np.float32))
    t = GPUTensor(ctx, 1, n * 3 * h * w, rng.uniform(0, 1, n * 3 * h * w).astype(np.float32))
    g, loss = GPUTensor(ctx, 1, n * 3 * h * w), GPUTensor(ctx, 1, n)
    ms = C.c_double()
    args = (ctx.handle, C.c_void_p(r.ptr), C.c_void_p(t.ptr), n, h, w, 0, 0, C.c_void_p(g.ptr),
            C.c_void_p(loss.ptr))
    call("yl_sobel_edge_loss", *args)  # warm-up
    call("yl_session_begin", ctx.handle)
    for _ in range(reps):
        call("yl_sobel_edge_loss", *args)
    call("yl_session_end", ctx.handle, 60.0, C.byref(ms))
    per = ms.value / reps
    print(json.dumps({"sobel": [n, 3, h, w], "ms": per,
                      "gbs": 36.0 * n * h * w / (per * 1e-3) / 1e9}), flush=True)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="vae", choices=["vae", "unet", "epilogue", "small"])
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--only", default=None)
    ap.add_argument("--groupnorm", action="store_true")
    ap.add_argument("--layered", action="store_true",
                    help="layered 8-channel loss + gradient (108 B per pixel)")
    ap.add_argument("--sobel", action="store_true",
                    help="Sobel edge loss + gradient on 8 RGB frames of 480x856 (NCHW)")
    ap.add_argument("--adam", action="store_true",
                    help="one multi-tensor Adam step over the joint step's 28.5 M parameters")
    a = ap.parse_args(argv)
    ctx = Context.shared(0)
    shapes = {"vae": VAE_SHAPES, "unet": UNET_SHAPES, "epilogue": EPILOGUE_SHAPES,
              "small": SMALL_SHAPES}[a.shapes]
    for name, n, c, h, w, oc, k, s, up in shapes:
        if a.only and a.only != name:
            continue
        p = ConvProfile()
        call("yl_profile_conv", ctx.handle, n, c, h, w, oc, k, s, up, a.reps, C.byref(p))
        row = {"shape": name, "n": n, "c": c, "h": h, "w": w, "oc": oc, "k": k, "stride": s,
               "up": up, "gflop": p.flops / 1e9, "wgrad_splits": p.wgrad_splits}
        for m in ("fprop", "dgrad", "wgrad"):
            ms = getattr(p, m + "_ms")
            row[m + "_ms"] = round(ms, 4)
            row[m + "_tflops"] = round(p.flops / (ms * 1e-3) / 1e12, 1)
        print(json.dumps(row), flush=True)
    if a.groupnorm:
        gn_shapes = ([(8, 128, 480, 856), (8, 256, 240, 428)] if a.shapes == "vae"
                     else [(8, 128, 192, 192)])
        for (n, c, h, w) in gn_shapes:
            f, b, ap = C.c_double(), C.c_double(), C.c_double()
            call("yl_profile_groupnorm", ctx.handle, n, c, h, w, a.reps, C.byref(f), C.byref(b),
                 C.byref(ap))
            e = n * c * h * w * 4
            print(json.dumps({"groupnorm": [n, c, h, w], "fwd_ms": f.value, "bwd_ms": b.value,
                              "apply_ms": ap.value, "apply_gbs": 2 * e / (ap.value * 1e-3) / 1e9,
                              "fwd_gbs": 3 * e / (f.value * 1e-3) / 1e9,
                              "bwd_gbs": 5 * e / (b.value * 1e-3) / 1e9}), flush=True)
    if a.adam:
        n, tensors = 13404612 + 15092896, 48  # VAE + motion U-Net parameter counts
        ms = C.c_double()
        call("yl_profile_adam", ctx.handle, n, tensors, a.reps, C.byref(ms))
        print(json.dumps({"adam_params": n, "ms": ms.value,
                          "gbs": 28.0 * n / (ms.value * 1e-3) / 1e9}), flush=True)
    if a.sobel:
        _sobel(ctx, a.reps)
    if a.layered:
        n, plane = (8, 480 * 856) if a.shapes == "vae" else (4, 480 * 856)
        ms = C.c_double()
        call("yl_profile_layered", ctx.handle, n, plane, a.reps, C.byref(ms))
        print(json.dumps({"layered_loss": [n, 8, plane], "ms": ms.value,
                          "gbs": 108.0 * n * plane / (ms.value * 1e-3) / 1e9}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
