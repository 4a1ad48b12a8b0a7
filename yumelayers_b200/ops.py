"""numpy-in / numpy-out wrappers of the batched C-ABI operators.

Convenience for callers without a device allocator (and for the parity
tests): each call uploads its inputs into library-owned device buffers,
runs the CUDA operator and downloads the result.  The layout of every
activation array is the reference's NCHW (per-image CHW stacked).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import LAYOUT_NCHW, AdamTensor, ConvDesc, call
from .session import Context, GPUTensor


def _dev(ctx: Context, a) -> GPUTensor:
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    return GPUTensor(ctx, 1, a.size, a.reshape(-1)) if a.size else GPUTensor(ctx, 1, 1)


def _out(ctx: Context, n: int) -> GPUTensor:
    return GPUTensor(ctx, 1, max(int(n), 1))


def _ptr(t: GPUTensor | None):
    return C.c_void_p(t.ptr) if t is not None else None


def conv_desc(x_shape, oc, k=3, stride=1, pad=1, up=False, up_hw=None,
              layout=LAYOUT_NCHW) -> ConvDesc:
    n, c, h, w = x_shape
    uh, uw = up_hw if up_hw is not None else ((2 * h, 2 * w) if up else (0, 0))
    return ConvDesc(n, c, h, w, oc, k, stride, pad, int(bool(up)), uh, uw, layout)


def conv_out_shape(d: ConvDesc) -> tuple[int, int]:
    oh, ow = C.c_int(), C.c_int()
    call("yl_conv2d_out_shape", C.byref(d), C.byref(oh), C.byref(ow))
    return oh.value, ow.value


def conv2d_fwd(x, w, b=None, stride=1, pad=1, up=False, up_hw=None, residual=None,
               ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    oc, k = w.shape[0], w.shape[-1]
    d = conv_desc(x.shape, oc, k, stride, pad, up, up_hw)
    oh, ow = conv_out_shape(d)
    xd, wd = _dev(ctx, x), _dev(ctx, w)
    bd = _dev(ctx, b) if b is not None else None
    rd = _dev(ctx, residual) if residual is not None else None
    yd = _out(ctx, x.shape[0] * oc * oh * ow)
    call("yl_conv2d_fwd", ctx.handle, C.byref(d), _ptr(xd), _ptr(wd), _ptr(bd), _ptr(rd), _ptr(yd))
    return yd.toArray().reshape(x.shape[0], oc, oh, ow)


def conv2d_bwd_data(dy, w, x_shape, stride=1, pad=1, up=False, up_hw=None,
                    ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    d = conv_desc(x_shape, w.shape[0], w.shape[-1], stride, pad, up, up_hw)
    dyd, wd = _dev(ctx, dy), _dev(ctx, w)
    dxd = _out(ctx, int(np.prod(x_shape)))
    call("yl_conv2d_bwd_data", ctx.handle, C.byref(d), _ptr(dyd), _ptr(wd), _ptr(dxd))
    return dxd.toArray().reshape(x_shape)


def conv2d_bwd_filter(x, dy, w_shape, stride=1, pad=1, up=False, up_hw=None,
                      ctx: Context | None = None) -> tuple[np.ndarray, np.ndarray]:
    ctx = ctx or Context.shared()
    d = conv_desc(x.shape, w_shape[0], w_shape[-1], stride, pad, up, up_hw)
    xd, dyd = _dev(ctx, x), _dev(ctx, dy)
    dwd, dbd = _out(ctx, int(np.prod(w_shape))), _out(ctx, w_shape[0])
    call("yl_conv2d_bwd_filter", ctx.handle, C.byref(d), _ptr(xd), _ptr(dyd), _ptr(dwd), _ptr(dbd))
    return dwd.toArray().reshape(w_shape), dbd.toArray()[: w_shape[0]]


def groupnorm_silu_fwd(x, groups, eps=1e-6, gamma=None, beta=None, silu=True, mode=0,
                       ctx: Context | None = None):
    ctx = ctx or Context.shared()
    n, c, h, w = x.shape
    xd = _dev(ctx, x)
    gd = _dev(ctx, gamma) if gamma is not None else None
    bd = _dev(ctx, beta) if beta is not None else None
    yd, md, rd = _out(ctx, x.size), _out(ctx, n * groups), _out(ctx, n * groups)
    call("yl_groupnorm_silu_fwd", ctx.handle, _ptr(xd), n, c, h, w, LAYOUT_NCHW, groups,
         float(eps), mode, _ptr(gd), _ptr(bd), int(silu), _ptr(yd), _ptr(md), _ptr(rd))
    return (yd.toArray().reshape(x.shape), md.toArray()[: n * groups],
            rd.toArray()[: n * groups])


def groupnorm_silu_bwd(x, dy, groups, eps=1e-6, gamma=None, beta=None, silu=True, mode=0,
                       addend=None, ctx: Context | None = None):
    ctx = ctx or Context.shared()
    n, c, h, w = x.shape
    xd, dyd = _dev(ctx, x), _dev(ctx, dy)
    gd = _dev(ctx, gamma) if gamma is not None else None
    bd = _dev(ctx, beta) if beta is not None else None
    ad = _dev(ctx, addend) if addend is not None else None
    dxd, dgd, dbd = _out(ctx, x.size), _out(ctx, c), _out(ctx, c)
    call("yl_groupnorm_silu_bwd", ctx.handle, _ptr(xd), _ptr(dyd), n, c, h, w, LAYOUT_NCHW,
         groups, float(eps), mode, _ptr(gd), _ptr(bd), int(silu), None, None, _ptr(ad),
         _ptr(dxd), _ptr(dgd), _ptr(dbd))
    return dxd.toArray().reshape(x.shape), dgd.toArray()[:c], dbd.toArray()[:c]


def linear_fwd(X, W, b=None, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    n, ic = X.shape
    oc = W.shape[0]
    xd, wd = _dev(ctx, X), _dev(ctx, W)
    bd = _dev(ctx, b) if b is not None else None
    yd = _out(ctx, n * oc)
    call("yl_linear_fwd", ctx.handle, _ptr(xd), _ptr(wd), _ptr(bd), _ptr(yd), n, ic, oc)
    return yd.toArray()[: n * oc].reshape(n, oc)


def linear_bwd(X, W, dY, ctx: Context | None = None):
    ctx = ctx or Context.shared()
    n, ic = X.shape
    oc = W.shape[0]
    xd, wd, dyd = _dev(ctx, X), _dev(ctx, W), _dev(ctx, dY)
    dxd, dwd, dbd = _out(ctx, n * ic), _out(ctx, oc * ic), _out(ctx, oc)
    call("yl_linear_bwd", ctx.handle, _ptr(xd), _ptr(wd), _ptr(dyd), _ptr(dxd), _ptr(dwd),
         _ptr(dbd), n, ic, oc)
    return (dxd.toArray()[: n * ic].reshape(n, ic), dwd.toArray()[: oc * ic].reshape(oc, ic),
            dbd.toArray()[:oc])


def timestep_embedding(t, dim=128, variant=0, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    t = np.asarray(t, dtype=np.float32).reshape(-1)
    td = _dev(ctx, t)
    od = _out(ctx, t.size * dim)
    call("yl_timestep_embedding", ctx.handle, _ptr(td), t.size, dim, variant, _ptr(od))
    return od.toArray()[: t.size * dim].reshape(t.size, dim)


def adam_multi(params, grads, ms, vs, lr, t, b1=0.9, b2=0.999, eps=1e-8, grad_scale=1.0,
               clip_max_norm=0.0, sanitize=False, ctx: Context | None = None):
    """Runs one multi-tensor Adam step; returns (params, ms, vs, norm) as numpy."""
    ctx = ctx or Context.shared()
    dev = [[_dev(ctx, a) for a in group] for group in (params, grads, ms, vs)]
    table = (AdamTensor * len(params))()
    for i in range(len(params)):
        table[i] = AdamTensor(dev[0][i].ptr, dev[1][i].ptr, dev[2][i].ptr, dev[3][i].ptr,
                              int(np.asarray(params[i]).size))
    nd = _out(ctx, 1)
    call("yl_adam_multi", ctx.handle, table, len(params), float(lr), float(b1), float(b2),
         float(eps), int(t), float(grad_scale), float(clip_max_norm), int(sanitize), _ptr(nd))
    sizes = [int(np.asarray(p).size) for p in params]
    out = [[d.toArray()[:s] for d, s in zip(dev[k], sizes)] for k in (0, 2, 3)]
    return out[0], out[1], out[2], float(nd.toArray()[0])


def vae_latent_head_fwd(e, step, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    n, c2, h, w = e.shape
    ed = _dev(ctx, e)
    zd = _out(ctx, n * (c2 // 2) * h * w)
    call("yl_vae_latent_head_fwd", ctx.handle, _ptr(ed), n, c2 // 2, h, w, LAYOUT_NCHW,
         int(step), _ptr(zd))
    return zd.toArray().reshape(n, c2 // 2, h, w)


def vae_latent_head_bwd(e, dz, step, beta, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or Context.shared()
    n, c2, h, w = e.shape
    ed, dzd = _dev(ctx, e), _dev(ctx, dz)
    ded = _out(ctx, e.size)
    call("yl_vae_latent_head_bwd", ctx.handle, _ptr(ed), _ptr(dzd), n, c2 // 2, h, w,
         LAYOUT_NCHW, int(step), float(beta), _ptr(ded))
    return ded.toArray().reshape(e.shape)


def loss_l1_kl(recon, target, e=None, beta=1e-6, ctx: Context | None = None):
    ctx = ctx or Context.shared()
    rd, td = _dev(ctx, recon), _dev(ctx, target)
    ed = _dev(ctx, e) if e is not None else None
    gd, ld = _out(ctx, recon.size), _out(ctx, 1)
    if e is not None:
        n, c2, h, w = e.shape
    else:
        n, c2, h, w = 0, 0, 0, 0
    call("yl_loss_l1_kl", ctx.handle, _ptr(rd), _ptr(td), recon.size, _ptr(ed), n, c2 // 2, h, w,
         LAYOUT_NCHW, float(beta), _ptr(gd), _ptr(ld))
    return float(ld.toArray()[0]), gd.toArray()[: recon.size].reshape(recon.shape)


def sobel_edge_loss(recon, target, ctx: Context | None = None):
    """Per-image Sobel edge loss and its gradient for NCHW [n][3][h][w] arrays."""
    ctx = ctx or Context.shared()
    n, c, h, w = recon.shape
    rd, td = _dev(ctx, recon), _dev(ctx, target)
    gd, ld = _out(ctx, recon.size), _out(ctx, n)
    call("yl_sobel_edge_loss", ctx.handle, _ptr(rd), _ptr(td), n, h, w, LAYOUT_NCHW, 0, _ptr(gd),
         _ptr(ld))
    return ld.toArray()[:n], gd.toArray()[: recon.size].reshape(recon.shape)


def layered_loss(recon, target, comp, layer_weight=1.0, compose_weight=1.0,
                 ctx: Context | None = None):
    """Per-image layered 8-channel loss and its gradient (layeredGrad,
    GpuSessionOps.swift:565-585, with the loss of layeredLoss): recon and
    target [n][8][h*w] CHW planes, comp [n][3][h*w]."""
    ctx = ctx or Context.shared()
    n = recon.shape[0]
    plane = recon.size // (8 * n)
    rd, td, cd = _dev(ctx, recon), _dev(ctx, target), _dev(ctx, comp)
    gd, ld = _out(ctx, recon.size), _out(ctx, n)
    call("yl_layered_loss", ctx.handle, _ptr(rd), _ptr(td), _ptr(cd), n, plane,
         float(layer_weight), float(compose_weight), _ptr(gd), _ptr(ld))
    return ld.toArray()[:n], gd.toArray()[: recon.size].reshape(recon.shape)


def layered_compose(recon, ctx: Context | None = None):
    """composeCHW (LayeredVAELoss.swift:95-110) of [n][8][h*w] planes -> [n][3][h*w]."""
    ctx = ctx or Context.shared()
    n = recon.shape[0]
    plane = recon.size // (8 * n)
    rd, od = _dev(ctx, recon), _out(ctx, 3 * n * plane)
    call("yl_layered_compose", ctx.handle, _ptr(rd), n, plane, _ptr(od))
    return od.toArray()[: 3 * n * plane].reshape(n, 3, plane)
