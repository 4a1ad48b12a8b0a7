"""CPU restatement of the joint VAE + motion-net training step -- TEST
INFRASTRUCTURE and the timed CPU baseline; never part of the product path.

Every layer is composed from the oracle's restatements of the reference's
kernels (oracle.c): ConvLayerGPU forward/backward (ConvGPU.swift:57-81) as
im2col + GEMM + biasRow / gradW + biasRowGrad + col2im; GroupNorm with the
reference's CPU statistics (LossFunctions.swift:97-176) in affine form +
SiLU; LinearGPU (DenoiserMLP.swift:51-64); motionTimeEmbedding
(MotionPlanner.swift:155-165); the latent head (split2/expHalf/randn/fma,
vae_grad_kernel MetalKernelSourcesB.swift:365-402) with trainingNoiseSeed
(ConvVAEHelpers.swift:33-37); L1 (l1grad_kernel B:453-461) + beta * mean KL
(ConvGPU.swift:435-438); Adam (MetalKernelSourcesA.swift:271-287).  The
network tables are the same as the CUDA executor's (the 854x480 conv VAE and
motion U-Net), read from the trainer's parameter table so the two start
from identical weights.  Layout: NCHW numpy arrays.
"""
from __future__ import annotations

import numpy as np

from oracle_ctypes import (conv2d_bwd, conv2d_fwd, f32, gn_silu_bwd, gn_silu_fwd, load_oracle,
                           ptr)

EPS_GN = 1e-6


def _r4(c: int) -> int:
    return (c + 3) & ~3


class Params:
    """Named parameter arrays built from (and written back to) a flat buffer laid
    out like the CUDA executor's (conv weights [oc][k*k][ic rounded up to 4])."""

    def __init__(self, table, flat: np.ndarray):
        self.table = table
        self.p: dict[str, np.ndarray] = {}
        for e in table:
            self.p[e.name] = self._get(e, flat)

    @staticmethod
    def _get(e, flat):
        d0, d1, d2, d3 = e.shape
        if e.name.endswith(".weight") and d2 >= 1:  # conv (Linear weights have no kernel dims)
            k, icp = d2, _r4(d1)
            blk = flat[e.offset:e.offset + _r4(d0) * k * k * icp].reshape(_r4(d0), k * k, icp)
            return np.ascontiguousarray(
                blk[:d0, :, :d1].transpose(0, 2, 1).reshape(d0, d1, k, k)).astype(np.float32)
        if e.name.endswith(".weight"):  # Linear (oc, ic)
            return flat[e.offset:e.offset + d0 * d1].reshape(d0, d1).astype(np.float32).copy()
        return flat[e.offset:e.offset + d0].astype(np.float32).copy()

    def to_flat(self, values: dict[str, np.ndarray], n: int) -> np.ndarray:
        out = np.zeros(n, np.float32)
        for e in self.table:
            v = values[e.name]
            d0, d1, d2, d3 = e.shape
            if v.ndim == 4:
                k, icp = d2, _r4(d1)
                blk = np.zeros((_r4(d0), k * k, icp), np.float32)
                blk[:d0, :, :d1] = v.reshape(d0, d1, k * k).transpose(0, 2, 1)
                out[e.offset:e.offset + blk.size] = blk.ravel()
            else:
                out[e.offset:e.offset + v.size] = v.ravel()
        return out


class Ops:
    """Thin numpy wrappers around the oracle's C functions."""

    def __init__(self, L=None):
        self.L = L or load_oracle()

    def conv(self, p, name, x, stride=1, pad=1, up=False, up_hw=None, residual=None,
             bias2d=None):
        w = p[name + ".weight"]
        return conv2d_fwd(self.L, x, w, p[name + ".bias"], stride, pad, up, up_hw,
                          bias2d=bias2d, residual=residual)

    def conv_bwd(self, p, g, name, x, dy, stride=1, pad=1, up=False, up_hw=None,
                 need_dx=True):
        w = p[name + ".weight"]
        dx, dw, db, dbi = conv2d_bwd(self.L, x, w, dy, stride, pad, up, up_hw)
        g[name + ".weight"] = dw
        g[name + ".bias"] = db
        return (dx if need_dx else None), dbi

    def gn(self, p, name, x):
        y, m, r = gn_silu_fwd(self.L, x, 32, EPS_GN, p[name + ".gamma"], p[name + ".beta"])
        return y

    def gn_bwd(self, p, g, name, x, dy, addend=None):
        dx, dg, db = gn_silu_bwd(self.L, x, dy, 32, EPS_GN, p[name + ".gamma"],
                                 p[name + ".beta"], addend=addend)
        g[name + ".gamma"] = dg
        g[name + ".beta"] = db
        return dx

    def linear(self, p, name, x):
        W, b = p[name + ".weight"], p[name + ".bias"]
        n, ic = x.shape
        y = np.zeros((n, W.shape[0]), np.float32)
        self.L.orc_linear_fwd(ptr(f32(x)), ptr(W), ptr(b), ptr(y), n, ic, W.shape[0], 0)
        return y

    def linear_bwd(self, p, g, name, x, dy):
        W = p[name + ".weight"]
        n, ic = x.shape
        dx = np.zeros_like(x, dtype=np.float32)
        dw = np.zeros_like(W)
        db = np.zeros(W.shape[0], np.float32)
        self.L.orc_linear_bwd(ptr(f32(x)), ptr(W), ptr(f32(dy)), ptr(dx), ptr(dw), ptr(db), n,
                              ic, W.shape[0])
        g[name + ".weight"] = dw
        g[name + ".bias"] = db
        return dx

    def silu(self, x):
        x = f32(x)
        y = np.zeros_like(x)
        self.L.orc_unary(6, ptr(x), ptr(y), x.size)
        return y

    def silu_bwd(self, x, dy):
        x, dy = f32(x), f32(dy)
        out = np.zeros_like(x)
        self.L.orc_binary(5, ptr(x), ptr(dy), ptr(out), x.size)
        return out


# ------------------------------------------------------------------ blocks
def rb_fwd(o, p, name, x, cin, cout, proj=None):
    c = {}
    c["h1"] = o.gn(p, name + ".norm1", x)
    c["c1"] = o.conv(p, name + ".conv1", c["h1"], bias2d=proj)
    c["h2"] = o.gn(p, name + ".norm2", c["c1"])
    res = o.conv(p, name + ".skip", x, pad=0) if cin != cout else x
    c["y"] = o.conv(p, name + ".conv2", c["h2"], residual=res)
    return c["y"], c


def rb_bwd(o, p, g, name, x, c, dy, cin, cout):
    dh2, _ = o.conv_bwd(p, g, name + ".conv2", c["h2"], dy)
    dc1 = o.gn_bwd(p, g, name + ".norm2", c["c1"], dh2)
    dh1, dproj = o.conv_bwd(p, g, name + ".conv1", c["h1"], dc1)
    if cin != cout:
        dxs, _ = o.conv_bwd(p, g, name + ".skip", x, dy, pad=0)
    else:
        dxs = dy
    dx = o.gn_bwd(p, g, name + ".norm1", x, dh1, addend=dxs)
    return dx, dproj


def noise_seed(L, step: int, img: int) -> int:
    return L.orc_training_noise_seed(step, img)


class VAE:
    """The 854x480-frame conv VAE (same layer table as the CUDA executor)."""
    ENC = [("enc.rb1a", 128, 128), ("enc.rb1b", 128, 128), ("enc.down1", 128, 128),
           ("enc.rb2a", 128, 256), ("enc.rb2b", 256, 256), ("enc.down2", 256, 256),
           ("enc.rb3a", 256, 256), ("enc.rb3b", 256, 256), ("enc.down3", 256, 256)]
    DEC = [("dec.up1", 256, 256), ("dec.rb1a", 256, 256), ("dec.rb1b", 256, 256),
           ("dec.up2", 256, 256), ("dec.rb2a", 256, 256), ("dec.rb2b", 256, 256),
           ("dec.up3", 256, 128), ("dec.rb3a", 128, 128), ("dec.rb3b", 128, 128)]

    def __init__(self, ops: Ops, params: Params):
        self.o, self.P = ops, params

    def encode(self, x):
        o, p = self.o, self.P.p
        cache = {"x": x}
        h = o.conv(p, "enc.conv_in", x)
        cache["a0"] = h
        for name, cin, cout in self.ENC:
            if "down" in name:
                cache[name + ".in"] = h
                h = o.conv(p, name, h, stride=2)
            else:
                cache[name + ".in"] = h
                h, cache[name] = rb_fwd(o, p, name, h, cin, cout)
        cache["a3"] = h
        cache["hg"] = o.gn(p, "enc.norm_out", h)
        e = o.conv(p, "enc.conv_out", cache["hg"])
        cache["e"] = e
        return e, cache

    def decode(self, z, cache):
        o, p = self.o, self.P.p
        cache["z"] = z
        h = o.conv(p, "dec.conv_in", z)
        for name, cin, cout in self.DEC:
            cache[name + ".in"] = h
            if "up" in name:
                hh, ww = 2 * h.shape[2], 2 * h.shape[3]
                h = o.conv(p, name, h, up=True, up_hw=(hh, ww))
            else:
                h, cache[name] = rb_fwd(o, p, name, h, cin, cout)
        cache["d3"] = h
        cache["hd"] = o.gn(p, "dec.norm_out", h)
        return o.conv(p, "dec.conv_out", cache["hd"])

    def latent(self, e, step):
        n, c2, h, w = e.shape
        c = c2 // 2
        mu, lv = e[:, :c], np.clip(e[:, c:], -10, 10)
        eps = np.zeros((n, c * h * w), np.float32)
        for img in range(n):
            self.o.L.orc_randn(ptr(eps[img]), noise_seed(self.o.L, step, img), c * h * w)
        eps = eps.reshape(n, c, h, w)
        return (mu + np.exp(0.5 * lv) * eps).astype(np.float32), eps

    def train_forward_backward(self, x, step, beta):
        """Returns (loss, grads dict, e) for one VAE step on frames x (n,3,H,W)."""
        o, p = self.o, self.P.p
        e, cache = self.encode(x)
        z, eps = self.latent(e, step)
        recon = self.decode(z, cache)
        n, c2, h, w = e.shape
        c = c2 // 2
        dr = np.zeros(recon.size, np.float32)
        loss = o.L.orc_l1_kl_loss(ptr(f32(recon).ravel()), ptr(f32(x).ravel()), recon.size,
                                  ptr(f32(e[:, :c])), ptr(f32(e[:, c:])), n * c * h * w,
                                  float(beta), ptr(dr))
        g = {}
        dy, _ = o.conv_bwd(p, g, "dec.conv_out", cache["hd"], dr.reshape(recon.shape))
        dy = o.gn_bwd(p, g, "dec.norm_out", cache["d3"], dy)
        for name, cin, cout in reversed(self.DEC):
            xin = cache[name + ".in"]
            if "up" in name:
                dy, _ = o.conv_bwd(p, g, name, xin, dy, up=True,
                                   up_hw=(2 * xin.shape[2], 2 * xin.shape[3]))
            else:
                dy, _ = rb_bwd(o, p, g, name, xin, cache[name], dy, cin, cout)
        dz, _ = o.conv_bwd(p, g, "dec.conv_in", cache["z"], dy)
        M = n * c * h * w
        dmu = np.zeros(M, np.float32)
        dlv = np.zeros(M, np.float32)
        o.L.orc_vae_grad(ptr(f32(dz)), ptr(f32(e[:, :c])), ptr(f32(e[:, c:])), ptr(f32(eps)),
                         ptr(dmu), ptr(dlv), np.float32(beta / M), np.float32(0.5 * beta / M), M)
        de = np.concatenate([dmu.reshape(n, c, h, w), dlv.reshape(n, c, h, w)], axis=1)
        dy, _ = o.conv_bwd(p, g, "enc.conv_out", cache["hg"], de)
        dy = o.gn_bwd(p, g, "enc.norm_out", cache["a3"], dy)
        for name, cin, cout in reversed(self.ENC):
            xin = cache[name + ".in"]
            if "down" in name:
                dy, _ = o.conv_bwd(p, g, name, xin, dy, stride=2)
            else:
                dy, _ = rb_bwd(o, p, g, name, xin, cache[name], dy, cin, cout)
        o.conv_bwd(p, g, "enc.conv_in", x, dy, need_dx=False)
        return float(loss), g, e


class UNet:
    """The latent-space motion U-Net (same table as the CUDA executor)."""
    BLOCKS = ["down1.rb_a", "down1.rb_b", "down2.rb_a", "down2.rb_b", "mid.rb_a", "mid.rb_b",
              "up1.rb_a", "up1.rb_b", "up2.rb_a", "up2.rb_b"]
    CH = {"down1.rb_a": (128, 128), "down1.rb_b": (128, 128), "down2.rb_a": (128, 256),
          "down2.rb_b": (256, 256), "mid.rb_a": (256, 384), "mid.rb_b": (384, 384),
          "up1.rb_a": (512, 256), "up1.rb_b": (256, 256), "up2.rb_a": (256, 128),
          "up2.rb_b": (128, 128)}

    def __init__(self, ops: Ops, params: Params):
        self.o, self.P = ops, params

    def predict(self, za, zb, t):
        """Forward only: the predicted intermediate latent for (zA, zB, t)."""
        return self._forward(za, zb, t)[0]

    def _forward(self, za, zb, t):
        o, p = self.o, self.P.p
        n, c, h, w = za.shape
        tt = t.reshape(n, 1, 1, 1)
        lerp = ((1 - tt) * za + tt * zb).astype(np.float32)
        inp = np.concatenate([za, zb, lerp], axis=1).astype(np.float32)
        emb = np.zeros((n, 128), np.float32)
        for i in range(n):
            o.L.orc_motion_time_embedding(float(t[i]), 128, ptr(emb[i]))
        th = o.linear(p, "time.fc1", emb)
        ta = o.silu(th)
        temb = o.linear(p, "time.fc2", ta)
        ts = o.silu(temb)
        pj = {b: o.linear(p, b + ".temb_proj", ts) for b in self.BLOCKS}
        C = {}
        h0 = o.conv(p, "conv_in", inp)
        r1a, C["down1.rb_a"] = rb_fwd(o, p, "down1.rb_a", h0, 128, 128, pj["down1.rb_a"])
        s1, C["down1.rb_b"] = rb_fwd(o, p, "down1.rb_b", r1a, 128, 128, pj["down1.rb_b"])
        p1 = o.conv(p, "down1.conv", s1, stride=2)
        r2a, C["down2.rb_a"] = rb_fwd(o, p, "down2.rb_a", p1, 128, 256, pj["down2.rb_a"])
        s2, C["down2.rb_b"] = rb_fwd(o, p, "down2.rb_b", r2a, 256, 256, pj["down2.rb_b"])
        p2 = o.conv(p, "down2.conv", s2, stride=2)
        r3a, C["mid.rb_a"] = rb_fwd(o, p, "mid.rb_a", p2, 256, 384, pj["mid.rb_a"])
        r3b, C["mid.rb_b"] = rb_fwd(o, p, "mid.rb_b", r3a, 384, 384, pj["mid.rb_b"])
        u1 = o.conv(p, "up1.conv", r3b, up=True, up_hw=s2.shape[2:])
        cat1 = np.concatenate([u1, s2], axis=1)
        r4a, C["up1.rb_a"] = rb_fwd(o, p, "up1.rb_a", cat1, 512, 256, pj["up1.rb_a"])
        r4b, C["up1.rb_b"] = rb_fwd(o, p, "up1.rb_b", r4a, 256, 256, pj["up1.rb_b"])
        u2 = o.conv(p, "up2.conv", r4b, up=True, up_hw=s1.shape[2:])
        cat2 = np.concatenate([u2, s1], axis=1)
        r5a, C["up2.rb_a"] = rb_fwd(o, p, "up2.rb_a", cat2, 256, 128, pj["up2.rb_a"])
        r5b, C["up2.rb_b"] = rb_fwd(o, p, "up2.rb_b", r5a, 128, 128, pj["up2.rb_b"])
        ho = o.gn(p, "norm_out", r5b)
        pred = o.conv(p, "conv_out", ho, residual=lerp)
        return pred, (inp, emb, th, ta, temb, ts, pj, C, h0, r1a, s1, p1, r2a, s2, p2, r3a, r3b,
                      u1, cat1, r4a, r4b, u2, cat2, r5a, r5b, ho)

    def train_forward_backward(self, za, zb, t, target):
        o, p = self.o, self.P.p
        pred, (inp, emb, th, ta, temb, ts, pj, C, h0, r1a, s1, p1, r2a, s2, p2, r3a, r3b, u1, cat1,
               r4a, r4b, u2, cat2, r5a, r5b, ho) = self._forward(za, zb, t)
        d = (pred.astype(np.float64) - target)
        loss = float((d * d).mean())
        dpred = (2.0 * d / d.size).astype(np.float32)
        g = {}
        dproj = {}
        dy, _ = o.conv_bwd(p, g, "conv_out", ho, dpred)
        dy = o.gn_bwd(p, g, "norm_out", r5b, dy)
        dy, dproj["up2.rb_b"] = rb_bwd(o, p, g, "up2.rb_b", r5a, C["up2.rb_b"], dy, 128, 128)
        dcat2, dproj["up2.rb_a"] = rb_bwd(o, p, g, "up2.rb_a", cat2, C["up2.rb_a"], dy, 256, 128)
        dy, _ = o.conv_bwd(p, g, "up2.conv", r4b, np.ascontiguousarray(dcat2[:, :128]), up=True,
                           up_hw=s1.shape[2:])
        dy, dproj["up1.rb_b"] = rb_bwd(o, p, g, "up1.rb_b", r4a, C["up1.rb_b"], dy, 256, 256)
        dcat1, dproj["up1.rb_a"] = rb_bwd(o, p, g, "up1.rb_a", cat1, C["up1.rb_a"], dy, 512, 256)
        dy, _ = o.conv_bwd(p, g, "up1.conv", r3b, np.ascontiguousarray(dcat1[:, :256]), up=True,
                           up_hw=s2.shape[2:])
        dy, dproj["mid.rb_b"] = rb_bwd(o, p, g, "mid.rb_b", r3a, C["mid.rb_b"], dy, 384, 384)
        dy, dproj["mid.rb_a"] = rb_bwd(o, p, g, "mid.rb_a", p2, C["mid.rb_a"], dy, 256, 384)
        dy, _ = o.conv_bwd(p, g, "down2.conv", s2, dy, stride=2)
        dy = dy + dcat1[:, 256:]
        dy, dproj["down2.rb_b"] = rb_bwd(o, p, g, "down2.rb_b", r2a, C["down2.rb_b"], dy, 256, 256)
        dy, dproj["down2.rb_a"] = rb_bwd(o, p, g, "down2.rb_a", p1, C["down2.rb_a"], dy, 128, 256)
        dy, _ = o.conv_bwd(p, g, "down1.conv", s1, dy, stride=2)
        dy = dy + dcat2[:, 128:]
        dy, dproj["down1.rb_b"] = rb_bwd(o, p, g, "down1.rb_b", r1a, C["down1.rb_b"], dy, 128, 128)
        dy, dproj["down1.rb_a"] = rb_bwd(o, p, g, "down1.rb_a", h0, C["down1.rb_a"], dy, 128, 128)
        o.conv_bwd(p, g, "conv_in", inp, dy, need_dx=False)
        dts = np.zeros_like(ts)
        for b in self.BLOCKS:
            dts += o.linear_bwd(p, g, b + ".temb_proj", ts, dproj[b])
        dtemb = o.silu_bwd(temb, dts)
        dta = o.linear_bwd(p, g, "time.fc2", ta, dtemb)
        dth = o.silu_bwd(th, dta)
        o.linear_bwd(p, g, "time.fc1", emb, dth)
        return loss, g


class JointStep:
    """One rank of the joint step, mirroring yl_trainer_step."""

    def __init__(self, vae_params: Params, unet_params: Params, n_vae: int, n_unet: int,
                 lr_vae=2e-4, lr_motion=2e-4, beta=1e-6, ops: Ops | None = None):
        self.o = ops or Ops()
        self.vp, self.up = vae_params, unet_params
        self.vae = VAE(self.o, vae_params)
        self.unet = UNet(self.o, unet_params)
        self.n_vae, self.n_unet = n_vae, n_unet
        self.lr_vae, self.lr_motion, self.beta = lr_vae, lr_motion, beta
        self.flat = {0: vae_params.to_flat(vae_params.p, n_vae),
                     1: unet_params.to_flat(unet_params.p, n_unet)}
        self.m = {k: np.zeros_like(v) for k, v in self.flat.items()}
        self.v = {k: np.zeros_like(v) for k, v in self.flat.items()}
        self.step_no = 0

    def step(self, frames: np.ndarray, t: np.ndarray) -> tuple[float, float]:
        """frames [3][n][3][H][W] (frame 0, 16, k), t [n] -> (VAE loss, motion loss)."""
        self.step_no += 1
        c = 32
        e0, _ = self.vae.encode(frames[0])
        e16, _ = self.vae.encode(frames[1])
        lv, gv, ek = self.vae.train_forward_backward(frames[2], self.step_no, self.beta)
        lm, gm = self.unet.train_forward_backward(e0[:, :c], e16[:, :c], t, ek[:, :c])
        for which, (P, grads, lr) in enumerate([(self.vp, gv, self.lr_vae),
                                                (self.up, gm, self.lr_motion)]):
            gflat = P.to_flat(grads, self.flat[which].size)
            n = self.flat[which].size
            self.o.L.orc_adam(ptr(self.flat[which]), ptr(gflat), ptr(self.m[which]),
                              ptr(self.v[which]), n, self.step_no, lr, 0.9, 0.999, 1e-8)
            fresh = Params(P.table, self.flat[which])
            P.p.update(fresh.p)
        return lv, lm


# ------------------------------------------------------------------ standalone tables
class _Entry:
    def __init__(self, name, offset, shape):
        self.name, self.offset, self.shape = name, offset, shape


def _builder():
    tab, off = [], [0]

    def res(n):
        o = off[0]
        off[0] += (n + 3) & ~3
        return o

    def conv(name, cin, cout, k=3):
        tab.append(_Entry(name + ".weight", res(_r4(cout) * k * k * _r4(cin)), (cout, cin, k, k)))
        tab.append(_Entry(name + ".bias", res(_r4(cout)), (cout, 1, 1, 1)))

    def gn(name, c):
        tab.append(_Entry(name + ".gamma", res(c), (c, 1, 1, 1)))
        tab.append(_Entry(name + ".beta", res(c), (c, 1, 1, 1)))

    def lin(name, ic, oc):
        tab.append(_Entry(name + ".weight", res(oc * ic), (oc, ic, 0, 0)))
        tab.append(_Entry(name + ".bias", res(oc), (oc, 1, 1, 1)))

    def rb(name, cin, cout):
        gn(name + ".norm1", cin)
        conv(name + ".conv1", cin, cout)
        gn(name + ".norm2", cout)
        conv(name + ".conv2", cout, cout)
        if cin != cout:
            conv(name + ".skip", cin, cout, 1)

    return tab, off, conv, gn, lin, rb


def vae_table():
    """Parameter table in the executor's registration order (yl_nets.cu VAE::build)."""
    tab, off, conv, gn, lin, rb = _builder()
    conv("enc.conv_in", 3, 128)
    for n, ci, co in VAE.ENC:
        conv(n, ci, co) if "down" in n else rb(n, ci, co)
    gn("enc.norm_out", 256)
    conv("enc.conv_out", 256, 64)
    conv("dec.conv_in", 32, 256)
    for n, ci, co in VAE.DEC:
        conv(n, ci, co) if "up" in n else rb(n, ci, co)
    gn("dec.norm_out", 128)
    conv("dec.conv_out", 128, 3)
    return tab, off[0]


def unet_table():
    """Parameter table in the executor's registration order (yl_nets.cu UNet::build)."""
    tab, off, conv, gn, lin, rb = _builder()
    lin("time.fc1", 128, 512)
    lin("time.fc2", 512, 512)
    for b in UNet.BLOCKS:
        lin(b + ".temb_proj", 512, UNet.CH[b][1])
    conv("conv_in", 96, 128)
    order = [("down1.rb_a",), ("down1.rb_b",), ("down1.conv", 128, 128), ("down2.rb_a",),
             ("down2.rb_b",), ("down2.conv", 256, 256), ("mid.rb_a",), ("mid.rb_b",),
             ("up1.conv", 384, 256), ("up1.rb_a",), ("up1.rb_b",), ("up2.conv", 256, 128),
             ("up2.rb_a",), ("up2.rb_b",)]
    for item in order:
        if len(item) == 1:
            rb(item[0], *UNet.CH[item[0]])
        else:
            conv(*item)
    gn("norm_out", 128)
    conv("conv_out", 128, 32)
    return tab, off[0]


def init_flat(table, count, seed, zero=("conv_out",)):
    """Seeded init with the executor's distributions: Kaiming-uniform convs,
    U(+-1/sqrt(ic)) Linear, GN gamma = 1 + 0.02 N, beta = 0.02 N, zero biases,
    zero-initialised motion output conv (its prediction starts at the lerp)."""
    rng = np.random.default_rng(seed)
    vals = {}
    for e in table:
        d0, d1, d2, d3 = e.shape
        if e.name.endswith(".gamma"):
            vals[e.name] = (1 + 0.02 * rng.standard_normal(d0)).astype(np.float32)
        elif e.name.endswith(".beta"):
            vals[e.name] = (0.02 * rng.standard_normal(d0)).astype(np.float32)
        elif e.name.endswith(".bias"):
            vals[e.name] = np.zeros(d0, np.float32)
        elif d2 >= 1:  # conv weight (Linear weights have no kernel dims)
            bound = np.sqrt(6.0 / (d1 * d2 * d3))
            if e.name.startswith(zero):
                bound = 0.0
            vals[e.name] = rng.uniform(-bound, bound, (d0, d1, d2, d3)).astype(np.float32)
        else:
            b = 1.0 / np.sqrt(d1)
            vals[e.name] = rng.uniform(-b, b, (d0, d1)).astype(np.float32)
    p = Params.__new__(Params)
    p.table = table
    p.p = vals
    return p.to_flat(vals, count)


def standalone_joint_step(seed=0, ops: Ops | None = None) -> JointStep:
    """A JointStep with its own seeded weights (no GPU involved)."""
    vt, nv = vae_table()
    ut, nu = unet_table()
    vp = Params(vt, init_flat(vt, nv, seed))
    up = Params(ut, init_flat(ut, nu, seed + 1))
    return JointStep(vp, up, nv, nu, ops=ops)
