"""Parity at the shapes the benchmark runs, against the oracle.

The reference checks whole conv nets and residual blocks against CPU
arithmetic (Sources/YumeLayersCore/Diagnostics.swift:271-348
checkConvGradients; Tests/YumeLayersTests/TestGroup11.swift:209
testResidualBlockGradients).  These tests do the same at full size:

* the ResNet block of the block benchmark (N=8, C=128, 128x128, GroupNorm 32
  groups, eps 1e-6, SiLU, two 3x3 convs, identity residual), forward and
  backward, every op within 1e-3 relative L2 of the oracle on the same
  inputs, and the chained block within 2e-3;
* one 3x3 128 -> 128 conv at the frame resolution 480x856 through the kernel
  templates the training step runs there (forward and dX on 2 frames; dW and
  db on 8 frames, the step's 3.3 M-pixel split-K contraction);
* the 60-row lattices of the latent level at batch 8 (8-row tiles whose last
  tile row hangs over the image);
* one joint VAE + motion-net step at 480x856, batch 1: both losses within
  1e-3 of the oracle's forward pass from the same weights and frames.

Tolerance: relative L2 <= 1e-3 per op.  The GPU convs multiply tf32
operands (10-bit mantissa, round to nearest) with fp32 accumulation; the
oracle is fp32 throughout.  A 1152-deep tf32 dot product of N(0,1) data
carries ~3e-4 relative error, so 1e-3 leaves 3x headroom.  A chain of four
ops adds the per-op errors in quadrature and gets 2e-3.
"""
import numpy as np
import pytest

from oracle_lib import conv2d_bwd, conv2d_fwd, f32, gn_silu_bwd, gn_silu_fwd, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3
CHAIN_TOL = 2e-3
G, EPS = 32, 1e-6


def kaiming(rng, oc, ic, k):
    b = np.sqrt(6.0 / (ic * k * k))
    return f32(rng.uniform(-b, b, (oc, ic, k, k)))


def gn_affine(rng, c):
    return f32(1 + 0.02 * rng.standard_normal(c)), f32(0.02 * rng.standard_normal(c))


def test_resnet_block_n8_c128_128x128(oracle, ctx):
    """The block benchmark's ResNet block: GN32 -> SiLU -> conv3x3 -> GN32 ->
    SiLU -> conv3x3 + x, forward and backward (dY ~ N(0,1))."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(0)
    n, c, h, w = 8, 128, 128, 128
    x = f32(rng.standard_normal((n, c, h, w)))
    g1, b1 = gn_affine(rng, c)
    g2, b2 = gn_affine(rng, c)
    w1, w2 = kaiming(rng, c, c, 3), kaiming(rng, c, c, 3)
    cb1, cb2 = f32(0.02 * rng.standard_normal(c)), f32(0.02 * rng.standard_normal(c))
    dy = f32(rng.standard_normal((n, c, h, w)))

    # forward, oracle chain
    h1, _, _ = gn_silu_fwd(oracle, x, G, EPS, g1, b1)
    c1 = conv2d_fwd(oracle, h1, w1, cb1)
    h2, _, _ = gn_silu_fwd(oracle, c1, G, EPS, g2, b2)
    y = conv2d_fwd(oracle, h2, w2, cb2, residual=x)
    # forward, per op on the oracle's inputs
    errs = {}
    errs["gn1"] = rel_l2(ops.groupnorm_silu_fwd(x, G, EPS, g1, b1, ctx=ctx)[0], h1)
    errs["conv1"] = rel_l2(ops.conv2d_fwd(h1, w1, cb1, ctx=ctx), c1)
    assert ctx.last_kernel(0) == "conv_tma_fprop_kernel<128, 2, 1, 1>"
    errs["gn2"] = rel_l2(ops.groupnorm_silu_fwd(c1, G, EPS, g2, b2, ctx=ctx)[0], h2)
    errs["conv2+res"] = rel_l2(ops.conv2d_fwd(h2, w2, cb2, residual=x, ctx=ctx), y)

    # backward, oracle chain
    dh2, dw2, db2, _ = conv2d_bwd(oracle, h2, w2, dy)
    dc1, dg2, dbe2 = gn_silu_bwd(oracle, c1, dh2, G, EPS, g2, b2)
    dh1, dw1, db1, _ = conv2d_bwd(oracle, h1, w1, dc1)
    dx, dg1, dbe1 = gn_silu_bwd(oracle, x, dh1, G, EPS, g1, b1, addend=dy)
    # backward, per op on the oracle's inputs
    errs["conv2.dX"] = rel_l2(ops.conv2d_bwd_data(dy, w2, h2.shape, ctx=ctx), dh2)
    gw2, gb2 = ops.conv2d_bwd_filter(h2, dy, w2.shape, ctx=ctx)
    errs["conv2.dW"], errs["conv2.db"] = rel_l2(gw2, dw2), rel_l2(gb2, db2)
    gdc1, gdg2, gdb2 = ops.groupnorm_silu_bwd(c1, dh2, G, EPS, g2, b2, ctx=ctx)
    errs["gn2.dX"], errs["gn2.dgamma"], errs["gn2.dbeta"] = (
        rel_l2(gdc1, dc1), rel_l2(gdg2, dg2), rel_l2(gdb2, dbe2))
    errs["conv1.dX"] = rel_l2(ops.conv2d_bwd_data(dc1, w1, h1.shape, ctx=ctx), dh1)
    gw1, gb1 = ops.conv2d_bwd_filter(h1, dc1, w1.shape, ctx=ctx)
    errs["conv1.dW"], errs["conv1.db"] = rel_l2(gw1, dw1), rel_l2(gb1, db1)
    gdx, gdg1, gdb1 = ops.groupnorm_silu_bwd(x, dh1, G, EPS, g1, b1, addend=dy, ctx=ctx)
    errs["gn1.dX+res"], errs["gn1.dgamma"], errs["gn1.dbeta"] = (
        rel_l2(gdx, dx), rel_l2(gdg1, dg1), rel_l2(gdb1, dbe1))
    bad = {k: v for k, v in errs.items() if not v < TOL}
    assert not bad, f"per-op relative L2 above {TOL}: {bad} (all: {errs})"

    # the chained GPU block against the chained oracle block
    gh1 = ops.groupnorm_silu_fwd(x, G, EPS, g1, b1, ctx=ctx)[0]
    gc1 = ops.conv2d_fwd(gh1, w1, cb1, ctx=ctx)
    gh2 = ops.groupnorm_silu_fwd(gc1, G, EPS, g2, b2, ctx=ctx)[0]
    gy = ops.conv2d_fwd(gh2, w2, cb2, residual=x, ctx=ctx)
    gdh2 = ops.conv2d_bwd_data(dy, w2, h2.shape, ctx=ctx)
    gdc1 = ops.groupnorm_silu_bwd(gc1, gdh2, G, EPS, g2, b2, ctx=ctx)[0]
    gdh1 = ops.conv2d_bwd_data(gdc1, w1, h1.shape, ctx=ctx)
    gdx = ops.groupnorm_silu_bwd(x, gdh1, G, EPS, g1, b1, addend=dy, ctx=ctx)[0]
    assert rel_l2(gy - x, y - x) < CHAIN_TOL
    assert rel_l2(gdx - dy, dx - dy) < CHAIN_TOL


def test_frame_resolution_conv_128ch_480x856(oracle, ctx):
    """3x3, 128 -> 128 at 480x856: forward and dX on 2 frames through the
    halo-box template, dW and db on 8 frames (3.29 M pixels of split-K)."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(1)
    c, h, w = 128, 480, 856
    wt = kaiming(rng, c, c, 3)
    b = f32(0.1 * rng.standard_normal(c))
    x2 = f32(rng.standard_normal((2, c, h, w)))
    y = ops.conv2d_fwd(x2, wt, b, ctx=ctx)
    assert ctx.last_kernel(0) == "conv_tma_fprop_kernel<128, 2, 1, 1>"
    assert rel_l2(y, conv2d_fwd(oracle, x2, wt, b)) < TOL
    dy2 = f32(rng.standard_normal(y.shape))
    dx = ops.conv2d_bwd_data(dy2, wt, x2.shape, ctx=ctx)
    assert ctx.last_kernel(0) == "conv_tma_fprop_kernel<128, 2, 1, 1>"
    dx_ref, _, _, _ = conv2d_bwd(oracle, x2, wt, dy2)
    assert rel_l2(dx, dx_ref) < TOL
    del x2, y, dy2, dx, dx_ref
    x8 = f32(rng.standard_normal((8, c, h, w)))
    dy8 = f32(rng.standard_normal((8, c, h, w)))
    dw, db = ops.conv2d_bwd_filter(x8, dy8, wt.shape, ctx=ctx)
    assert ctx.last_kernel(1) == "conv_tma_wgrad_kernel<1, 2, 192, 32>"
    _, dw_ref, db_ref, _ = conv2d_bwd(oracle, x8, wt, dy8)
    assert rel_l2(dw, dw_ref) < TOL
    assert rel_l2(db, db_ref) < TOL


@pytest.mark.parametrize("c,oc", [(128, 128), (256, 64), (256, 256)])
def test_latent_lattice_60x107_batch8(oracle, ctx, c, oc):
    """The 60 x 107 latent level at the per-GPU batch (the U-Net's first level,
    the VAE's bottleneck convs): 8-row tiles over 60 rows leave a half-empty
    last tile row that the halo boxes and the epilogue must clip."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(2)
    x = f32(rng.standard_normal((8, c, 60, 107)))
    wt = kaiming(rng, oc, c, 3)
    b = f32(0.1 * rng.standard_normal(oc))
    y = ops.conv2d_fwd(x, wt, b, ctx=ctx)
    assert rel_l2(y, conv2d_fwd(oracle, x, wt, b)) < TOL
    dy = f32(rng.standard_normal(y.shape))
    dx_ref, dw_ref, db_ref, _ = conv2d_bwd(oracle, x, wt, dy)
    assert rel_l2(ops.conv2d_bwd_data(dy, wt, x.shape, ctx=ctx), dx_ref) < TOL
    dw, db = ops.conv2d_bwd_filter(x, dy, wt.shape, ctx=ctx)
    assert rel_l2(dw, dw_ref) < TOL
    assert rel_l2(db, db_ref) < TOL


def _oracle_step_losses(js, frames, t, step, beta=1e-6):
    """The oracle's losses of one joint step (forward passes only): L1 + beta*KL
    of the VAE on frame k (latent noise of `step`), and the motion U-Net's MSE
    against the encoder mean of frame k, from frames 0 and 16."""
    from oracle_lib import ptr
    o, vae, unet, c = js.o, js.vae, js.unet, 32
    e0, _ = vae.encode(frames[0])
    e16, _ = vae.encode(frames[1])
    ek, cache = vae.encode(frames[2])
    z, _ = vae.latent(ek, step)
    recon = vae.decode(z, cache)
    n, c2, h, w = ek.shape
    dr = np.empty(recon.size, np.float32)
    lv = o.L.orc_l1_kl_loss(ptr(f32(recon).ravel()), ptr(f32(frames[2]).ravel()), recon.size,
                            ptr(f32(ek[:, :c])), ptr(f32(ek[:, c:])), n * c * h * w, float(beta),
                            ptr(dr))
    pred = unet.predict(f32(e0[:, :c]), f32(e16[:, :c]), t)
    d = pred.astype(np.float64) - ek[:, :c]
    return float(lv), float((d * d).mean())


def test_joint_step_losses_at_480x856():
    """One joint training step at the benchmark's frame size (batch 1) from the
    GPU trainer's own initial weights: VAE and motion losses within 1e-3."""
    import nets
    from yumelayers_b200 import synth
    from yumelayers_b200.trainer import Trainer, default_config
    tr = Trainer(default_config(batch=1, height=480, width=856, seed=4))
    try:
        vp = nets.Params(tr.param_table(0), tr.download(0))
        up = nets.Params(tr.param_table(1), tr.download(1))
        js = nets.JointStep(vp, up, tr.param_count(0), tr.param_count(1))
        clip = synth.make_clip(9, h=480, w=854, width_padded=856)
        frames, t = synth.sample_batch([clip], 1, seed=3)
        gpu = tr.step_host(frames, t)
        cpu = _oracle_step_losses(js, frames, t, step=1)
        rel = [abs(g - c) / abs(c) for g, c in zip(gpu, cpu)]
        assert max(rel) < TOL, f"GPU {list(gpu)} vs oracle {cpu}: rel {rel}"
    finally:
        tr.close()
