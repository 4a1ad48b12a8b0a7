"""Fused GroupNorm+SiLU, multi-tensor Adam, Linear, timestep embedding and the
VAE heads on the GPU against the oracle (and, for the embedding, the golden
vectors generated from the reference's PyTorch prototype)."""
import math
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import f32, gn_silu_bwd, gn_silu_fwd, ptr, rel_l2

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("shape,G", [((2, 16, 5, 7), 4), ((2, 128, 24, 20), 32),
                                     ((1, 256, 30, 54), 32), ((1, 384, 15, 27), 32),
                                     ((1, 512, 9, 11), 32)])
def test_groupnorm_silu_forward_backward(oracle, shape, G):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(0)
    x = f32(rng.standard_normal(shape) * 1.5 + 0.3)
    c = shape[1]
    ga = f32(1 + 0.02 * rng.standard_normal(c))
    be = f32(0.02 * rng.standard_normal(c))
    y_ref, m_ref, r_ref = gn_silu_fwd(oracle, x, G, 1e-6, ga, be)
    y, m, r = ops.groupnorm_silu_fwd(x, G, 1e-6, ga, be)
    assert rel_l2(y, y_ref) < 1e-5
    assert rel_l2(m, m_ref) < 1e-5 and rel_l2(r, r_ref) < 1e-5
    dy = f32(rng.standard_normal(shape))
    add = f32(rng.standard_normal(shape))
    dx_ref, dg_ref, db_ref = gn_silu_bwd(oracle, x, dy, G, 1e-6, ga, be, addend=add)
    dx, dg, db = ops.groupnorm_silu_bwd(x, dy, G, 1e-6, ga, be, addend=add)
    assert rel_l2(dx, dx_ref) < 1e-5
    assert rel_l2(dg, dg_ref) < 1e-4 and rel_l2(db, db_ref) < 1e-4


def test_groupnorm_reference_variance_rule(oracle):
    """mode 1 = groupnorm_kernel's clamp (var >= 1e-5, no eps, no affine)."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(1)
    x = f32(rng.uniform(-2, 2, (1, 8, 4, 8)))
    x[0, :4] = 0.25  # a constant group: variance 0 -> clamped
    y, _, _ = ops.groupnorm_silu_fwd(x, 2, 0.0, silu=False, mode=1)
    ref = np.zeros(x.size, np.float32)
    oracle.orc_groupnorm_ref(ptr(x.reshape(-1)), ptr(ref), 8, 2, 32)
    assert np.abs(y.reshape(-1) - ref).max() < 1e-4


def test_adam_multi_matches_oracle(oracle):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(2)
    sizes = [1000, 3, 4097, 128 * 1152]
    ps = [f32(rng.standard_normal(s)) for s in sizes]
    gs = [f32(rng.standard_normal(s) * 0.1) for s in sizes]
    ms = [f32(rng.standard_normal(s) * 0.01) for s in sizes]
    vs = [f32(np.abs(rng.standard_normal(s)) * 0.001) for s in sizes]
    p2, m2, v2, _ = ops.adam_multi(ps, gs, ms, vs, lr=2e-4, t=7)
    for i in range(len(sizes)):
        p, m, v = ps[i].copy(), ms[i].copy(), vs[i].copy()
        oracle.orc_adam(ptr(p), ptr(gs[i]), ptr(m), ptr(v), p.size, 7, 2e-4, 0.9, 0.999, 1e-8)
        assert np.abs(p2[i] - p).max() < 1e-6
        assert rel_l2(m2[i], m) < 1e-6 and rel_l2(v2[i], v) < 1e-6


def test_adam_multi_sanitize_and_clip(oracle):
    """GradSanitize.swift:18-101 semantics folded into the Adam launch."""
    import ctypes as C
    from yumelayers_b200 import ops
    rng = np.random.default_rng(3)
    g = f32(rng.standard_normal(5000) * 3)
    g[10], g[20] = np.nan, np.inf
    p = f32(rng.standard_normal(5000))
    z = np.zeros(5000, np.float32)
    p2, _, _, norm = ops.adam_multi([p], [g], [z], [z], lr=1e-3, t=1, grad_scale=0.125,
                                    clip_max_norm=1.0, sanitize=True)
    gs = g.copy()
    fixed = C.c_long()
    ref_norm = oracle.orc_sanitize_grads(ptr(gs), gs.size, 1.0, 0.125, C.byref(fixed))
    assert fixed.value == 2 and abs(norm - ref_norm) / ref_norm < 1e-5
    pr, m, v = p.copy(), np.zeros_like(p), np.zeros_like(p)
    oracle.orc_adam(ptr(pr), ptr(gs), ptr(m), ptr(v), p.size, 1, 1e-3, 0.9, 0.999, 1e-8)
    assert np.isfinite(p2[0]).all() and np.abs(p2[0] - pr).max() < 1e-5


def test_linear(oracle):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(4)
    n, ic, oc = 32, 128, 512
    X, W, b = f32(rng.standard_normal((n, ic))), f32(rng.standard_normal((oc, ic)) * 0.1), f32(
        rng.standard_normal(oc))
    Y = ops.linear_fwd(X, W, b)
    Yr = np.zeros((n, oc), np.float32)
    oracle.orc_linear_fwd(ptr(X), ptr(W), ptr(b), ptr(Yr), n, ic, oc, 0)
    assert rel_l2(Y, Yr) < 1e-5
    dY = f32(rng.standard_normal((n, oc)))
    dX, dW, db = ops.linear_bwd(X, W, dY)
    rX, rW, rb = np.zeros_like(X), np.zeros_like(W), np.zeros_like(b)
    oracle.orc_linear_bwd(ptr(X), ptr(W), ptr(dY), ptr(rX), ptr(rW), ptr(rb), n, ic, oc)
    assert rel_l2(dX, rX) < 1e-5 and rel_l2(dW, rW) < 1e-5 and rel_l2(db, rb) < 1e-5


def test_timestep_embeddings(oracle):
    from yumelayers_b200 import ops
    t = f32([0.0, 0.125, 0.5, 0.99, 1.0, 3.0, -1.0])
    e = ops.timestep_embedding(t, 128, variant=0)
    for i, tv in enumerate(t):
        ref = np.zeros(128, np.float32)
        oracle.orc_motion_time_embedding(float(tv), 128, ptr(ref))
        assert np.abs(e[i] - ref).max() < 1e-6
    g = np.load(GOLDEN / "prototype_golden.npz")
    e1 = ops.timestep_embedding(g["temb_t"], 128, variant=1)
    assert np.abs(e1 - g["temb_out"]).max() < 1e-3  # fp32 args up to 1000 rad


def test_latent_head_and_loss(oracle):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(5)
    n, c, h, w = 2, 32, 6, 9
    e = f32(rng.standard_normal((n, 2 * c, h, w)))
    e[0, c:c + 2] = 15.0  # logvar clamp range
    step = 11
    z = ops.vae_latent_head_fwd(e, step)
    eps = np.zeros((n, c * h * w), np.float32)
    for img in range(n):
        seed = oracle.orc_training_noise_seed(step, img)
        oracle.orc_randn(ptr(eps[img]), seed, c * h * w)
    eps = eps.reshape(n, c, h, w)
    mu, lv = e[:, :c], np.clip(e[:, c:], -10, 10)
    assert rel_l2(z, mu + np.exp(0.5 * lv) * eps) < 1e-5
    dz = f32(rng.standard_normal((n, c, h, w)))
    beta = 1e-2
    de = ops.vae_latent_head_bwd(e, dz, step, beta)
    M = n * c * h * w
    dmu, dlv = np.zeros(M, np.float32), np.zeros(M, np.float32)
    oracle.orc_vae_grad(ptr(f32(dz)), ptr(f32(e[:, :c])), ptr(f32(e[:, c:])), ptr(f32(eps)),
                        ptr(dmu), ptr(dlv), beta / M, 0.5 * beta / M, M)
    assert rel_l2(de[:, :c], dmu.reshape(n, c, h, w)) < 1e-3
    assert rel_l2(de[:, c:], dlv.reshape(n, c, h, w)) < 1e-3
    recon = f32(rng.standard_normal((n, 3, 16, 24)))
    target = f32(rng.standard_normal((n, 3, 16, 24)))
    loss, dr = ops.loss_l1_kl(recon, target, e, beta)
    dr_ref = np.zeros(recon.size, np.float32)
    ref_loss = oracle.orc_l1_kl_loss(ptr(recon.reshape(-1)), ptr(target.reshape(-1)), recon.size,
                                     ptr(f32(e[:, :c])), ptr(f32(e[:, c:])), M, beta, ptr(dr_ref))
    assert abs(loss - ref_loss) / abs(ref_loss) < 1e-5
    assert np.array_equal(dr.reshape(-1), dr_ref)
