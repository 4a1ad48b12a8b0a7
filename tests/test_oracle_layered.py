"""Layered 8-channel loss in the oracle against the reference's own checks
(TestGroup6.swift:312-393, testLayeredLossMath): exact composition, zero loss
for a perfect reconstruction, finite differences of the analytic gradient on
the 4x4 known-answer case, and the composition term reaching the background,
mask and light gradients.  A float64 numpy restatement of the same formulas
(LayeredVAELoss.swift:95-196) is a second, independent check."""
import numpy as np

from oracle_lib import f32, ptr


def _compose_np(recon, n):
    r = recon.reshape(8, n).astype(np.float32)
    m, l = r[6], r[7]
    v = (r[0:3] * (np.float32(1) - m) + r[3:6] * m) * l
    return np.clip(v, 0, 1).astype(np.float32).reshape(-1)


def _loss_np(recon, target, comp, n, wl=1.0, wc=1.0):
    # differences in float, squares and sums in double (LayeredVAELoss.swift:133-145)
    layer = np.mean(((recon - target).astype(np.float64)) ** 2)
    y = _compose_np(recon, n)
    compose = np.mean(((y - comp).astype(np.float64)) ** 2)
    return float(np.float32(wl)) * layer + float(np.float32(wc)) * compose


def _oracle_grad(oracle, recon, target, comp, n, wl=1.0, wc=1.0):
    g = np.zeros(8 * n, np.float32)
    oracle.orc_layered_grad(ptr(recon), ptr(target), ptr(comp), n, wl, wc, ptr(g))
    return g


def _scene(rng, n):
    """8 target planes in [0, 1] and the frame they compose to."""
    t = f32(rng.uniform(0, 1, 8 * n))
    return t, _compose_np(t, n)


def test_compose_and_zero_loss(oracle):
    n = 32 * 32
    rng = np.random.default_rng(2026)
    target, comp = _scene(rng, n)
    got = np.zeros(3 * n, np.float32)
    oracle.orc_layered_compose(ptr(target), n, ptr(got))
    np.testing.assert_array_equal(got, comp)
    assert oracle.orc_layered_loss(ptr(target), ptr(target), ptr(comp), n, 1.0, 1.0) == 0.0
    bad = f32(np.clip(target + 0.05, 0, 1))
    lb = oracle.orc_layered_loss(ptr(bad), ptr(target), ptr(comp), n, 1.0, 1.0)
    assert lb > 0
    np.testing.assert_allclose(lb, _loss_np(bad, target, comp, n), rtol=1e-12)


def test_gradient_finite_differences_known_case(oracle):
    """The reference's 4x4 case: channels 0.25 + 0.03*(idx/n) + 0.01*(idx%n),
    composite 0.42, recon 0.30 + 0.02*(i%7); central differences with eps 1e-3
    at pixels 0, 5, 11 of every channel within 5% (TestGroup6.swift:338-372)."""
    n = 16
    idx = np.arange(8 * n)
    target = f32(0.25 + 0.03 * (idx // n) + 0.01 * (idx % n))
    comp = f32(np.full(3 * n, 0.42))
    recon = f32(0.30 + 0.02 * (idx % 7))
    g = _oracle_grad(oracle, recon, target, comp, n)
    eps = np.float32(1e-3)
    worst = 0.0
    for ch in range(8):
        for i in (0, 5, 11):
            k = ch * n + i
            rp, rm = recon.copy(), recon.copy()
            rp[k] += eps
            rm[k] -= eps
            lp = oracle.orc_layered_loss(ptr(rp), ptr(target), ptr(comp), n, 1.0, 1.0)
            lm = oracle.orc_layered_loss(ptr(rm), ptr(target), ptr(comp), n, 1.0, 1.0)
            num = (lp - lm) / (2 * float(eps))
            rel = abs(g[k] - num) / max(1e-6, abs(g[k]) + abs(num))
            worst = max(worst, rel)
    assert worst < 0.05, worst
    # the composition term reaches the mask/light and the background planes
    g0 = _oracle_grad(oracle, recon, target, comp, n, 1.0, 0.0)
    assert np.abs(g[6 * n:] - g0[6 * n:]).max() > 1e-6
    assert np.abs(g[:3 * n] - g0[:3 * n]).max() > 1e-6


def test_gradient_matches_float64_restatement(oracle):
    """Random planes, some composed values outside (0, 1) so the clamp's zero
    derivative is exercised; the analytic gradient of the numpy loss."""
    n = 24 * 20
    rng = np.random.default_rng(5)
    target, comp = _scene(rng, n)
    recon = f32(rng.uniform(-0.2, 1.3, 8 * n))
    wl, wc = 0.7, 1.9
    g = _oracle_grad(oracle, recon, target, comp, n, wl, wc)
    r = recon.reshape(8, n).astype(np.float32)
    m, l = r[6], r[7]
    base = r[0:3] * (np.float32(1) - m) + r[3:6] * m
    v = base * l
    y = np.clip(v, 0, 1)
    e = (y - comp.reshape(3, n)).astype(np.float64)
    gc = 2 * wc / (3 * n) * e * ((v > 0) & (v < 1))
    dl = 2 * wl / (8 * n) * (r.astype(np.float64) - target.reshape(8, n))
    ref = dl.copy()
    ref[0:3] += gc * (l * (np.float32(1) - m))
    ref[3:6] += gc * (l * m)
    ref[6] += (gc * l.astype(np.float64) * (r[3:6] - r[0:3]).astype(np.float64)).sum(0)
    ref[7] += (gc * base.astype(np.float64)).sum(0)
    np.testing.assert_allclose(g, ref.reshape(-1), rtol=1e-5, atol=1e-10)
    loss = oracle.orc_layered_loss(ptr(recon), ptr(target), ptr(comp), n, wl, wc)
    np.testing.assert_allclose(loss, _loss_np(recon, target, comp, n, wl, wc), rtol=1e-12)
