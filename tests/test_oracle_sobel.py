"""Sobel edge loss in the oracle against the reference's own checks
(TestGroup11.swift:4-80): uniform image, vertical edge, identical and
blurred images, finite differences of the gradient, zero self-gradient."""
import numpy as np

from oracle_lib import f32, ptr


def _edge(w=16, h=16):
    img = np.zeros((h, w, 3), np.float32)
    img[:, 8:] = 1.0
    return img


def test_sobel_maps_and_loss(oracle):
    flat = np.full((16, 16, 3), 0.5, np.float32)
    g = np.zeros(256, np.float32)
    oracle.orc_sobel_luma(ptr(flat), 16, 16, ptr(g))
    assert (g == 0).all()
    edge = _edge()
    oracle.orc_sobel_luma(ptr(edge), 16, 16, ptr(g))
    assert g.max() > 0.1
    assert abs(oracle.orc_sobel_edge_loss(ptr(edge), ptr(edge), 16, 16)) < 1e-9
    x = np.arange(16)
    v = (np.minimum(15, x + 3) / 15.0).astype(np.float32)
    blurred = np.repeat(np.tile(v, (16, 1))[:, :, None], 3, axis=2).astype(np.float32)
    assert oracle.orc_sobel_edge_loss(ptr(blurred), ptr(edge), 16, 16) > 0.01


def test_sobel_grad_finite_differences(oracle):
    w, h = 16, 12
    rng = np.random.default_rng(1234)
    recon = f32(rng.uniform(0, 1, (h, w, 3)))
    target = f32(rng.uniform(0, 1, (h, w, 3)))
    grad = np.zeros(w * h * 3, np.float32)
    oracle.orc_sobel_edge_grad(ptr(recon), ptr(target), w, h, ptr(grad))
    flat = recon.reshape(-1)
    eps = 1e-3
    for idx in [(w * 7 + 8) * 3, (w * h - 1) * 3 + 2, 5 * 3 + 1, (w * 3 + 4) * 3 + 1]:
        orig = flat[idx]
        flat[idx] = orig + eps
        lp = oracle.orc_sobel_edge_loss(ptr(flat), ptr(target), w, h)
        flat[idx] = orig - eps
        lm = oracle.orc_sobel_edge_loss(ptr(flat), ptr(target), w, h)
        flat[idx] = orig
        num = (lp - lm) / (2 * eps)
        ana = float(grad[idx])
        assert abs(ana - num) / max(1e-9, abs(ana) + abs(num)) < 0.02, (idx, ana, num)
    oracle.orc_sobel_edge_grad(ptr(target), ptr(target), w, h, ptr(grad))
    assert (grad == 0).all()
