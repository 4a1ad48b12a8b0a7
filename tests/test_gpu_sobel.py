"""Sobel edge loss on the GPU against the oracle (LossFunctions.swift:29-66,
194-235), per image, in both layouts."""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import f32, ptr, rel_l2

pytestmark = pytest.mark.gpu


def _oracle(oracle, r, t):
    """NCHW image batch -> (losses, NCHW grads) through the HWC oracle."""
    n, _, h, w = r.shape
    losses, grads = [], []
    for i in range(n):
        rh, th = f32(r[i].transpose(1, 2, 0)), f32(t[i].transpose(1, 2, 0))
        losses.append(oracle.orc_sobel_edge_loss(ptr(rh), ptr(th), w, h))
        g = np.zeros(h * w * 3, np.float32)
        oracle.orc_sobel_edge_grad(ptr(rh), ptr(th), w, h, ptr(g))
        grads.append(g.reshape(h, w, 3).transpose(2, 0, 1))
    return np.array(losses), np.stack(grads)


def test_sobel_nchw_matches_oracle(oracle):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(7)
    r = f32(rng.uniform(0, 1, (2, 3, 24, 40)))
    t = f32(rng.uniform(0, 1, (2, 3, 24, 40)))
    loss, grad = ops.sobel_edge_loss(r, t)
    lref, gref = _oracle(oracle, r, t)
    np.testing.assert_allclose(loss, lref, rtol=1e-5)
    assert rel_l2(grad, gref) < 1e-5
    loss0, grad0 = ops.sobel_edge_loss(t, t)
    assert np.all(loss0 == 0) and np.all(grad0 == 0)


def test_sobel_nhwc_with_pixel_stride(oracle, ctx):
    from yumelayers_b200._lib import LAYOUT_NHWC, call
    from yumelayers_b200.session import GPUTensor
    rng = np.random.default_rng(8)
    n, h, w = 2, 17, 23
    r = f32(rng.uniform(0, 1, (n, 3, h, w)))
    t = f32(rng.uniform(0, 1, (n, 3, h, w)))
    def nhwc4(a):
        out = np.zeros((n, h, w, 4), np.float32)
        out[..., :3] = a.transpose(0, 2, 3, 1)
        return out
    rd, td = GPUTensor(ctx, 1, n * h * w * 4, nhwc4(r)), GPUTensor(ctx, 1, n * h * w * 4, nhwc4(t))
    gd, ld = GPUTensor(ctx, 1, n * h * w * 4), GPUTensor(ctx, 1, n)
    call("yl_sobel_edge_loss", ctx.handle, C.c_void_p(rd.ptr), C.c_void_p(td.ptr), n, h, w,
         LAYOUT_NHWC, 4, C.c_void_p(gd.ptr), C.c_void_p(ld.ptr))
    lref, gref = _oracle(oracle, r, t)
    np.testing.assert_allclose(ld.toArray()[:n], lref, rtol=1e-5)
    g = gd.toArray()[: n * h * w * 4].reshape(n, h, w, 4)[..., :3].transpose(0, 3, 1, 2)
    assert rel_l2(g, gref) < 1e-5


@pytest.mark.parametrize("n,h,w", [(2, 100, 150), (1, 480, 856), (1, 3, 3), (1, 16, 64)])
def test_sobel_tiles_and_edges_match_oracle(oracle, n, h, w):
    """Several 64 x 16 tiles with ragged last tiles, the frame size, the
    smallest image with an interior pixel, and exactly one tile."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(h * 1000 + w)
    r = f32(rng.uniform(0, 1, (n, 3, h, w)))
    t = f32(np.clip(r + 0.1 * rng.standard_normal((n, 3, h, w)), 0, 1))
    loss, grad = ops.sobel_edge_loss(r, t)
    lref, gref = _oracle(oracle, r, t)
    np.testing.assert_allclose(loss, lref, rtol=1e-5)
    assert rel_l2(grad, gref) < 1e-5
