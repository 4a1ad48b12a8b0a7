"""Reference-mode operators on the GPU (through the C ABI) against the oracle.

Ports of the reference's own GPU op tests (Tests/YumeLayersTests/
TestGroup3.swift:296-537, TestGroup4.swift:116-221, TestGroup11.swift:130-206,
TestGroup2.swift:115-145) with their tolerances, plus element-for-element
comparisons with the oracle at larger sizes.
"""
import math

import numpy as np
import pytest

from oracle_lib import f32, ptr, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def S():
    from yumelayers_b200.session import GpuSession
    return GpuSession()


def T(S, data, rows):
    from yumelayers_b200.session import GPUTensor
    return GPUTensor(S.ctx, rows, data=data)


def test_matmul_small_and_trans(S, oracle):
    rng = np.random.default_rng(0)
    A, B = rng.uniform(-1, 1, (7, 5)), rng.uniform(-1, 1, (5, 9))
    S.begin()
    Cg = S.matmul(T(S, A, 7), T(S, B, 5))
    S.end()
    assert np.abs(Cg.toArray().reshape(7, 9) - A @ B).max() < 1e-5
    M, K, N = 9, 6, 7
    Ar, Br = rng.uniform(-1, 1, (K, M)), rng.uniform(-1, 1, (N, K))
    S.begin()
    Cg = S.matmul(T(S, Ar, K), T(S, Br, N), transA=True, transB=True, M=M, N=N, K=K)
    S.end()
    assert np.abs(Cg.toArray().reshape(M, N) - Ar.T @ Br.T).max() < 1e-5


def test_matmul_ragged_tiles(S):
    M, K, N = 37, 41, 53
    a = np.array([(i % 13) * 0.1 for i in range(M * K)], np.float32)
    b = np.array([(i % 7) * 0.2 for i in range(K * N)], np.float32)
    S.begin()
    Cg = S.matmul(T(S, a, M), T(S, b, K))
    S.end()
    ref = a.reshape(M, K).astype(np.float64) @ b.reshape(K, N)
    assert np.abs(Cg.toArray().reshape(M, N) - ref).max() < 1e-4


def test_add_bias_sum_cols(S):
    S.begin()
    r = S.addBias(T(S, [1, 2, 3, 4, 5, 6], 2), T(S, [10, 20, 30], 1))
    s = S.sumCols(T(S, np.arange(1, 13), 4))
    S.end()
    assert r.toArray().tolist() == [11, 22, 33, 14, 25, 36]
    assert s.toArray().tolist() == [22, 26, 30]


def test_activations_and_grads(S):
    x = [-2, -0.5, 0, 0.5, 2]
    t = T(S, x, 1)
    S.begin()
    relu, sig, th = S.relu(t), S.sigmoid(t), S.tanh(t)
    S.end()
    for i, xi in enumerate(x):
        assert abs(relu.toArray()[i] - max(0, xi)) < 1e-6
        assert abs(sig.toArray()[i] - 1 / (1 + math.exp(-xi))) < 1e-5
        assert abs(th.toArray()[i] - math.tanh(xi)) < 1e-5
    z = [-1.3, -0.2, 0.4, 1.7]
    zt, gt = T(S, z, 1), T(S, [1, 1, 1, 1], 1)
    S.begin()
    rg = S.reluGrad(T(S, [max(0, v) for v in z], 1), gt)
    sg, tg = S.sigmoidGrad(zt, gt), S.tanhGrad(zt)
    S.end()
    for i, zi in enumerate(z):
        assert abs(rg.toArray()[i] - (1 if zi > 0 else 0)) < 1e-6
        s = 1 / (1 + math.exp(-zi))
        assert abs(sg.toArray()[i] - s * (1 - s)) < 1e-5
        assert abs(tg.toArray()[i] - (1 - math.tanh(zi) ** 2)) < 1e-5


def test_adam_one_step(S):
    from yumelayers_b200.session import GPUTensor
    p, g = [1, -2, 0.5, 0], [0.1, -0.4, 0, 0.3]
    pt, gt = T(S, p, 1), T(S, g, 1)
    m, v = GPUTensor(S.ctx, 1, 4), GPUTensor(S.ctx, 1, 4)
    S.begin()
    S.zeroFill(m)
    S.zeroFill(v)
    S.adamUpdate(pt, gt, m, v, 1, 0.001)
    S.end()
    out = pt.toArray()
    for i in range(4):
        mh, vh = (0.1 * g[i]) / 0.1, (0.001 * g[i] ** 2) / 0.001
        assert abs(out[i] - (p[i] - 0.001 * mh / (math.sqrt(vh) + 1e-8))) < 1e-5


def test_conv_primitives(S, oracle):
    ic, ih, iw, k, pad = 2, 6, 5, 3, 1
    x = np.arange(ic * ih * iw, dtype=np.float32) * 0.1
    S.begin()
    cols = S.im2col(T(S, x, ic), ih, iw, ic, k, k, 1, pad)
    S.end()
    assert cols.rows == ic * k * k and cols.cols == ih * iw
    ref = np.zeros(ic * k * k * ih * iw, np.float32)
    oracle.orc_im2col(ptr(x), ptr(ref), ic, ih, iw, k, k, 1, pad)
    assert np.array_equal(cols.toArray(), ref)
    c, h, w = 2, 2, 3
    xs = np.arange(1, 13, dtype=np.float32)
    S.begin()
    up = S.upsample2x(T(S, xs, c), h, w)
    down = S.downsample2x(up, h, w)
    S.end()
    assert np.allclose(down.toArray(), 4 * xs, atol=1e-6)
    oc, kk, K = 3, 4, 25
    a = np.array([((i % 9) - 4) * 0.3 for i in range(oc * K)], np.float32)
    b = np.array([((i % 7) - 3) * 0.2 for i in range(kk * K)], np.float32)
    S.begin()
    g = S.gradW(T(S, a, oc), T(S, b, kk), oc, kk)
    S.end()
    ref = a.reshape(oc, K).astype(np.float64) @ b.reshape(kk, K).T
    assert np.abs(g.toArray().reshape(oc, kk) - ref).max() < 1e-5
    for ncols in (64, 5000):
        d = np.array([(i % 11) * 0.01 for i in range(3 * ncols)], np.float32)
        S.begin()
        gg = S.biasRowGrad(T(S, d, 3))
        S.end()
        assert np.abs(gg.toArray() - d.reshape(3, ncols).sum(1)).max() < 1e-3


@pytest.mark.parametrize("stride", [1, 2])
def test_col2im_and_back_input_vs_oracle(S, oracle, stride):
    rng = np.random.default_rng(2)
    ic, oc, ih, iw, k, pad = 5, 7, 13, 11, 3, 1
    oh, ow = (ih + 2 * pad - k) // stride + 1, (iw + 2 * pad - k) // stride + 1
    dcols = f32(rng.standard_normal((ic * k * k, oh * ow)))
    S.begin()
    G = S.col2im(T(S, dcols, ic * k * k), ic, ih, iw, k, k, stride, pad, oh, ow)
    S.end()
    ref = np.zeros(ic * ih * iw, np.float32)
    oracle.orc_col2im(ptr(dcols), ptr(ref), ic, ih, iw, k, k, stride, pad, oh, ow)
    assert rel_l2(G.toArray(), ref) < 1e-6
    if stride == 1:
        dout = f32(rng.standard_normal((oc, ih * iw)))
        W = f32(rng.standard_normal((oc, ic * k * k)))
        S.begin()
        dx = S.convBackInputS1(T(S, dout, oc), T(S, W, oc), ic, oc, ih, iw, k, pad)
        S.end()
        ref = np.zeros(ic * ih * iw, np.float32)
        oracle.orc_conv_back_input_s1(ptr(dout), ptr(W), ptr(ref), ic, oc, ih, iw, k, k, pad)
        assert rel_l2(dx.toArray(), ref) < 1e-6


def test_groupnorm_reference_mode(S, oracle):
    rng = np.random.default_rng(77)
    C_, P_, G = 8, 16, 4
    x = f32(rng.uniform(-2, 2, C_ * P_))
    S.begin()
    y = S.groupNorm(T(S, x, C_), G)
    S.end()
    ref = np.zeros_like(x)
    oracle.orc_groupnorm_ref(ptr(x), ptr(ref), C_, G, P_)
    assert np.abs(y.toArray() - ref).max() < 1e-3
    C_, G, P_ = 8, 2, 32 * 24
    x = f32(rng.uniform(-2, 2, C_ * P_))
    dy = f32(rng.uniform(-1, 1, C_ * P_))
    S.begin()
    g = S.encodeGroupNormGrad(T(S, x, C_), T(S, dy, C_), G)
    S.end()
    ref = np.zeros_like(x)
    oracle.orc_groupnorm_grad_ref(ptr(x), ptr(dy), ptr(ref), C_, G, P_)
    assert np.abs(g.toArray() - ref).max() < 1e-4


def test_vae_primitives(S, oracle):
    S.begin()
    e = S.exp(T(S, [0, 1, -2], 1))
    s = S.expHalf(T(S, [0, 1.386294361, 40, -40], 1))
    a = S.addConst(T(S, [1, 2, 3], 1), -1.5)
    f = S.fma(T(S, [1, 2, 3], 1), T(S, [2, 2, 2], 1), T(S, [0.5, 1, -1], 1))
    S.end()
    ev, sv = e.toArray(), s.toArray()
    assert abs(ev[0] - 1) < 1e-6 and abs(ev[1] - 2.718281828) < 1e-5
    assert abs(sv[1] - 2) < 1e-5 and abs(sv[2] - math.exp(5)) < 1e-3 and abs(sv[3] - math.exp(-5)) < 1e-6
    assert a.toArray().tolist() == [-0.5, 0.5, 1.5] and f.toArray().tolist() == [2, 4, 1]
    c, plane = 3, 5
    raw = np.array([ch * 100 + i for ch in range(2 * c) for i in range(plane)], np.float32)
    S.begin()
    mu, lv = S.split2(T(S, raw, 2 * c), c, plane)
    back = S.merge2(mu, lv, c, plane)
    S.end()
    assert np.array_equal(back.toArray(), raw) and mu.toArray()[0] == 0 and lv.toArray()[0] == 300
    n = 1 << 16
    S.begin()
    g1, g2, g3 = S.randn(7, 1, n), S.randn(7, 1, n), S.randn(8, 1, n)
    S.end()
    v1 = g1.toArray()
    assert np.array_equal(v1, g2.toArray()) and np.abs(v1 - g3.toArray()).max() > 0.1
    assert abs(v1.astype(np.float64).mean()) < 0.02 and abs(v1.std() - 1) < 0.02
    ref = np.zeros(n, np.float32)
    oracle.orc_randn(ptr(ref), 7, n)
    assert np.abs(v1 - ref).max() < 1e-5  # same hash; libm ulps differ
    S.begin()
    k0 = S.kl(T(S, np.zeros(10), 1), T(S, np.zeros(10), 1))
    k1 = S.kl(T(S, np.ones(10), 1), T(S, np.zeros(10), 1))
    S.end()
    assert abs(k0.value()) < 1e-5 and abs(k1.value() - 5.0) < 1e-4


def test_mse_and_l1_grad(S, oracle):
    w, h = 80, 56
    n = 3 * w * h
    a = np.array([((i * 37) % 251) / 251 for i in range(n)], np.float32)
    b = np.array([((i * 91) % 241) / 241 for i in range(n)], np.float32)
    S.begin()
    buf = S.encodeMSE(T(S, a, 3), T(S, b, 3))
    g = S.encodeL1Grad(T(S, a, 3), T(S, b, 3))
    S.end()
    cpu = float(((a.astype(np.float64) - b) ** 2).sum())
    assert abs(buf.value() - cpu) / cpu < 1e-5
    ref = np.zeros(n, np.float32)
    oracle.orc_l1grad(ptr(a), ptr(b), ptr(ref), np.float32(1.0 / n), n)
    assert np.array_equal(g.toArray(), ref)


def test_vae_grad(S, oracle):
    rng = np.random.default_rng(9)
    n = 1000
    dz, mu, eps = (f32(rng.standard_normal(n)) for _ in range(3))
    lv = f32(rng.uniform(-12, 12, n))
    S.begin()
    dmu, dlv = S.vaeGrad(T(S, dz, 1), T(S, mu, 1), T(S, lv, 1), T(S, eps, 1), 0.25, 0.125)
    S.end()
    rm, rl = np.zeros(n, np.float32), np.zeros(n, np.float32)
    oracle.orc_vae_grad(ptr(dz), ptr(mu), ptr(lv), ptr(eps), ptr(rm), ptr(rl), 0.25, 0.125, n)
    assert rel_l2(dmu.toArray(), rm) < 1e-6 and rel_l2(dlv.toArray(), rl) < 1e-5


def test_session_timeout_and_errors(S):
    from yumelayers_b200 import YumeError
    S.begin()
    ms = S.end(timeout_s=5.0)
    assert ms >= 0.0
    with pytest.raises(YumeError):
        S.groupNorm(T(S, np.zeros(6), 3), 2)  # rows % groups != 0 -> YL_ERR_SHAPE
