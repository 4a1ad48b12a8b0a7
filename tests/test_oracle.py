"""Pins the CPU oracle before it is trusted as the checker.

1. Known-answer tests copied (as values and tolerances) from the reference's
   own unit tests: Tests/YumeLayersTests/TestGroup3.swift:296-537,
   TestGroup4.swift:116-221, TestGroup11.swift:82-206, TestGroup2.swift:115-145.
2. Cross-checks of the ops that exist only in the reference's PyTorch
   prototype (Conv2d, SiLU, GroupNorm with affine, Linear, Adam) against torch
   on CPU, and against golden vectors generated from the prototype's own code
   (tests/golden/make_golden.py).
"""
import ctypes as C
import math
from pathlib import Path

import numpy as np
import pytest

from oracle_lib import conv2d_bwd, conv2d_fwd, f32, gn_silu_bwd, gn_silu_fwd, ptr, rel_l2

GOLDEN = Path(__file__).resolve().parent / "golden"


# ------------------------------------------------------------ reference KATs
def test_add_bias_kat(oracle):  # TestGroup3.swift:369-377
    a = f32([1, 2, 3, 4, 5, 6])
    b = f32([10, 20, 30])
    out = np.zeros(6, np.float32)
    oracle.orc_add_bias(ptr(a), ptr(b), ptr(out), 6, 3)
    assert out.tolist() == [11, 22, 33, 14, 25, 36]


def test_sum_cols_kat(oracle):  # TestGroup3.swift:379-387
    a = f32(np.arange(1, 13))
    out = np.zeros(3, np.float32)
    oracle.orc_sum_cols(ptr(a), ptr(out), 4, 3)
    assert out.tolist() == [22, 26, 30]


def test_adam_one_step_kat(oracle):  # TestGroup3.swift:426-446
    p = f32([1, -2, 0.5, 0])
    g = f32([0.1, -0.4, 0, 0.3])
    m = np.zeros(4, np.float32)
    v = np.zeros(4, np.float32)
    p0 = p.copy()
    oracle.orc_adam(ptr(p), ptr(g), ptr(m), ptr(v), 4, 1, 1e-3, 0.9, 0.999, 1e-8)
    for i in range(4):
        mh = (0.1 * g[i]) / 0.1
        vh = (0.001 * g[i] * g[i]) / 0.001
        exp = p0[i] - 0.001 * mh / (math.sqrt(vh) + 1e-8)
        assert abs(p[i] - exp) < 1e-5


def test_adam_t0_is_clamped(oracle):  # GpuSessionOps.swift:246-248
    p, g = f32([1.0]), f32([0.5])
    m, v = np.zeros(1, np.float32), np.zeros(1, np.float32)
    oracle.orc_adam(ptr(p), ptr(g), ptr(m), ptr(v), 1, 0, 1e-3, 0.9, 0.999, 1e-8)
    assert np.isfinite(p).all()


def test_matmul_ragged_kat(oracle):  # TestGroup3.swift:345-366
    M, K, N = 37, 41, 53
    a = f32([(i % 13) * 0.1 for i in range(M * K)])
    b = f32([(i % 7) * 0.2 for i in range(K * N)])
    c = np.zeros(M * N, np.float32)
    oracle.orc_matmul(ptr(a), ptr(b), ptr(c), M, N, K, 0, 0)
    ref = a.reshape(M, K).astype(np.float64) @ b.reshape(K, N)
    assert np.abs(c.reshape(M, N) - ref).max() < 1e-4


def test_matmul_trans_kat(oracle):  # TestGroup3.swift:322-343
    rng = np.random.default_rng(1)
    M, K, N = 9, 6, 7
    a = f32(rng.uniform(-1, 1, K * M))  # stored K x M
    b = f32(rng.uniform(-1, 1, N * K))  # stored N x K
    c = np.zeros(M * N, np.float32)
    oracle.orc_matmul(ptr(a), ptr(b), ptr(c), M, N, K, 1, 1)
    ref = a.reshape(K, M).T.astype(np.float64) @ b.reshape(N, K).T
    assert np.abs(c.reshape(M, N) - ref).max() < 1e-5


def test_im2col_corner_kat(oracle):  # TestGroup3.swift:458-474
    ic, ih, iw, k, pad = 2, 6, 5, 3, 1
    x = f32(np.arange(ic * ih * iw) * 0.1)
    cols = np.zeros(ic * k * k * ih * iw, np.float32)
    oracle.orc_im2col(ptr(x), ptr(cols), ic, ih, iw, k, k, 1, pad)
    # col 0 is (c=0, ky=0, kx=0); its first entries sit in the padding ring
    assert cols[0] == 0.0 and cols[1] == 0.0
    # centre tap (ky=1,kx=1) of channel 0 reproduces the image
    centre = cols[4 * ih * iw:5 * ih * iw]
    assert np.array_equal(centre, x[: ih * iw])


def test_up_down_identity_kat(oracle):  # TestGroup3.swift:477-493
    c, h, w = 2, 2, 3
    x = f32(np.arange(1, 13))
    up = np.zeros(c * 4 * h * w, np.float32)
    down = np.zeros(c * h * w, np.float32)
    oracle.orc_upsample2x(ptr(x), ptr(up), c, h, w)
    oracle.orc_downsample2x(ptr(up), ptr(down), c, h, w)
    assert np.allclose(down, 4 * x, atol=1e-6)


def test_gradw_kat(oracle):  # TestGroup3.swift:496-516
    oc, kk, K = 3, 4, 25
    a = f32([((i % 9) - 4) * 0.3 for i in range(oc * K)])
    b = f32([((i % 7) - 3) * 0.2 for i in range(kk * K)])
    c = np.zeros(oc * kk, np.float32)
    oracle.orc_gradw(ptr(a), ptr(b), ptr(c), oc, kk, K)
    ref = a.reshape(oc, K).astype(np.float64) @ b.reshape(kk, K).T
    assert np.abs(c.reshape(oc, kk) - ref).max() < 1e-5


@pytest.mark.parametrize("cols", [64, 5000])
def test_bias_row_grad_kat(oracle, cols):  # TestGroup3.swift:519-536
    rows = 3
    d = f32([(i % 11) * 0.01 for i in range(rows * cols)])
    out = np.zeros(rows, np.float32)
    oracle.orc_bias_row_grad(ptr(d), ptr(out), rows, cols)
    assert np.abs(out - d.reshape(rows, cols).astype(np.float64).sum(1)).max() < 1e-3


def test_vae_primitive_kats(oracle):  # TestGroup4.swift:116-221
    e = np.zeros(3, np.float32)
    oracle.orc_unary(4, ptr(f32([0, 1, -2])), ptr(e), 3)
    assert abs(e[0] - 1) < 1e-6 and abs(e[1] - 2.718281828) < 1e-5 and abs(e[2] - 0.135335283) < 1e-6
    s = np.zeros(4, np.float32)
    oracle.orc_unary(5, ptr(f32([0, 1.386294361, 40, -40])), ptr(s), 4)
    assert abs(s[0] - 1) < 1e-6 and abs(s[1] - 2) < 1e-5
    assert abs(s[2] - math.exp(5)) < 1e-3 and abs(s[3] - math.exp(-5)) < 1e-6
    o = np.zeros(3, np.float32)
    oracle.orc_addconst(ptr(f32([1, 2, 3])), ptr(o), -1.5, 3)
    assert o.tolist() == [-0.5, 0.5, 1.5]
    oracle.orc_fma(ptr(f32([1, 2, 3])), ptr(f32([2, 2, 2])), ptr(f32([0.5, 1, -1])), ptr(o), 3)
    assert o.tolist() == [2, 4, 1]
    c, plane = 3, 5
    raw = f32([ch * 100 + i for ch in range(2 * c) for i in range(plane)])
    mu, lv = np.zeros(c * plane, np.float32), np.zeros(c * plane, np.float32)
    back = np.zeros_like(raw)
    oracle.orc_split2(ptr(raw), ptr(mu), ptr(lv), c, plane)
    oracle.orc_merge2(ptr(mu), ptr(lv), ptr(back), c, plane)
    assert np.array_equal(back, raw) and mu[0] == 0 and lv[0] == 300


def test_randn_statistics_kat(oracle):  # TestGroup4.swift:193-206
    n = 1 << 16
    a, b, c = (np.zeros(n, np.float32) for _ in range(3))
    oracle.orc_randn(ptr(a), 7, n)
    oracle.orc_randn(ptr(b), 7, n)
    oracle.orc_randn(ptr(c), 8, n)
    assert np.array_equal(a, b)
    assert np.abs(a - c).max() > 0.1
    assert abs(a.astype(np.float64).mean()) < 0.02
    assert abs(a.astype(np.float64).std() - 1) < 0.02
    assert np.isfinite(a).all()


def test_kl_kats(oracle):  # TestGroup4.swift:208-220
    z = np.zeros(10, np.float32)
    assert abs(oracle.orc_kl_sum(ptr(z), ptr(z), 10)) < 1e-5
    assert abs(oracle.orc_kl_sum(ptr(np.ones(10, np.float32)), ptr(z), 10) - 5.0) < 1e-4


def test_activation_kats(oracle):  # TestGroup3.swift:389-424
    x = f32([-2, -0.5, 0, 0.5, 2])
    r, s, t = (np.zeros(5, np.float32) for _ in range(3))
    oracle.orc_unary(0, ptr(x), ptr(r), 5)
    oracle.orc_unary(1, ptr(x), ptr(s), 5)
    oracle.orc_unary(2, ptr(x), ptr(t), 5)
    for i, xi in enumerate(x):
        assert abs(r[i] - max(0, xi)) < 1e-6
        assert abs(s[i] - 1 / (1 + math.exp(-xi))) < 1e-5
        assert abs(t[i] - math.tanh(xi)) < 1e-5
    z = f32([-1.3, -0.2, 0.4, 1.7])
    g = np.ones(4, np.float32)
    sg, tg = np.zeros(4, np.float32), np.zeros(4, np.float32)
    oracle.orc_binary(4, ptr(z), ptr(g), ptr(sg), 4)
    oracle.orc_unary(3, ptr(z), ptr(tg), 4)
    for i, zi in enumerate(z):
        sv = 1 / (1 + math.exp(-zi))
        assert abs(sg[i] - sv * (1 - sv)) < 1e-5
        assert abs(tg[i] - (1 - math.tanh(zi) ** 2)) < 1e-5


def test_mse_sum_kat(oracle):  # TestGroup2.swift:115-145
    w, h = 80, 56
    n = 3 * w * h
    a = f32([((i * 37) % 251) / 251 for i in range(n)])
    b = f32([((i * 91) % 241) / 241 for i in range(n)])
    got = oracle.orc_mse_sum(ptr(a), ptr(b), n)
    ref = float(((a.astype(np.float64) - b) ** 2).sum())
    assert abs(got - ref) / ref < 1e-5


def _gn_np(x, groups):
    c, p = x.shape
    out = np.zeros_like(x, dtype=np.float64)
    gs = c // groups
    for g in range(groups):
        blk = x[g * gs:(g + 1) * gs].astype(np.float64)
        mean = blk.mean()
        var = max((blk ** 2).mean() - mean ** 2, 1e-5)
        out[g * gs:(g + 1) * gs] = (blk - mean) / math.sqrt(var)
    return out


def test_groupnorm_ref_kat(oracle):  # TestGroup11.swift:180-206 (C8 P16 G4)
    rng = np.random.default_rng(77)
    C_, P_, G = 8, 16, 4
    x = f32(rng.uniform(-2, 2, C_ * P_))
    y = np.zeros_like(x)
    oracle.orc_groupnorm_ref(ptr(x), ptr(y), C_, G, P_)
    assert np.abs(y - _gn_np(x.reshape(C_, P_), G).ravel()).max() < 1e-3
    assert abs(y[: (C_ // G) * P_].astype(np.float64).mean()) < 1e-3


def test_groupnorm_grad_finite_differences(oracle):  # TestGroup11.swift:82-127 (rel < 2%)
    rng = np.random.default_rng(77)
    C_, G, P_ = 8, 2, 24
    x = rng.uniform(-2, 2, C_ * P_).astype(np.float32)
    dy = rng.uniform(-1, 1, C_ * P_).astype(np.float32)
    dx = np.zeros_like(x)
    oracle.orc_groupnorm_grad_ref(ptr(x), ptr(dy), ptr(dx), C_, G, P_)

    def loss(xx):
        return float((_gn_np(xx.reshape(C_, P_), G).ravel() * dy).sum())

    eps = 1e-3
    for i in rng.choice(x.size, 12, replace=False):
        xp, xm = x.astype(np.float64).copy(), x.astype(np.float64).copy()
        xp[i] += eps
        xm[i] -= eps
        num = (loss(xp) - loss(xm)) / (2 * eps)
        assert abs(num - dx[i]) <= 0.02 * max(abs(num), 1e-2)


def test_splitmix64_and_noise_seed(oracle):  # ConvVAEHelpers.swift:10-37
    s = C.c_uint64(0)
    a = [oracle.orc_splitmix64_next(C.byref(s)) for _ in range(3)]
    s2 = C.c_uint64(0)
    b = [oracle.orc_splitmix64_next(C.byref(s2)) for _ in range(3)]
    assert a == b and len(set(a)) == 3
    # Published SplitMix64 first output for seed 0.
    assert a[0] == 0xE220A8397B1DCDAF
    seeds = {oracle.orc_training_noise_seed(step, b) for step in range(4) for b in range(4)}
    assert len(seeds) == 16


def test_motion_time_embedding_kat(oracle):  # MotionPlanner.swift:155-165
    out = np.zeros(128, np.float32)
    oracle.orc_motion_time_embedding(0.25, 128, ptr(out))
    i = np.arange(0, 128, 2)
    w = 1000.0 ** (i / 128)
    assert np.allclose(out[0::2], np.sin(0.25 * w), atol=1e-6)
    assert np.allclose(out[1::2], np.cos(0.25 * w), atol=1e-6)
    oracle.orc_motion_time_embedding(7.0, 128, ptr(out))  # clamped to 1
    assert np.allclose(out[0::2], np.sin(w), atol=1e-6)
    oracle.orc_motion_time_embedding(float("nan"), 128, ptr(out))  # non-finite -> 0
    assert np.allclose(out[0::2], 0, atol=1e-7) and np.allclose(out[1::2], 1, atol=1e-7)


def test_sanitize_grads_kat(oracle):  # GradSanitize.swift:18-101
    g = f32([3.0, 4.0, float("nan"), float("inf")])
    fixed = C.c_long()
    norm = oracle.orc_sanitize_grads(ptr(g), 4, 1.0, 1.0, C.byref(fixed))
    assert fixed.value == 2 and abs(norm - 5.0) < 1e-6
    assert np.allclose(g, [0.6, 0.8, 0, 0], atol=1e-6)


# ------------------------------------------------------------ oracle vs torch / prototype
torch = pytest.importorskip("torch")


@pytest.mark.parametrize("stride,up,hw", [(1, False, (9, 11)), (2, False, (9, 11)),
                                          (1, True, (5, 6)), (1, True, (5, 6, 9, 11))])
def test_conv_oracle_vs_torch(oracle, stride, up, hw):
    rng = np.random.default_rng(3)
    n, c, oc = 2, 8, 12
    h, w = hw[:2]
    x = f32(rng.standard_normal((n, c, h, w)))
    wt = f32(rng.uniform(-0.3, 0.3, (oc, c, 3, 3)))
    b = f32(rng.standard_normal(oc))
    up_hw = hw[2:] if len(hw) == 4 else None
    y = conv2d_fwd(oracle, x, wt, b, stride, 1, up, up_hw)
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    xin = tx
    if up:
        xin = torch.nn.functional.interpolate(tx, scale_factor=2, mode="nearest")
        if up_hw:
            xin = xin[:, :, : up_hw[0], : up_hw[1]]
    tw = torch.tensor(wt, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    ty = torch.nn.functional.conv2d(xin, tw, tb, stride=stride, padding=1)
    assert rel_l2(y, ty.detach().numpy()) < 1e-5
    dy = f32(rng.standard_normal(ty.shape))
    ty.backward(torch.tensor(dy, dtype=torch.float64))
    dx, dw, db, _ = conv2d_bwd(oracle, x, wt, dy, stride, 1, up, up_hw)
    assert rel_l2(dx, tx.grad.numpy()) < 1e-5
    assert rel_l2(dw, tw.grad.numpy()) < 1e-5
    assert rel_l2(db, tb.grad.numpy()) < 1e-5


def test_gn_silu_oracle_vs_torch(oracle):
    rng = np.random.default_rng(4)
    n, c, h, w, G = 2, 16, 5, 7, 4
    x = f32(rng.standard_normal((n, c, h, w)) * 2 + 0.5)
    ga = f32(1 + 0.02 * rng.standard_normal(c))
    be = f32(0.02 * rng.standard_normal(c))
    y, _, _ = gn_silu_fwd(oracle, x, G, 1e-6, ga, be)
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tg = torch.tensor(ga, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(be, dtype=torch.float64, requires_grad=True)
    ty = torch.nn.functional.silu(torch.nn.functional.group_norm(tx, G, tg, tb, 1e-6))
    assert rel_l2(y, ty.detach().numpy()) < 1e-6
    dy = f32(rng.standard_normal(x.shape))
    ty.backward(torch.tensor(dy, dtype=torch.float64))
    dx, dg, db = gn_silu_bwd(oracle, x, dy, G, 1e-6, ga, be)
    assert rel_l2(dx, tx.grad.numpy()) < 1e-5
    assert rel_l2(dg, tg.grad.numpy()) < 1e-5
    assert rel_l2(db, tb.grad.numpy()) < 1e-5


def test_linear_oracle_vs_torch(oracle):
    rng = np.random.default_rng(5)
    n, ic, oc = 6, 13, 9
    X = f32(rng.standard_normal((n, ic)))
    W = f32(rng.standard_normal((oc, ic)))
    b = f32(rng.standard_normal(oc))
    Y = np.zeros((n, oc), np.float32)
    oracle.orc_linear_fwd(ptr(X), ptr(W), ptr(b), ptr(Y), n, ic, oc, 0)
    tX = torch.tensor(X, dtype=torch.float64, requires_grad=True)
    tW = torch.tensor(W, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    tY = torch.nn.functional.linear(tX, tW, tb)
    assert rel_l2(Y, tY.detach().numpy()) < 1e-6
    dY = f32(rng.standard_normal((n, oc)))
    tY.backward(torch.tensor(dY, dtype=torch.float64))
    dX, dW, db = np.zeros_like(X), np.zeros_like(W), np.zeros_like(b)
    oracle.orc_linear_bwd(ptr(X), ptr(W), ptr(dY), ptr(dX), ptr(dW), ptr(db), n, ic, oc)
    assert rel_l2(dX, tX.grad.numpy()) < 1e-6
    assert rel_l2(dW, tW.grad.numpy()) < 1e-6
    assert rel_l2(db, tb.grad.numpy()) < 1e-6


def test_adam_oracle_vs_torch(oracle):
    rng = np.random.default_rng(6)
    p = f32(rng.standard_normal(100))
    tp = torch.nn.Parameter(torch.tensor(p.copy()))
    opt = torch.optim.Adam([tp], lr=2e-4, betas=(0.9, 0.999), eps=1e-8)
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    for t in range(1, 6):
        g = f32(rng.standard_normal(100))
        oracle.orc_adam(ptr(p), ptr(g), ptr(m), ptr(v), 100, t, 2e-4, 0.9, 0.999, 1e-8)
        tp.grad = torch.tensor(g)
        opt.step()
    assert np.abs(p - tp.detach().numpy()).max() < 1e-6


# ------------------------------------------------------------ golden vectors from the prototype
def test_timestep_embedding_golden(oracle):
    g = np.load(GOLDEN / "prototype_golden.npz")
    t = f32(g["temb_t"])
    out = np.zeros((t.size, 128), np.float32)
    oracle.orc_timestep_embedding_torch(ptr(t), t.size, 128, 10000.0, ptr(out))
    assert np.abs(out - g["temb_out"]).max() < 2e-5


def test_resblock_golden(oracle):
    """x + conv(SiLU(conv(x))) of src/vae.py:7-15 from the oracle's layer math."""
    g = np.load(GOLDEN / "prototype_golden.npz")
    x, w1, b1, w2, b2 = (g[k] for k in ("rb_x", "rb_w1", "rb_b1", "rb_w2", "rb_b2"))
    h = conv2d_fwd(oracle, x, w1, b1)
    hs = np.zeros_like(h)
    oracle.orc_unary(6, ptr(h), ptr(hs), h.size)
    y = conv2d_fwd(oracle, hs, w2, b2, residual=x)
    assert rel_l2(y, g["rb_y"]) < 1e-5


def _silu(oracle, z):
    out = np.empty_like(z)
    oracle.orc_unary(6, ptr(z), ptr(out), z.size)
    return out


def _silu_grad(oracle, z, g):
    out = np.empty_like(z)
    oracle.orc_binary(5, ptr(f32(z)), ptr(f32(g)), ptr(out), z.size)
    return out


@pytest.mark.parametrize("name", ["up", "down"])
def test_decoder_and_encoder_stage_golden(oracle, name):
    """One stage of the prototype's decoder (src/vae.py:44-45: ResBlock, nearest
    x2 upsample, 3x3 conv, SiLU) or encoder (src/vae.py:27-28: ResBlock,
    stride-2 3x3 conv, SiLU), forward and backward (torch autograd for an
    upstream gradient g), against the oracle's conv / SiLU layer math: the
    upsample conv's dX is the 2x2 sum of the upsampled-input gradient, the
    stride-2 conv's the col2im gather."""
    g = np.load(GOLDEN / "prototype_golden.npz")
    k = lambda s: f32(g[f"{name}_{s}"])  # noqa: E731
    up, stride = name == "up", 1 if name == "up" else 2
    x = k("x")
    h = conv2d_fwd(oracle, x, k("rb_w1"), k("rb_b1"))
    hs = _silu(oracle, h)
    r = conv2d_fwd(oracle, hs, k("rb_w2"), k("rb_b2"), residual=x)
    p = conv2d_fwd(oracle, r, k("w"), k("b"), stride=stride, up=up)
    y = _silu(oracle, p)
    assert rel_l2(y, k("y")) < 1e-5
    dp = _silu_grad(oracle, p, k("g"))
    dr, dw, db, _ = conv2d_bwd(oracle, r, k("w"), dp, stride=stride, up=up)
    dhs, dw2, db2, _ = conv2d_bwd(oracle, hs, k("rb_w2"), dr)
    dx1, dw1, db1, _ = conv2d_bwd(oracle, x, k("rb_w1"), _silu_grad(oracle, h, dhs))
    for got, key in ((dw, "dw"), (db, "db"), (dw2, "drb_w2"), (db2, "drb_b2"), (dw1, "drb_w1"),
                     (db1, "drb_b1"), (dx1 + dr, "dx")):
        assert rel_l2(got, k(key)) < 1e-5, key


def test_time_conditioning_mlp_golden(oracle):
    """The prototype's time conditioning (src/diffusion.py:38,49: DiT.time_mlp,
    Linear -> SiLU -> Linear, over timestep_embedding(t, 128)), forward and the
    weight gradients for an upstream gradient g, from the oracle's embedding,
    Linear and SiLU."""
    g = np.load(GOLDEN / "prototype_golden.npz")
    k = lambda s: f32(g[f"tmlp_{s}"])  # noqa: E731
    t = k("t")
    n, d = t.size, 128
    emb = np.empty((n, d), np.float32)
    oracle.orc_timestep_embedding_torch(ptr(t), n, d, 10000.0, ptr(emb))
    h = np.empty((n, d), np.float32)
    oracle.orc_linear_fwd(ptr(emb), ptr(k("w1")), ptr(k("b1")), ptr(h), n, d, d, 0)
    hs = _silu(oracle, h)
    y = np.empty((n, d), np.float32)
    oracle.orc_linear_fwd(ptr(hs), ptr(k("w2")), ptr(k("b2")), ptr(y), n, d, d, 0)
    assert rel_l2(y, k("y")) < 1e-5
    dhs, dw2, db2 = np.empty_like(hs), np.empty((d, d), np.float32), np.empty(d, np.float32)
    oracle.orc_linear_bwd(ptr(hs), ptr(k("w2")), ptr(k("g")), ptr(dhs), ptr(dw2), ptr(db2), n, d, d)
    dh = _silu_grad(oracle, h, dhs)
    dw1, db1 = np.empty((d, d), np.float32), np.empty(d, np.float32)
    oracle.orc_linear_bwd(ptr(emb), ptr(k("w1")), ptr(dh), None, ptr(dw1), ptr(db1), n, d, d)
    for got, key in ((dw2, "dw2"), (db2, "db2"), (dw1, "dw1"), (db1, "db1")):
        assert rel_l2(got, k(key)) < 1e-5, key
