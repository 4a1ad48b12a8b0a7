"""tcgen05 implicit-GEMM convolution (forward, dX, dW, db) against the oracle.

The oracle composes the reference's own kernels per image (im2col + matmul +
biasRow forward; gradW + biasRowGrad + convBackInputS1 / col2im backward,
ConvGPU.swift:57-81).  Tolerance: relative L2 <= 1e-3 per op (tf32 operands,
fp32 accumulation; tf32 rounding alone gives ~4e-4).
"""
import numpy as np
import pytest

from oracle_lib import conv2d_bwd, conv2d_fwd, f32, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def kaiming_uniform(rng, oc, ic, k):
    bound = np.sqrt(6.0 / (ic * k * k))
    return f32(rng.uniform(-bound, bound, (oc, ic, k, k)))


CASES = [
    # (name, n, c, oc, h, w, k, stride, pad, up, up_hw)
    ("n2_c32_64x64", 2, 32, 32, 64, 64, 3, 1, 1, False, None),
    ("ragged", 1, 12, 20, 9, 13, 3, 1, 1, False, None),
    ("stride2", 2, 16, 24, 15, 17, 3, 2, 1, False, None),
    ("up", 2, 8, 16, 5, 6, 3, 1, 1, True, None),
    ("up_crop", 2, 8, 16, 5, 6, 3, 1, 1, True, (9, 11)),
    ("conv_in_rgb", 1, 3, 32, 20, 24, 3, 1, 1, False, None),
    ("conv_out_rgb", 1, 32, 3, 20, 24, 3, 1, 1, False, None),
    ("conv_in_rgb_c128", 2, 3, 128, 24, 40, 3, 1, 1, False, None),
    ("conv_out_rgb_c128", 2, 128, 3, 24, 40, 3, 1, 1, False, None),
    ("skip1x1", 2, 64, 128, 12, 10, 1, 1, 0, False, None),
    ("c128", 2, 128, 128, 24, 20, 3, 1, 1, False, None),
    ("c256", 1, 256, 256, 16, 18, 3, 1, 1, False, None),
    ("c128_to_384", 1, 128, 384, 15, 27, 3, 1, 1, False, None),
    ("s2_c128", 2, 128, 128, 30, 54, 3, 2, 1, False, None),
    # TMA phase-view paths: upsample + conv as four 2x2 phase convs, stride-2
    # via input phase views / output phases, odd extents, and a cropped upsample
    ("up_c128", 2, 128, 128, 10, 12, 3, 1, 1, True, None),
    ("up_c256_128", 1, 256, 128, 8, 14, 3, 1, 1, True, None),
    ("up_crop_c128", 1, 128, 128, 8, 9, 3, 1, 1, True, (15, 17)),
    ("up_c256_256", 2, 256, 256, 6, 10, 3, 1, 1, True, None),
    ("s2_odd_c128_256", 1, 128, 256, 15, 17, 3, 2, 1, False, None),
    ("c256_to_128", 1, 256, 128, 30, 54, 3, 1, 1, False, None),
    ("c128_tall_ragged", 1, 128, 128, 67, 40, 3, 1, 1, False, None),
    ("c128_h60_wide", 2, 128, 128, 60, 300, 3, 1, 1, False, None),
    ("c96_128", 2, 96, 128, 20, 36, 3, 1, 1, False, None),
    # one-row inputs: phase plans whose second row phase has no output pixels
    ("s2_h1", 1, 32, 32, 1, 9, 3, 2, 1, False, None),
    ("up_crop_h1", 1, 32, 32, 1, 5, 3, 1, 1, True, (1, 9)),
    # the motion U-Net's cut up level (30x54 -> 60x107, 256 -> 128): merged
    # phase taps over the x2 grid, then the border terms of the cut column
    ("up_crop_unet_256_128", 2, 256, 128, 30, 54, 3, 1, 1, True, (60, 107)),
    ("up_crop_rows_c64", 1, 64, 128, 7, 6, 3, 1, 1, True, (13, 12)),
    # a 1x1 conv of an upsampled input: no merged 3x3 taps for its dX
    ("up_k1", 1, 32, 32, 6, 7, 1, 1, 0, True, None),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_conv_forward_backward(case, oracle):
    from yumelayers_b200 import ops
    name, n, c, oc, h, w, k, stride, pad, up, up_hw = case
    rng = np.random.default_rng(0)
    x = f32(rng.standard_normal((n, c, h, w)))
    wt = kaiming_uniform(rng, oc, c, k)
    b = f32(rng.standard_normal(oc) * 0.1)
    y_ref = conv2d_fwd(oracle, x, wt, b, stride, pad, up, up_hw)
    y = ops.conv2d_fwd(x, wt, b, stride, pad, up, up_hw)
    assert y.shape == y_ref.shape
    assert rel_l2(y, y_ref) < TOL, name
    dy = f32(rng.standard_normal(y_ref.shape))
    dx_ref, dw_ref, db_ref, _ = conv2d_bwd(oracle, x, wt, dy, stride, pad, up, up_hw)
    dx = ops.conv2d_bwd_data(dy, wt, x.shape, stride, pad, up, up_hw)
    assert rel_l2(dx, dx_ref) < TOL, name
    dw, db = ops.conv2d_bwd_filter(x, dy, wt.shape, stride, pad, up, up_hw)
    assert rel_l2(dw, dw_ref) < TOL, name
    assert rel_l2(db, db_ref) < 1e-5, name


def test_conv_residual_and_determinism(oracle):
    from yumelayers_b200 import ops
    rng = np.random.default_rng(1)
    x = f32(rng.standard_normal((2, 32, 17, 19)))
    wt = kaiming_uniform(rng, 32, 32, 3)
    res = f32(rng.standard_normal((2, 32, 17, 19)))
    y_ref = conv2d_fwd(oracle, x, wt, None, residual=res)
    y1 = ops.conv2d_fwd(x, wt, None, residual=res)
    y2 = ops.conv2d_fwd(x, wt, None, residual=res)
    assert rel_l2(y1, y_ref) < TOL
    assert np.array_equal(y1, y2)  # fixed reduction order: bit-identical reruns
    dy = f32(rng.standard_normal(y_ref.shape))
    dw1, _ = ops.conv2d_bwd_filter(x, dy, wt.shape)
    dw2, _ = ops.conv2d_bwd_filter(x, dy, wt.shape)
    assert np.array_equal(dw1, dw2)


def test_conv_large_k_splitk(oracle):
    """dW with a long pixel contraction exercises the split-K partials."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(2)
    x = f32(rng.standard_normal((4, 32, 96, 96)))
    wt = kaiming_uniform(rng, 64, 32, 3)
    dy = f32(rng.standard_normal((4, 64, 96, 96)))
    _, dw_ref, db_ref, _ = conv2d_bwd(oracle, x, wt, dy)
    dw, db = ops.conv2d_bwd_filter(x, dy, wt.shape)
    assert rel_l2(dw, dw_ref) < TOL
    assert rel_l2(db, db_ref) < 1e-5


def test_conv_transpose_is_adjoint(oracle):
    """<convT(x), y> == <x, conv(y)>: the transposed conv is the conv's adjoint."""
    from yumelayers_b200 import _lib, ops
    import ctypes as C
    from yumelayers_b200.session import Context, GPUTensor
    rng = np.random.default_rng(3)
    n, c, oc, h, w = 2, 8, 12, 11, 13
    wt = kaiming_uniform(rng, oc, c, 3)
    d = ops.conv_desc((n, c, h, w), oc, 3, 2, 1)
    oh, ow = ops.conv_out_shape(d)
    xs = f32(rng.standard_normal((n, oc, oh, ow)))
    ys = f32(rng.standard_normal((n, c, h, w)))
    ctx = Context.shared()
    xd, wd = GPUTensor(ctx, 1, xs.size, xs), GPUTensor(ctx, 1, wt.size, wt)
    out = GPUTensor(ctx, 1, ys.size)
    _lib.call("yl_conv_transpose2d_fwd", ctx.handle, C.byref(d), C.c_void_p(xd.ptr),
              C.c_void_p(wd.ptr), None, C.c_void_p(out.ptr))
    ct = out.toArray().astype(np.float64)
    lhs = float((ct * ys.ravel()).sum())
    cy = conv2d_fwd(oracle, ys, wt, None, stride=2, pad=1)  # exact-ish fp32 oracle
    rhs = float((xs.astype(np.float64) * cy).sum())
    # tf32 error bound scales with the operand norms, not with the (cancelling) sum
    assert abs(lhs - rhs) <= 1e-3 * np.linalg.norm(ct) * np.linalg.norm(ys)
