"""yl_groupnorm_silu_fwd_noalloc (statistics partials in a fixed array inside
the library) against yl_groupnorm_silu_fwd on the same NHWC inputs, twice in
a row, and against the oracle's GroupNorm + SiLU, plus its size limit.
Collected last so that it also runs after every other GPU test has used the
context."""
import ctypes as C

import numpy as np
import pytest

from oracle_lib import gn_silu_fwd
from yumelayers_b200._lib import LAYOUT_NHWC, call, lib
from yumelayers_b200.session import GPUTensor

pytestmark = pytest.mark.gpu

TOL = 1e-6  # relative L2; both paths run the same statistics and apply arithmetic


def _dev(ctx, a):
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    return GPUTensor(ctx, 1, a.size, a)


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("n,c,h,w,g", [(2, 128, 24, 20, 32), (8, 256, 30, 54, 32),
                                       (1, 64, 7, 9, 16)])
def test_noalloc_matches_allocating_entry_point_twice(ctx, oracle, n, c, h, w, g):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((n, h, w, c)) * 1.3 + 0.2).astype(np.float32)
    ga = (1 + 0.02 * rng.standard_normal(c)).astype(np.float32)
    be = (0.02 * rng.standard_normal(c)).astype(np.float32)
    xd, gd, bd = _dev(ctx, x), _dev(ctx, ga), _dev(ctx, be)
    ref_y, ref_m, ref_r = (GPUTensor(ctx, 1, x.size), GPUTensor(ctx, 1, n * g),
                           GPUTensor(ctx, 1, n * g))
    call("yl_groupnorm_silu_fwd", ctx.handle, C.c_void_p(xd.ptr), n, c, h, w, LAYOUT_NHWC, g,
         1e-6, 0, C.c_void_p(gd.ptr), C.c_void_p(bd.ptr), 1, C.c_void_p(ref_y.ptr),
         C.c_void_p(ref_m.ptr), C.c_void_p(ref_r.ptr))
    want = (ref_y.toArray()[: x.size], ref_m.toArray()[: n * g], ref_r.toArray()[: n * g])
    for _ in range(2):
        y, m, r = GPUTensor(ctx, 1, x.size), GPUTensor(ctx, 1, n * g), GPUTensor(ctx, 1, n * g)
        call("yl_groupnorm_silu_fwd_noalloc", ctx.handle, C.c_void_p(xd.ptr), n, c, h, w, g,
             1e-6, 0, C.c_void_p(gd.ptr), C.c_void_p(bd.ptr), 1, C.c_void_p(y.ptr),
             C.c_void_p(m.ptr), C.c_void_p(r.ptr))
        got = (y.toArray()[: x.size], m.toArray()[: n * g], r.toArray()[: n * g])
        for a, b in zip(got, want):
            assert _rel(a, b) < TOL
    # and against the oracle's GroupNorm + SiLU (double statistics) directly
    ref_y, _, _ = gn_silu_fwd(oracle, x.transpose(0, 3, 1, 2), g, 1e-6, ga, be)
    assert _rel(got[0].reshape(n, h, w, c).transpose(0, 3, 1, 2), ref_y) < 1e-5


def test_noalloc_rejects_requests_above_its_fixed_scratch(ctx):
    # 1024 groups on two 64x64 images need 2 * 256 * 2 * 1024 doubles > 131072
    n, c, h, w, g = 2, 4096, 64, 64, 1024
    x = GPUTensor(ctx, 1, n * h * w * c)
    y = GPUTensor(ctx, 1, n * h * w * c)
    m, r = GPUTensor(ctx, 1, n * g), GPUTensor(ctx, 1, n * g)
    st = lib().yl_groupnorm_silu_fwd_noalloc(ctx.handle, C.c_void_p(x.ptr), n, c, h, w, g, 1e-6,
                                             0, None, None, 1, C.c_void_p(y.ptr),
                                             C.c_void_p(m.ptr), C.c_void_p(r.ptr))
    assert st == 1  # YL_ERR_SHAPE
    assert b"fixed" in lib().yl_last_error_message()
