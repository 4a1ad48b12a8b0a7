"""The failure paths of the bounded waits, driven without a GPU fault.

The reference guards a hung GPU on the host: GpuSession.end waits with a
deadline and exits with 70 when it passes (GpuTraining.swift:72-112, policy
GpuWaitPolicy.swift:54-61, tested by TestGroup1.swift:129 testGpuWaitPolicy).
This backend bounds every device-side wait as well and returns a status:

* a kernel whose wait nothing satisfies gives up after the context's wait
  limit and the host reads YL_ERR_TIMEOUT;
* the conv kernels, given a wait limit shorter than their own pipeline
  latency, take that same exit on every warp (drain their copies and MMAs in
  flight, release TMEM) and the context stays usable;
* yl_session_end returns YL_ERR_TIMEOUT when its deadline passes before the
  work ends, and a later end succeeds.
"""
import time

import numpy as np
import pytest

from oracle_lib import conv2d_fwd, f32, rel_l2
from yumelayers_b200._lib import YumeError, call

pytestmark = pytest.mark.gpu
YL_ERR_TIMEOUT = 3


def test_device_wait_gives_up_with_timeout_status(ctx):
    ctx.check_device_errors()  # start from a clean error word
    try:
        ctx.set_wait_limit(1_000_000)  # ~0.6 ms at the SM clock
        call("yl_debug_wait_probe", ctx.handle)
        with pytest.raises(YumeError) as ei:
            ctx.check_device_errors()
        assert ei.value.status == YL_ERR_TIMEOUT
        ctx.check_device_errors()  # the word was cleared
    finally:
        ctx.set_wait_limit(0)


def test_conv_kernels_take_the_timeout_exit_and_the_context_recovers(oracle, ctx):
    """A 200-cycle limit is shorter than one TMA load: the producer, MMA and
    epilogue warps of the forward (halo) and filter-gradient kernels all give
    up, report YL_DEVERR_TIMEOUT and exit; with the default limit restored the
    same convs are exact again."""
    from yumelayers_b200 import ops
    rng = np.random.default_rng(0)
    x = f32(rng.standard_normal((2, 128, 64, 64)))
    wt = f32(rng.uniform(-0.03, 0.03, (128, 128, 3, 3)))
    dy = f32(rng.standard_normal((2, 128, 64, 64)))
    ctx.check_device_errors()
    try:
        ctx.set_wait_limit(200)
        ops.conv2d_fwd(x, wt, None, ctx=ctx)
        assert ctx.last_kernel(0) == "conv_tma_fprop_kernel<128, 2, 1, 1>"
        with pytest.raises(YumeError) as ei:
            ctx.check_device_errors()
        assert ei.value.status == YL_ERR_TIMEOUT
        ops.conv2d_bwd_filter(x, dy, wt.shape, ctx=ctx)
        assert ctx.last_kernel(1).startswith("conv_tma_wgrad_kernel")
        with pytest.raises(YumeError) as ei:
            ctx.check_device_errors()
        assert ei.value.status == YL_ERR_TIMEOUT
    finally:
        ctx.set_wait_limit(0)
    y = ops.conv2d_fwd(x, wt, None, ctx=ctx)
    ctx.check_device_errors()
    assert rel_l2(y, conv2d_fwd(oracle, x, wt, None)) < 1e-3


def test_session_end_deadline_then_recovery(ctx):
    from yumelayers_b200.session import GpuSession
    s = GpuSession(ctx)
    s.begin()
    call("yl_debug_spin", ctx.handle, 0.3)
    t0 = time.monotonic()
    with pytest.raises(YumeError) as ei:
        s.end(timeout_s=0.05)
    assert ei.value.status == YL_ERR_TIMEOUT
    assert time.monotonic() - t0 < 0.25  # the deadline, not the kernel, ended the wait
    s.end(timeout_s=5.0)  # the spin finishes; the next end succeeds
