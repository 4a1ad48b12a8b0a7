"""The inference path on the GPU (encode A and B -> motion net or smoothstep
lerp -> decode, Interpolation.swift:263-373) against the oracle's composition
of the same forward passes, from the trainer's own weights."""
import numpy as np
import pytest

from oracle_lib import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-2  # relative L2 of each decoded frame after ~60 tf32 convs (fp32 oracle)


def _smoothstep(t):
    x = min(max(t, 0.0), 1.0)
    return x * x * (3 - 2 * x)


@pytest.mark.parametrize("mode", [0, 1])
def test_interpolation_matches_oracle(mode):
    import nets
    from yumelayers_b200.trainer import Trainer, default_config, interpolation_plan
    tr = Trainer(default_config(batch=2, height=32, width=48, seed=9))
    rng = np.random.default_rng(3)
    a = np.clip(rng.standard_normal((3, 32, 48)) * 0.5, -1, 1).astype(np.float32)
    b = np.clip(rng.standard_normal((3, 32, 48)) * 0.5, -1, 1).astype(np.float32)
    times = interpolation_plan(0.5, 10)  # 5 frames: 3 interior, decoded in 2 groups
    got = tr.interpolate(a, b, times, mode)
    assert got.shape == (5, 3, 32, 48)
    np.testing.assert_array_equal(got[0], a)
    np.testing.assert_array_equal(got[-1], b)

    ops = nets.Ops()
    vae = nets.VAE(ops, nets.Params(tr.param_table(0), tr.download(0)))
    unet = nets.UNet(ops, nets.Params(tr.param_table(1), tr.download(1)))
    e, _ = vae.encode(np.stack([a, b]))
    mu = e[:, :32]
    for i in range(1, times.size - 1):
        t = float(times[i])
        if mode == 0:
            z = unet.predict(mu[:1], mu[1:], np.array([t], np.float32))
        else:
            s = _smoothstep(t)
            z = (mu[:1] + (mu[1:] - mu[:1]) * np.float32(s)).astype(np.float32)
        ref = vae.decode(z, {})[0, :3]
        assert rel_l2(got[i], ref) < TOL, (i, rel_l2(got[i], ref))
    tr.close()
