"""Checkpoint container formats (Train.swift:54-317, MotionTrainer.swift:49-155)
on CPU: byte layout, round trips, the reference's error codes, and the
flat-buffer <-> reference-matrix conversion of the trainer's tables."""
import json
import struct
from types import SimpleNamespace

import numpy as np
import pytest

from yumelayers_b200 import checkpoint as ck


def _mats(rng):
    return [rng.standard_normal((4, 27)).astype(np.float32),
            rng.standard_normal((4, 1)).astype(np.float32),
            rng.standard_normal((3, 5)).astype(np.float32)]


def test_layout_and_round_trip_with_optimizer(tmp_path, rng):
    mats = _mats(rng)
    mom = [rng.standard_normal(m.shape).astype(np.float32) for m in mats for _ in (0, 1)]
    p = tmp_path / "vae.safetensors"
    ck.save_state(p, mats, epoch=3, step=40, total_steps=100, fingerprint="abc",
                  optimizer=ck.OptimizerState(40, mom), model_width=2, latent_channels=32,
                  arch_version=6)
    raw = p.read_bytes()
    assert raw[:8] == b"<safeten"
    (hlen,) = struct.unpack_from("<Q", raw, 8)
    hdr = json.loads(raw[16:16 + hlen])
    assert hdr["p0"] == {"dtype": "F32", "shape": [4, 27], "data_offsets": [0, 432]}
    assert hdr["__metadata__"]["format"] == "YumeLayers VAE"
    assert hdr["__metadata__"]["order"] == ["p0", "p1", "p2"]
    assert hdr["adam.v2"]["shape"] == [3, 5]
    assert len(raw) == 16 + hlen + 3 * 4 * sum(m.size for m in mats)
    st = ck.load_state_with_meta(p)
    assert (st.epoch, st.step, st.fingerprint, st.model_width, st.latent_channels,
            st.arch_version) == (3, 40, "abc", 2, 32, 6)
    for a, b in zip(st.mats, mats):
        np.testing.assert_array_equal(a, b)
    assert st.optimizer.step == 40
    for a, b in zip(st.optimizer.moments, mom):
        np.testing.assert_array_equal(a, b)


def test_old_checkpoint_without_optimizer_and_defaults(tmp_path, rng):
    p = tmp_path / "old.safetensors"
    ck.save_state(p, _mats(rng))
    st = ck.load_state_with_meta(p)
    assert st.optimizer is None and st.epoch == 0 and st.latent_channels == 16
    assert st.model_width == 1 and st.arch_version == 1


def test_reference_error_codes(tmp_path, rng):
    mats = _mats(rng)
    bad = [m.copy() for m in mats]
    bad[1][0, 0] = np.nan
    with pytest.raises(ck.CheckpointError) as e:
        ck.save_state(tmp_path / "x", bad)
    assert e.value.code == 7
    with pytest.raises(ck.CheckpointError) as e:
        ck.save_state(tmp_path / "x", mats, optimizer=ck.OptimizerState(1, mats))  # odd count
    assert e.value.code == 12
    p = tmp_path / "ok"
    ck.save_state(p, mats)
    raw = bytearray(p.read_bytes())
    (tmp_path / "nomagic").write_bytes(raw[8:])
    with pytest.raises(ck.CheckpointError) as e:
        ck.load_state_with_meta(tmp_path / "nomagic")
    assert e.value.code == 9
    trunc = raw[: len(raw) - 8]
    (tmp_path / "trunc").write_bytes(trunc)
    with pytest.raises(ck.CheckpointError) as e:
        ck.load_state_with_meta(tmp_path / "trunc")
    assert e.value.code == 9
    long = bytearray(raw)
    long[8:16] = struct.pack("<Q", len(raw))
    (tmp_path / "long").write_bytes(long)
    with pytest.raises(ck.CheckpointError) as e:
        ck.load_state_with_meta(tmp_path / "long")
    assert e.value.code == 9


def test_incomplete_moment_pair_is_rejected(tmp_path, rng):
    mats = _mats(rng)
    p = tmp_path / "pair"
    ck.save_state(p, mats, optimizer=ck.OptimizerState(5, [mats[0], mats[0]]))
    raw = bytearray(p.read_bytes())
    (hlen,) = struct.unpack_from("<Q", raw, 8)
    hdr = json.loads(raw[16:16 + hlen])
    hdr["adam.x0"] = hdr.pop("adam.v0")
    new = json.dumps(hdr).encode()
    (tmp_path / "pair2").write_bytes(bytes(raw[:8]) + struct.pack("<Q", len(new)) + new +
                                     bytes(raw[16 + hlen:]))
    with pytest.raises(ck.CheckpointError) as e:
        ck.load_state_with_meta(tmp_path / "pair2")
    assert e.value.code == 12


def test_motion_checkpoint_round_trip(tmp_path, rng):
    mats = _mats(rng)
    p = tmp_path / "motion.safetensors"
    ck.save_motion_checkpoint(p, mats, {"latentDim": 32, "dimEmb": 128, "hidden": 512})
    raw = p.read_bytes()
    (hlen,) = struct.unpack_from("<Q", raw, 0)
    assert json.loads(raw[8:8 + hlen])["format"] == "YumeLayers Motion"
    got, meta = ck.load_motion_checkpoint(p)
    assert meta["latentDim"] == 32 and meta["order"] == ["p0", "p1", "p2"]
    for a, b in zip(got, mats):
        np.testing.assert_array_equal(a, b)
    (tmp_path / "junk").write_bytes(b"\x05" * 20)
    assert ck.load_motion_checkpoint(tmp_path / "junk") is None


def test_flat_matrix_conversion_matches_reference_layouts(rng):
    E = SimpleNamespace
    table = [E(name="c.weight", offset=0, shape=(3, 2, 3, 3)),   # conv: [4][9][4] stored
             E(name="c.bias", offset=144, shape=(3, 1, 1, 1)),
             E(name="l.weight", offset=148, shape=(2, 5, 0, 0)),  # Linear
             E(name="g.gamma", offset=160, shape=(6, 1, 1, 1))]
    w = rng.standard_normal((3, 2, 3, 3)).astype(np.float32)      # OIHW
    flat = np.zeros(168, np.float32)
    blk = np.zeros((4, 9, 4), np.float32)
    blk[:3, :, :2] = w.reshape(3, 2, 9).transpose(0, 2, 1)
    flat[:144] = blk.ravel()
    flat[144:147] = [1, 2, 3]
    lw = rng.standard_normal((2, 5)).astype(np.float32)
    flat[148:158] = lw.ravel()
    flat[160:166] = np.arange(6)
    mats = ck.flat_to_matrices(table, flat)
    np.testing.assert_array_equal(mats[0], w.reshape(3, 18))  # (oc, ic*k*k), OIHW order
    np.testing.assert_array_equal(mats[1][:, 0], [1, 2, 3])
    np.testing.assert_array_equal(mats[2], lw)
    back = ck.matrices_to_flat(table, mats, 168)
    np.testing.assert_array_equal(back, flat)
    with pytest.raises(ck.CheckpointError) as e:
        ck.matrices_to_flat(table, [mats[0].T] + mats[1:], 168)
    assert e.value.code == 11
