"""The seeded synthetic workload data (yumelayers_b200/synth.py) keeps the
properties the benchmark configurations state: frames in [-1, 1] rendered
854 wide and edge-replicated to 856 (ImageIO.swift:52), 17-frame clips with
moving components, and samples (frame 0, frame 16, frame k, t = k/16) with k
in 1..15.  Host-only: no GPU."""
import numpy as np
import pytest

from yumelayers_b200 import synth


def test_frame_range_padding_and_determinism():
    f = synth.make_frame(3, h=40, w=94, width_padded=96)
    assert f.shape == (3, 40, 96) and f.dtype == np.float32
    assert f.min() >= -1.0 and f.max() <= 1.0
    np.testing.assert_array_equal(f[..., 94], f[..., 93])  # edge replication
    np.testing.assert_array_equal(f[..., 95], f[..., 93])
    np.testing.assert_array_equal(f, synth.make_frame(3, h=40, w=94, width_padded=96))
    assert not np.array_equal(f, synth.make_frame(4, h=40, w=94, width_padded=96))
    assert f.std() > 0.05  # blobs and gratings, not just the noise floor


def test_full_size_frame_shape():
    f = synth.make_frame(0)
    assert f.shape == (3, 480, 856)
    np.testing.assert_array_equal(f[..., 854:], np.repeat(f[..., 853:854], 2, axis=-1))


def test_clip_shape_range_and_motion():
    c = synth.make_clip(7, h=64, w=126, width_padded=128)
    assert c.shape == (17, 3, 64, 128) and c.dtype == np.float32
    assert c.min() >= -1.0 and c.max() <= 1.0
    np.testing.assert_array_equal(c[..., 126], c[..., 125])
    np.testing.assert_array_equal(c, synth.make_clip(7, h=64, w=126, width_padded=128))
    # every frame differs from the previous one by more than the N(0, 0.02) noise
    d = np.abs(np.diff(c, axis=0)).mean(axis=(1, 2, 3))
    assert (d > 0.03).all()


def test_pad_width_is_a_no_op_when_wide_enough():
    a = np.arange(12, dtype=np.float32).reshape(1, 3, 4)
    assert synth.pad_width(a, 4) is a
    assert synth.pad_width(a, 3) is a


@pytest.mark.parametrize("batch", [1, 8])
def test_sample_batch_picks_frames_0_16_k(batch):
    clips = [synth.make_clip(s, h=16, w=30, width_padded=32) for s in range(3)]
    frames, t = synth.sample_batch(clips, batch, seed=11)
    assert frames.shape == (3, batch, 3, 16, 32) and t.shape == (batch,)
    for b in range(batch):
        k = t[b] * 16.0
        assert k == round(k) and 1 <= k <= 15
        src = [j for j, c in enumerate(clips) if np.array_equal(frames[0, b], c[0])]
        assert len(src) == 1
        clip = clips[src[0]]
        np.testing.assert_array_equal(frames[1, b], clip[16])
        np.testing.assert_array_equal(frames[2, b], clip[int(round(k))])
    again, t2 = synth.sample_batch(clips, batch, seed=11)
    np.testing.assert_array_equal(again, frames)
    np.testing.assert_array_equal(t2, t)
