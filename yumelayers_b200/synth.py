"""Seeded synthetic frames and clips with the shapes and statistics of the
benchmark workloads (no dataset is used).

* ``make_frame``: a frame in [-1, 1] -- 24 random anisotropic Gaussian blobs
  (random RGB, sigma 10-80 px), 3 random-orientation sinusoidal gratings
  (period 8-64 px, amplitude 0.2) and N(0, 0.02) noise.
* ``make_clip``: 17 frames of such a background plus 4 textured elliptical
  sprites (radius 20-120 px); every component moves at a constant random
  velocity of up to 12 px/frame with wraparound, and a global brightness ramp
  of up to +-0.1 runs across the clip.
* Frames are rendered 854 wide and edge-replicated to 856 (the reference pads
  frames the same way, ImageIO.swift:52, ConvTrainerHelpers.swift:12-13).
* ``sample_batch``: (frame 0, frame 16, frame k, t = k/16), k uniform in 1..15.
"""
from __future__ import annotations

import numpy as np


def _blobs(rng, h, w, count=24, smin=10.0, smax=80.0):
    img = np.zeros((3, h, w), np.float32)
    yy = np.arange(h, dtype=np.float32)[:, None]
    xx = np.arange(w, dtype=np.float32)[None, :]
    for _ in range(count):
        cy, cx = rng.uniform(0, h), rng.uniform(0, w)
        sy, sx = rng.uniform(smin, smax, 2)
        th = rng.uniform(0, np.pi)
        col = rng.uniform(-1, 1, 3).astype(np.float32)
        r = 3.0 * max(sy, sx)
        y0, y1 = int(max(0, cy - r)), int(min(h, cy + r + 1))
        x0, x1 = int(max(0, cx - r)), int(min(w, cx + r + 1))
        if y0 >= y1 or x0 >= x1:
            continue
        dy = yy[y0:y1] - cy
        dx = xx[:, x0:x1] - cx
        c, s = np.cos(th), np.sin(th)
        u = (c * dx + s * dy) / sx
        v = (-s * dx + c * dy) / sy
        g = np.exp(-0.5 * (u * u + v * v)).astype(np.float32)
        img[:, y0:y1, x0:x1] += col[:, None, None] * g
    return img


def _gratings(rng, h, w, count=3, amp=0.2):
    yy = np.arange(h, dtype=np.float32)[:, None]
    xx = np.arange(w, dtype=np.float32)[None, :]
    out = np.zeros((3, h, w), np.float32)
    for _ in range(count):
        period = rng.uniform(8, 64)
        phi = rng.uniform(0, np.pi)
        phase = rng.uniform(0, 2 * np.pi)
        col = rng.uniform(-1, 1, 3).astype(np.float32)
        col /= max(np.abs(col).max(), 1e-3)
        wave = np.sin(2 * np.pi * (xx * np.cos(phi) + yy * np.sin(phi)) / period + phase)
        out += amp * col[:, None, None] * wave.astype(np.float32)
    return out


def pad_width(img: np.ndarray, width: int) -> np.ndarray:
    """Edge-replicate the last column(s) up to `width`."""
    extra = width - img.shape[-1]
    if extra <= 0:
        return img
    return np.concatenate([img, np.repeat(img[..., -1:], extra, axis=-1)], axis=-1)


def make_frame(seed: int, h: int = 480, w: int = 854, width_padded: int = 856) -> np.ndarray:
    """One config-3 frame, [3][h][width_padded] in [-1, 1]."""
    rng = np.random.default_rng(seed)
    img = _blobs(rng, h, w) + _gratings(rng, h, w)
    img += rng.normal(0, 0.02, img.shape).astype(np.float32)
    return pad_width(np.clip(img, -1, 1), width_padded)


def make_clip(seed: int, h: int = 480, w: int = 854, width_padded: int = 856,
              frames: int = 17) -> np.ndarray:
    """One config-5 clip, [frames][3][h][width_padded] in [-1, 1]."""
    rng = np.random.default_rng(seed)
    bg = _blobs(rng, h, w) + _gratings(rng, h, w)
    bg_v = rng.uniform(-12, 12, 2)
    sprites = []
    for _ in range(4):
        ry, rx = rng.uniform(20, 120, 2)
        sh, sw = int(2 * ry) + 1, int(2 * rx) + 1
        tex = _blobs(rng, sh, sw, count=6, smin=4.0, smax=30.0) + _gratings(rng, sh, sw, 1, 0.3)
        tex += rng.uniform(-0.5, 0.5, 3).astype(np.float32)[:, None, None]
        yy = (np.arange(sh, dtype=np.float32)[:, None] - ry) / ry
        xx = (np.arange(sw, dtype=np.float32)[None, :] - rx) / rx
        mask = (yy * yy + xx * xx <= 1.0).astype(np.float32)
        pos = rng.uniform(0, [h, w])
        vel = rng.uniform(-12, 12, 2)
        sprites.append((tex, mask, pos, vel))
    ramp = rng.uniform(-0.1, 0.1)
    out = np.empty((frames, 3, h, width_padded), np.float32)
    for f in range(frames):
        img = np.roll(bg, (int(round(bg_v[0] * f)), int(round(bg_v[1] * f))), axis=(1, 2)).copy()
        for tex, mask, pos, vel in sprites:
            sh, sw = mask.shape
            y0 = int(round(pos[0] + vel[0] * f)) % h
            x0 = int(round(pos[1] + vel[1] * f)) % w
            ys = (y0 + np.arange(sh)) % h
            xs = (x0 + np.arange(sw)) % w
            region = img[:, ys[:, None], xs[None, :]]
            img[:, ys[:, None], xs[None, :]] = region * (1 - mask) + tex * mask
        img += ramp * f / (frames - 1)
        img += rng.normal(0, 0.02, img.shape).astype(np.float32)
        out[f] = pad_width(np.clip(img, -1, 1), width_padded)
    return out


def sample_batch(clips: list[np.ndarray], batch: int, seed: int,
                 out: np.ndarray | None = None) -> tuple[np.ndarray, np.ndarray]:
    """(frames [3][batch][3][H][W] = frame 0, frame 16, frame k; t [batch] = k/16)."""
    rng = np.random.default_rng(seed)
    f, c, h, w = clips[0].shape
    if out is None:
        out = np.empty((3, batch, c, h, w), np.float32)
    t = np.empty(batch, np.float32)
    for b in range(batch):
        clip = clips[int(rng.integers(len(clips)))]
        k = int(rng.integers(1, 16))
        out[0, b] = clip[0]
        out[1, b] = clip[16]
        out[2, b] = clip[k]
        t[b] = k / 16.0
    return out, t
