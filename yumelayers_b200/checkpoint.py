"""Checkpoints in the reference's container formats, for the trainer's models.

VAE checkpoints follow saveState / loadStateWithMeta (Train.swift:54-317):

    b"<safeten" | u64 little-endian header length | JSON header | F32 data

The header maps "p0".."pN" (weights, in order) and "adam.m<i>"/"adam.v<i>"
(the Adam moments of weight i, optional) to {"dtype": "F32", "shape": [rows,
cols], "data_offsets": [begin, end]}; "__metadata__" holds format "YumeLayers
VAE", order, epoch, step, totalSteps, dataFingerprint, modelWidth,
latentChannels, archVersion and optimizerStep.  Weights must be finite
(error code 7), moments come in complete m/v pairs (code 12), malformed files
raise code 9 -- the NSError codes of the reference.

Motion-network checkpoints follow saveMotionCheckpoint / loadMotionCheckpoint
(MotionTrainer.swift:49-155): the same tensor entries without the magic, with
the metadata as top-level keys (format "YumeLayers Motion", order, ...).

Matrices use the reference's layouts: conv weights (oc, ic*k*k) in OIHW order
(ConvGPU.swift:18), Linear weights (oc, ic) (DenoiserMLP.swift:51-54), vectors
(n, 1).  The trainer's flat parameter buffers are converted on the host.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field

import numpy as np

MAGIC = b"<safeten"


class CheckpointError(RuntimeError):
    """A checkpoint the reference would reject; `code` is its NSError code."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


@dataclass
class OptimizerState:
    step: int
    moments: list  # m0, v0, m1, v1, ... (one pair per weight matrix)


@dataclass
class CheckpointState:
    mats: list
    epoch: int = 0
    step: int = 0
    fingerprint: str | None = None
    optimizer: OptimizerState | None = None
    model_width: int = 1
    latent_channels: int = 16
    arch_version: int = 1
    meta: dict = field(default_factory=dict)


def _matrix(a) -> np.ndarray:
    m = np.asarray(a, dtype=np.float32)
    if m.ndim == 1:
        m = m.reshape(-1, 1)
    if m.ndim != 2:
        raise CheckpointError(9, f"checkpoint tensors are matrices, got shape {m.shape}")
    return np.ascontiguousarray(m)


def _entries(names, mats, offset=0):
    hdr, blobs = {}, []
    for name, m in zip(names, mats):
        nbytes = m.size * 4
        hdr[name] = {"dtype": "F32", "shape": [int(m.shape[0]), int(m.shape[1])],
                     "data_offsets": [offset, offset + nbytes]}
        blobs.append(m.astype("<f4").tobytes())
        offset += nbytes
    return hdr, blobs, offset


def save_state(path, mats, epoch=None, step=None, total_steps=None, fingerprint=None,
               optimizer: OptimizerState | None = None, model_width=None, latent_channels=None,
               arch_version=None, extra_meta: dict | None = None) -> None:
    """saveState (Train.swift:54-131)."""
    mats = [_matrix(m) for m in mats]
    for i, m in enumerate(mats):
        if not np.isfinite(m).all():
            raise CheckpointError(7, f"NaN/Inf in weights p{i}: checkpoint not saved")
    order = [f"p{i}" for i in range(len(mats))]
    hdr, blobs, offset = _entries(order, mats)
    meta = {"format": "YumeLayers VAE", "order": order}
    for key, val in (("epoch", epoch), ("step", step), ("totalSteps", total_steps),
                     ("dataFingerprint", fingerprint), ("modelWidth", model_width),
                     ("latentChannels", latent_channels), ("archVersion", arch_version)):
        if val is not None:
            meta[key] = val
    if optimizer is not None:
        moments = [_matrix(m) for m in optimizer.moments]
        if len(moments) % 2:
            raise CheckpointError(12, "optimizer state damaged: moments must come in m/v pairs")
        for i, m in enumerate(moments):
            if not np.isfinite(m).all():
                raise CheckpointError(12, f"NaN/Inf in optimizer moment #{i}: not saved")
        names = [f"adam.{'m' if i % 2 == 0 else 'v'}{i // 2}" for i in range(len(moments))]
        h2, b2, offset = _entries(names, moments, offset)
        hdr.update(h2)
        blobs += b2
        meta["optimizerStep"] = int(optimizer.step)
    if extra_meta:
        meta.update(extra_meta)
    hdr["__metadata__"] = meta
    header = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        for b in blobs:
            f.write(b)


def _parse_entries(obj: dict, base: int, size: int):
    entries = []
    for k, v in obj.items():
        if k == "__metadata__":
            continue
        try:
            shape, off = v["shape"], v["data_offsets"]
            ok = v["dtype"] == "F32" and len(shape) == 2 and len(off) == 2
        except (TypeError, KeyError):
            ok = False
        if not ok:
            raise CheckpointError(9, f"checkpoint entry {k!r} is not an F32 matrix")
        entries.append((k, int(shape[0]), int(shape[1]), int(off[0]), int(off[1])))
    entries.sort(key=lambda e: e[3])
    return entries


def _decode(e, data: bytes, base: int) -> np.ndarray:
    name, rows, cols, start, end = e
    n = rows * cols
    if (rows <= 0 or cols <= 0 or start < 0 or end < start or end > len(data) - base
            or end - start != n * 4):
        raise CheckpointError(9, f"checkpoint damaged (data of {name})")
    m = np.frombuffer(data, dtype="<f4", count=n, offset=base + start).astype(np.float32)
    if not np.isfinite(m).all():
        raise CheckpointError(9, f"checkpoint damaged (non-finite values in {name})")
    return m.reshape(rows, cols)


def load_state_with_meta(path) -> CheckpointState:
    """loadStateWithMeta (Train.swift:267-317)."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 16 or data[:8] != MAGIC:
        raise CheckpointError(9, "checkpoint is not in the safetensors format")
    (hlen,) = struct.unpack_from("<Q", data, 8)
    if hlen > len(data) - 16:
        raise CheckpointError(9, "checkpoint damaged (length)")
    try:
        obj = json.loads(data[16:16 + hlen])
        assert isinstance(obj, dict)
    except Exception:
        raise CheckpointError(9, "checkpoint damaged (header)") from None
    base = 16 + hlen
    meta = obj.get("__metadata__") if isinstance(obj.get("__metadata__"), dict) else {}

    def num(key, default, lo=None):
        v = meta.get(key, default)
        v = int(v) if isinstance(v, (int, float)) else default
        return max(lo, v) if lo is not None else v

    entries = _parse_entries(obj, base, len(data))
    weights = [e for e in entries if not e[0].startswith("adam.")]
    moments = [e for e in entries if e[0].startswith("adam.")]
    mats = [_decode(e, data, base) for e in weights]
    opt = None
    if moments:
        pm, pv = {}, {}
        for e in moments:
            kind, idx = e[0][5:6], e[0][6:]
            if kind not in ("m", "v") or not idx.isdigit():
                raise CheckpointError(12, f"bad optimizer moment name: {e[0]}")
            (pm if kind == "m" else pv)[int(idx)] = _decode(e, data, base)
        flat = []
        for idx in sorted(pm):
            if idx not in pv:
                raise CheckpointError(12, f"optimizer state damaged: pair {idx} incomplete")
            flat += [pm[idx], pv[idx]]
        opt = OptimizerState(num("optimizerStep", 0), flat)
    fp = meta.get("dataFingerprint")
    return CheckpointState(mats, num("epoch", 0), num("step", 0),
                           fp if isinstance(fp, str) else None, opt,
                           num("modelWidth", 1, 1), num("latentChannels", 16, 1),
                           num("archVersion", 1, 1), dict(meta))


def save_motion_checkpoint(path, mats, meta: dict) -> None:
    """saveMotionCheckpoint (MotionTrainer.swift:49-94): no magic, metadata as
    top-level header keys."""
    mats = [_matrix(m) for m in mats]
    for i, m in enumerate(mats):
        if not np.isfinite(m).all():
            raise CheckpointError(1, f"NaN/Inf in motion-network weights p{i}")
    order = [f"p{i}" for i in range(len(mats))]
    hdr, blobs, _ = _entries(order, mats)
    hdr.update(meta)
    hdr["format"] = "YumeLayers Motion"
    hdr["order"] = order
    header = json.dumps(hdr).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header)
        for b in blobs:
            f.write(b)


def load_motion_checkpoint(path):
    """loadMotionCheckpoint (MotionTrainer.swift:103-155): (mats, meta), or None
    for a damaged or foreign file."""
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 8:
        return None
    (hlen,) = struct.unpack_from("<Q", data, 0)
    if hlen <= 0 or 8 + hlen > len(data):
        return None
    try:
        obj = json.loads(data[8:8 + hlen])
    except Exception:
        return None
    if not isinstance(obj, dict) or obj.get("format") != "YumeLayers Motion" or not isinstance(
            obj.get("order"), list):
        return None
    mats = []
    for name in obj["order"]:
        info = obj.get(name)
        try:
            rows, cols = info["shape"]
            o0, o1 = info["data_offsets"]
        except (TypeError, KeyError, ValueError):
            return None
        start, end = 8 + hlen + o0, 8 + hlen + o1
        if end > len(data) or end <= start or end - start != rows * cols * 4:
            return None
        mats.append(np.frombuffer(data, "<f4", rows * cols, start).reshape(rows, cols).copy())
    meta = {k: v for k, v in obj.items() if not (isinstance(v, dict) and "data_offsets" in v)}
    return mats, meta


# ------------------------------------------------------------------ trainer glue
def _r4(x: int) -> int:
    return (x + 3) & ~3


def flat_to_matrices(table, flat: np.ndarray) -> list:
    """The trainer's flat buffer as reference-layout matrices, in table order."""
    out = []
    for e in table:
        d0, d1, d2, d3 = e.shape
        if e.name.endswith(".weight") and d2 >= 1:  # conv: [oc_p][k*k][ic_p] -> (oc, ic*k*k)
            kk, icp = d2 * d3, _r4(d1)
            blk = flat[e.offset:e.offset + _r4(d0) * kk * icp].reshape(_r4(d0), kk, icp)
            out.append(np.ascontiguousarray(blk[:d0, :, :d1].transpose(0, 2, 1)).reshape(d0, d1 * kk))
        elif e.name.endswith(".weight"):  # Linear (oc, ic)
            out.append(flat[e.offset:e.offset + d0 * d1].reshape(d0, d1).copy())
        else:
            out.append(flat[e.offset:e.offset + d0].reshape(d0, 1).copy())
    return out


def matrices_to_flat(table, mats, count: int) -> np.ndarray:
    """Inverse of flat_to_matrices (padding lanes zero); checks every shape first
    (the reference validates all layers before copying any, ConvGPU.swift:557-571)."""
    if len(mats) < len(table):
        raise CheckpointError(10, f"checkpoint: {len(table)} matrices needed, {len(mats)} found")
    expect = []
    for e in table:
        d0, d1, d2, d3 = e.shape
        expect.append((d0, d1 * d2 * d3) if e.name.endswith(".weight") and d2 >= 1 else
                      (d0, d1) if e.name.endswith(".weight") else (d0, 1))
    for i, (m, shp) in enumerate(zip(mats, expect)):
        if tuple(np.asarray(m).shape) != shp:
            raise CheckpointError(11, f"checkpoint: shape mismatch of layer {i} "
                                      f"({np.asarray(m).shape} vs {shp})")
    flat = np.zeros(count, np.float32)
    for e, m in zip(table, mats):
        d0, d1, d2, d3 = e.shape
        m = np.asarray(m, np.float32)
        if e.name.endswith(".weight") and d2 >= 1:
            kk, icp = d2 * d3, _r4(d1)
            blk = np.zeros((_r4(d0), kk, icp), np.float32)
            blk[:d0, :, :d1] = m.reshape(d0, d1, kk).transpose(0, 2, 1)
            flat[e.offset:e.offset + blk.size] = blk.ravel()
        else:
            flat[e.offset:e.offset + m.size] = m.ravel()
    return flat


VAE_ARCH = 6     # GroupNorm32+SiLU residual VAE, 128/256 channels, 32-channel latent
MOTION_ARCH = 6  # latent-space conv U-Net with time MLP (the reference's MLP is 5)


def save_trainer(tr, vae_path, motion_path=None, epoch=None, fingerprint=None) -> None:
    """Both models of a Trainer with their Adam moments and step counter."""
    step = tr.step
    for which, path in ((0, vae_path), (1, motion_path)):
        if path is None:
            continue
        table = tr.param_table(which)
        mats = flat_to_matrices(table, tr.download(which, 0))
        moments = []
        for m, v in zip(flat_to_matrices(table, tr.download(which, 2)),
                        flat_to_matrices(table, tr.download(which, 3))):
            moments += [m, v]
        if which == 0:
            save_state(path, mats, epoch=epoch, step=step, fingerprint=fingerprint,
                       optimizer=OptimizerState(step, moments), latent_channels=32,
                       arch_version=VAE_ARCH,
                       extra_meta={"names": [e.name for e in table]})
        else:
            save_state(path, mats, epoch=epoch, step=step, fingerprint=fingerprint,
                       optimizer=OptimizerState(step, moments), arch_version=MOTION_ARCH,
                       extra_meta={"format": "YumeLayers Motion UNet",
                                   "names": [e.name for e in table]})


def load_trainer(tr, vae_path=None, motion_path=None) -> CheckpointState | None:
    """Weights, Adam moments and step counter back into a Trainer; returns the
    last loaded state."""
    state = None
    for which, path in ((0, vae_path), (1, motion_path)):
        if path is None:
            continue
        state = load_state_with_meta(path)
        table = tr.param_table(which)
        n = tr.param_count(which)
        flat = matrices_to_flat(table, state.mats, n)
        if state.optimizer is not None:
            mom = state.optimizer.moments
            if len(mom) != 2 * len(table):
                raise CheckpointError(13, f"optimizer state: {2 * len(table)} moments needed, "
                                          f"{len(mom)} found")
            tr.upload(which, matrices_to_flat(table, mom[0::2], n), kind=2)
            tr.upload(which, matrices_to_flat(table, mom[1::2], n), kind=3)
        tr.upload(which, flat, kind=0)
        if state.optimizer is not None:
            tr.step = state.optimizer.step
    return state
