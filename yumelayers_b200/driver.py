"""Training driver around the joint step: epochs of steps with per-step
cancel/pause gates, a NaN abort, epoch reports, plateau warning, periodic and
per-epoch checkpoints, and resume (the caller side of the hot path:
TrainConvVAE.swift:327-430 runStep / runEpochs, TrainingControl.swift:108-118,
TrainingHelpers.swift:30-60, ConvVAEHelpers.swift:40-49).
"""
from __future__ import annotations

import math
import threading
import time
from dataclasses import dataclass, field


class TrainingNaNError(RuntimeError):
    """A non-finite loss: training stops and no checkpoint is written
    (TrainConvVAE.swift:337-341)."""


class TrainingControl:
    """Cancel and pause flags shared with the caller (TrainingControl.swift)."""

    def __init__(self):
        self._cv = threading.Condition()
        self._cancelled = False
        self._paused = False

    @property
    def cancelled(self) -> bool:
        with self._cv:
            return self._cancelled

    @property
    def paused(self) -> bool:
        with self._cv:
            return self._paused

    def reset(self) -> None:
        with self._cv:
            self._cancelled = self._paused = False
            self._cv.notify_all()

    def cancel(self) -> None:
        with self._cv:
            self._cancelled = True
            self._cv.notify_all()

    def pause(self, on: bool = True) -> None:
        with self._cv:
            self._paused = on
            self._cv.notify_all()

    def wait_while_paused(self, timeout_s: float | None = None) -> None:
        with self._cv:
            self._cv.wait_for(lambda: not self._paused or self._cancelled, timeout_s)


def training_gate_action(cancelled: bool, paused: bool) -> str:
    """'stop' | 'wait' | 'proceed' (trainingGateAction, TrainingControl.swift:114-118)."""
    if cancelled:
        return "stop"
    if paused:
        return "wait"
    return "proceed"


def plateau_detected(losses, rel_tolerance: float = 0.02, window: int = 3) -> bool:
    """Relative improvement over the last `window` epochs below the tolerance
    (plateauDetected, TrainingHelpers.swift:30-37)."""
    if window < 1 or len(losses) < window + 1:
        return False
    recent = list(losses)[-(window + 1):]
    first, last = recent[0], recent[-1]
    if not (math.isfinite(first) and math.isfinite(last)) or first <= 0:
        return False
    return (first - last) / first < rel_tolerance


def resume_warmup_factor(step: int, warmup_steps: int) -> float:
    """Learning-rate ramp after resuming without optimizer state
    (resumeWarmupFactor, ConvVAEHelpers.swift:40-49)."""
    if warmup_steps <= 0:
        return 1.0
    return min(1.0, max(step, 1) / warmup_steps)


@dataclass
class RunResult:
    epochs_done: int = 0
    stopped: bool = False
    steps: int = 0
    epoch_losses: list = field(default_factory=list)  # mean (vae, motion) per epoch
    plateau: bool = False


def run_training(trainer, next_batch, *, epochs: int, epoch_steps: int, start_epoch: int = 0,
                 control: TrainingControl | None = None, save=None, save_every: int = 500,
                 warmup_steps: int = 0, on_progress=None) -> RunResult:
    """Epochs [start_epoch, epochs) of `epoch_steps` joint steps.

    next_batch(epoch, step) -> (frames [3][B][3][H][W], t [B]) host arrays.
    save(epoch_next, step_in_epoch) writes a checkpoint (every `save_every`
    steps and after each completed epoch); it is never called after a NaN.
    warmup_steps > 0 ramps both learning rates over the first steps of this
    run (for resumes without optimizer state).  Cancel is checked before every
    step; a stopped epoch is neither reported nor checkpointed.
    """
    control = control or TrainingControl()
    res = RunResult()
    base = (trainer.cfg.lr_vae, trainer.cfg.lr_motion)
    run_step = 0
    for ep in range(max(0, start_epoch), epochs):
        if control.cancelled:
            res.stopped = True
            break
        sums, done, stopped = [0.0, 0.0], 0, False
        for si in range(epoch_steps):
            action = training_gate_action(control.cancelled, control.paused)
            if action == "wait":
                control.wait_while_paused()
                action = "stop" if control.cancelled else "proceed"
            if action == "stop":
                stopped = True
                break
            if warmup_steps > 0:
                f = resume_warmup_factor(run_step + 1, warmup_steps)
                trainer.set_config(lr_vae=base[0] * f, lr_motion=base[1] * f)
            t0 = time.perf_counter()
            frames, t = next_batch(ep, si)
            losses = trainer.step_host(frames, t)
            if not all(math.isfinite(float(v)) for v in losses):
                raise TrainingNaNError(f"non-finite loss {list(losses)} at epoch {ep} step {si}")
            sums[0] += float(losses[0])
            sums[1] += float(losses[1])
            done += 1
            run_step += 1
            res.steps += 1
            if on_progress:
                on_progress(ep, si, [float(v) for v in losses], time.perf_counter() - t0)
            if save and save_every > 0 and (si + 1) % save_every == 0 and si + 1 < epoch_steps:
                save(ep, si + 1)
        if stopped:
            res.stopped = True
            break
        res.epoch_losses.append((sums[0] / max(done, 1), sums[1] / max(done, 1)))
        res.epochs_done += 1
        if not res.plateau and plateau_detected([l[0] + l[1] for l in res.epoch_losses]):
            res.plateau = True
        if save:
            save(ep + 1, 0)
    if warmup_steps > 0:
        trainer.set_config(lr_vae=base[0], lr_motion=base[1])
    return res
