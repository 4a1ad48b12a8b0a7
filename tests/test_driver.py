"""Training driver on CPU with a stand-in trainer: gates, NaN abort, epoch
bookkeeping, checkpoint calls, warm-up (TrainConvVAE.swift:327-430,
TrainingControl.swift:114-118, TrainingHelpers.swift:30-37,
ConvVAEHelpers.swift:40-49)."""
import threading
from types import SimpleNamespace

import numpy as np
import pytest

from yumelayers_b200 import driver as dv


class FakeTrainer:
    def __init__(self, losses):
        self.cfg = SimpleNamespace(lr_vae=2e-4, lr_motion=1e-4)
        self.losses = list(losses)
        self.lrs = []

    def set_config(self, **kw):
        for k, v in kw.items():
            setattr(self.cfg, k, v)

    def step_host(self, frames, t):
        self.lrs.append((self.cfg.lr_vae, self.cfg.lr_motion))
        return np.array(self.losses.pop(0), np.float32)


def _batch(ep, si):
    return np.zeros((3, 1, 3, 8, 8), np.float32), np.zeros(1, np.float32)


def test_pure_helpers():
    assert dv.training_gate_action(True, True) == "stop"
    assert dv.training_gate_action(False, True) == "wait"
    assert dv.training_gate_action(False, False) == "proceed"
    assert not dv.plateau_detected([1.0, 0.9, 0.8])
    assert dv.plateau_detected([1.0, 0.995, 0.99, 0.985])
    assert not dv.plateau_detected([1.0, 0.9, 0.85, 0.8])
    assert not dv.plateau_detected([float("nan"), 1, 1, 1])
    assert dv.resume_warmup_factor(0, 10) == 0.1 and dv.resume_warmup_factor(20, 10) == 1.0
    assert dv.resume_warmup_factor(5, 0) == 1.0


def test_epochs_checkpoints_and_warmup():
    tr = FakeTrainer([[1.0, 0.5]] * 8)
    saves = []
    res = dv.run_training(tr, _batch, epochs=5, epoch_steps=2, start_epoch=1,
                          save=lambda e, s: saves.append((e, s)), save_every=1, warmup_steps=4)
    assert res.epochs_done == 4 and res.steps == 8 and not res.stopped
    assert saves == [(1, 1), (2, 0), (2, 1), (3, 0), (3, 1), (4, 0), (4, 1), (5, 0)]
    assert res.epoch_losses == [(1.0, 0.5)] * 4
    assert res.plateau  # no improvement over four epochs
    np.testing.assert_allclose([l[0] for l in tr.lrs[:4]], [0.5e-4, 1e-4, 1.5e-4, 2e-4])
    assert tr.cfg.lr_vae == 2e-4  # restored


def test_nan_aborts_without_checkpoint():
    tr = FakeTrainer([[1.0, 0.5], [float("nan"), 0.5]])
    saves = []
    with pytest.raises(dv.TrainingNaNError):
        dv.run_training(tr, _batch, epochs=2, epoch_steps=2, save=lambda e, s: saves.append(e))
    assert saves == []


def test_cancel_stops_before_the_next_step_and_skips_the_epoch_checkpoint():
    ctl = dv.TrainingControl()
    tr = FakeTrainer([[1.0, 0.5]] * 10)
    saves = []

    def progress(ep, si, losses, secs):
        if si == 1:
            ctl.cancel()
    res = dv.run_training(tr, _batch, epochs=3, epoch_steps=4, control=ctl,
                          save=lambda e, s: saves.append(e), save_every=0, on_progress=progress)
    assert res.stopped and res.steps == 2 and res.epochs_done == 0 and saves == []


def test_pause_waits_until_resumed():
    ctl = dv.TrainingControl()
    ctl.pause(True)
    tr = FakeTrainer([[1.0, 0.5]] * 2)
    timer = threading.Timer(0.2, lambda: ctl.pause(False))
    timer.start()
    res = dv.run_training(tr, _batch, epochs=1, epoch_steps=2, control=ctl)
    timer.join()
    assert res.steps == 2 and not res.stopped
