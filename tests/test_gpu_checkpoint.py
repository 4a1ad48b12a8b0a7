"""Resume from a checkpoint: weights, Adam moments and the step counter saved
from one trainer and loaded into another give bit-identical next steps
(resume without moments would restart Adam's bias correction, Train.swift:32-45)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_resume_is_bit_identical(tmp_path):
    from yumelayers_b200 import checkpoint as ck
    from yumelayers_b200 import synth
    from yumelayers_b200.trainer import Trainer, default_config
    clips = [synth.make_clip(21, h=32, w=48, width_padded=48)]
    batches = [synth.sample_batch(clips, 2, seed=s) for s in range(3)]
    a = Trainer(default_config(batch=2, height=32, width=48, seed=1))
    for frames, t in batches[:2]:
        a.step_host(frames, t)
    ck.save_trainer(a, tmp_path / "vae.safetensors", tmp_path / "motion.safetensors", epoch=1)
    b = Trainer(default_config(batch=2, height=32, width=48, seed=2))
    st = ck.load_trainer(b, tmp_path / "vae.safetensors", tmp_path / "motion.safetensors")
    assert st.optimizer is not None and b.step == a.step == 2
    for which in (0, 1):
        for kind in (0, 2, 3):
            np.testing.assert_array_equal(b.download(which, kind), a.download(which, kind))
    frames, t = batches[2]
    la, lb = a.step_host(frames, t), b.step_host(frames, t)
    np.testing.assert_array_equal(la, lb)
    for which in (0, 1):
        np.testing.assert_array_equal(b.download(which), a.download(which))
    a.close()
    b.close()


def test_driver_runs_epochs_with_checkpoints_and_resumes(tmp_path):
    from yumelayers_b200 import checkpoint as ck
    from yumelayers_b200 import driver as dv
    from yumelayers_b200 import synth
    from yumelayers_b200.trainer import Trainer, default_config
    clips = [synth.make_clip(31, h=32, w=48, width_padded=48)]
    vae_p, mot_p = tmp_path / "vae.safetensors", tmp_path / "motion.safetensors"

    def batch(ep, si):
        return synth.sample_batch(clips, 2, seed=100 * ep + si)

    def save_for(tr):
        return lambda ep_next, si: ck.save_trainer(tr, vae_p, mot_p, epoch=ep_next)

    a = Trainer(default_config(batch=2, height=32, width=48, seed=4))
    res = dv.run_training(a, batch, epochs=2, epoch_steps=2, save=save_for(a))
    assert res.epochs_done == 2 and res.steps == 4
    assert all(np.isfinite(v) for l in res.epoch_losses for v in l)
    st = ck.load_state_with_meta(vae_p)
    assert st.epoch == 2 and st.optimizer.step == 4
    b = Trainer(default_config(batch=2, height=32, width=48, seed=5))
    st = ck.load_trainer(b, vae_p, mot_p)
    res2 = dv.run_training(b, batch, epochs=3, epoch_steps=2, start_epoch=st.epoch,
                           save=save_for(b))
    assert res2.epochs_done == 1 and b.step == 6
    assert ck.load_state_with_meta(vae_p).epoch == 3
    a.close()
    b.close()
