"""Data-parallel training over NCCL on two GPUs.

Each rank first runs one step of a single-GPU trainer (no communicator) on
its own batch from the same initial weights.  Then the two ranks train
together for three steps with different per-rank batches, and the test checks:

* after the first data-parallel step, each rank's gradient buffer (the
  all-reduce runs in place) equals the sum of the two single-GPU gradients --
  a bucket reduced while a backward kernel still wrote into it would break
  this while leaving the ranks identical to each other;
* the first step's loss equals the mean of the two single-GPU losses;
* after three steps both ranks hold bit-identical parameters and losses.

Skipped when fewer than two GPUs are visible."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import hashlib
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from yumelayers_b200 import synth
    from yumelayers_b200.session import Context
    from yumelayers_b200.trainer import Comm, Trainer, default_config, share_unique_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        ctx = Context(rank)
        cfg = default_config(batch=2, height=32, width=48, seed=11)
        clips = [synth.make_clip(50 + rank, h=32, w=48, width_padded=48)]
        batches = [synth.sample_batch(clips, 2, seed=7 * rank + step) for step in range(3)]
        solo = Trainer(cfg, ctx=ctx)  # this rank's batch alone, no communicator
        solo_loss = solo.step_host(*batches[0]).tolist()
        solo_grads = [solo.download(w, kind=1) for w in (0, 1)]
        solo.close()
        uid = share_unique_id(rank, Comm.unique_id, lambda o: dist.broadcast_object_list(o, src=0))
        comm = Comm(ctx, uid, rank, world)
        tr = Trainer(cfg, ctx=ctx, comm=comm)
        losses, dp_grads = [], None
        for step in range(3):
            losses.append(tr.step_host(*batches[step]).tolist())
            if step == 0:
                dp_grads = [tr.download(w, kind=1) for w in (0, 1)]
        digests = [hashlib.sha256(tr.download(w).tobytes()).hexdigest() for w in (0, 1)]
        out.put((rank, digests, losses, solo_loss, solo_grads, dp_grads))
        tr.close()
        comm.close()
    finally:
        dist.destroy_process_group()


def test_two_ranks_keep_identical_parameters():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][1] == res[1][1], "ranks diverged"
    np.testing.assert_allclose(res[0][2], res[1][2], rtol=0, atol=0)
    assert all(np.isfinite(v).all() for v in res[0][2])
    # the reduced gradient is the sum of the single-GPU gradients (fp32 a + b
    # of two operands is the same in either order, so this is near exact)
    for w in (0, 1):
        want = res[0][4][w].astype(np.float64) + res[1][4][w]
        for r in (0, 1):
            got = res[r][5][w].astype(np.float64)
            rel = np.linalg.norm(got - want) / np.linalg.norm(want)
            assert rel < 1e-6, (w, r, rel)
    mean_solo = (np.array(res[0][3]) + np.array(res[1][3])) / 2
    np.testing.assert_allclose(res[0][2][0], mean_solo, rtol=1e-6)
