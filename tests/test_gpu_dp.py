"""Data-parallel training over NCCL on two GPUs: after a few joint steps with
different per-rank batches, every rank holds bit-identical parameters (the
bucketed gradient all-reduce and the loss all-reduce ran on every rank in
the same order), and the averaged losses agree across ranks.  Skipped when
fewer than two GPUs are visible."""
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
        uid = share_unique_id(rank, Comm.unique_id, lambda o: dist.broadcast_object_list(o, src=0))
        comm = Comm(ctx, uid, rank, world)
        tr = Trainer(default_config(batch=2, height=32, width=48, seed=11), ctx=ctx, comm=comm)
        clips = [synth.make_clip(50 + rank, h=32, w=48, width_padded=48)]
        losses = []
        for step in range(3):
            frames, t = synth.sample_batch(clips, 2, seed=7 * rank + step)
            losses.append(tr.step_host(frames, t).tolist())
        digests = [hashlib.sha256(tr.download(w).tobytes()).hexdigest() for w in (0, 1)]
        out.put((rank, digests, losses))
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
