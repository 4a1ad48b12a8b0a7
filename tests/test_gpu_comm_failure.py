"""Failure handling of the data-parallel communicator, driven on the host.

The reference has no multi-GPU path; these tests hold the backend to the
same rule as its hang guard (GpuTraining.swift:72-112): a missing peer ends
in a status, never in a process blocked for good.  No GPU kernel is made to
fail: the faults are a rank that never joins and a rank that leaves between
steps, with none of its kernels or collectives in flight.  NVLink SHARP is
off in every child (NCCL_NVLS_ENABLE=0), so no rank's memory is bound to a
multicast object when another rank goes away.
"""
import os
import socket

import pytest
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
YL_ERR_TIMEOUT = 3


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _lonely_rank(out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from yumelayers_b200._lib import YumeError
    from yumelayers_b200.session import Context
    from yumelayers_b200.trainer import Comm
    ctx = Context(0)
    uid = Comm.unique_id()
    try:
        Comm(ctx, uid, 0, 2, timeout_s=3.0)  # rank 1 never calls init
        out.put(("joined", None))
    except YumeError as e:
        out.put(("error", e.status))


def test_comm_init_times_out_when_a_rank_never_joins():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        kind, status = q.get(timeout=120)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert (kind, status) == ("error", YL_ERR_TIMEOUT)
    assert p.exitcode == 0


def _leaving_rank(rank, world, port, out, trace_dir):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import faulthandler
    from datetime import timedelta
    # a child that stalls or dies leaves its last stage and its stacks behind
    # for the failure message
    trace = open(os.path.join(trace_dir, f"rank{rank}.txt"), "w", buffering=1)
    faulthandler.enable(file=trace, all_threads=True)
    faulthandler.dump_traceback_later(150, exit=False, file=trace)

    def stage(what):
        trace.write(f"rank {rank}: {what}\n")

    import numpy as np
    import torch
    import torch.distributed as dist

    from yumelayers_b200 import synth
    from yumelayers_b200.session import Context
    from yumelayers_b200.trainer import Comm, Trainer, default_config
    torch.cuda.set_device(rank)
    stage("store")
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    ctx = Context(rank)
    if rank == 0:
        store.set("uid", Comm.unique_id())
    stage("communicator")
    comm = Comm(ctx, store.get("uid"), rank, world, timeout_s=60.0)
    cfg = default_config(batch=1, height=32, width=48, seed=2)
    tr = Trainer(cfg, ctx=ctx, comm=comm)
    clips = [synth.make_clip(60 + rank, h=32, w=48, width_padded=48)]
    frames, t = synth.sample_batch(clips, 1, seed=rank)
    stage("step")
    loss = tr.step_host(frames, t)  # one data-parallel step; returns with nothing in flight
    if rank == 1:
        # leaves between steps: stops stepping, says so, and ends its side once
        # the other rank has aborted
        store.set("left", "1")
        stage("left; waiting for the other rank's abort")
        store.wait(["aborted"], timedelta(seconds=60))
        stage("abort")
        comm.abort()
        tr.close()  # the trainer borrows the communicator: release it first
        comm.close()
        out.put((rank, "left", float(loss[0])))
        return
    # rank 0 learns of it from the store before its next launch, aborts the
    # communicator and keeps working on its own
    store.wait(["left"], timedelta(seconds=60))
    stage("abort")
    comm.abort()
    stage("aborted")
    store.set("aborted", "1")
    tr.close()  # the trainer borrows the communicator: release it first
    comm.close()
    solo = Trainer(cfg, ctx=ctx)
    solo_loss = solo.step_host(frames, t)
    solo.close()
    out.put((rank, "aborted", bool(np.isfinite(solo_loss).all())))


def test_rank_leaving_between_steps_is_seen_and_the_comm_aborted():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import tempfile
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    trace_dir = tempfile.mkdtemp(prefix="yl_comm_")
    procs = [ctx.Process(target=_leaving_rank, args=(r, world, port, q, trace_dir))
             for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in range(world):
            res.append(q.get(timeout=240))
    except Exception:
        stacks = "".join(open(os.path.join(trace_dir, f)).read()
                         for f in sorted(os.listdir(trace_dir)))
        for p in procs:
            p.join(timeout=30)
        codes = [p.exitcode for p in procs]
        pytest.fail(f"ranks reported {res}; exit codes {codes}; stages and stacks:\n{stacks}")
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    res.sort()
    assert res[0][:2] == (0, "aborted") and res[0][2] is True
    assert res[1][:2] == (1, "left")
    assert all(p.exitcode == 0 for p in procs)
