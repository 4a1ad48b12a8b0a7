"""Data-parallel host logic on CPU: two gloo ranks exchange the communicator
id, split the global batch and take the max of their timings, the same calls
bench.py makes over NCCL on the GPUs (no GPU, no library compute)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from yumelayers_b200.trainer import shard_batch


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist

    from yumelayers_b200.trainer import max_over_ranks, share_unique_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def bcast(obj):
            dist.broadcast_object_list(obj, src=0)
        uid = share_unique_id(rank, lambda: bytes(range(128)), bcast)
        lo, hi = shard_batch(16, world, rank)
        slowest = max_over_ranks(10.0 + 7.5 * rank)
        alone = max_over_ranks(-1.0 * rank)
        out.put((rank, uid, lo, hi, slowest, alone))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_id_split_batch_and_take_max():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] == bytes(range(128)) for r in res)
    shards = [range(r[2], r[3]) for r in res]
    assert sorted(i for s in shards for i in s) == list(range(16))
    assert all(r[4] == 17.5 for r in res)
    assert all(r[5] == 0.0 for r in res)


def test_shard_batch_rejects_uneven_split():
    assert shard_batch(64, 8, 7) == (56, 64)
    with pytest.raises(ValueError):
        shard_batch(10, 4, 0)


def test_max_over_ranks_without_a_group_is_identity():
    from yumelayers_b200.trainer import max_over_ranks
    assert max_over_ranks(3.25) == 3.25
