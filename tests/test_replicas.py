"""Row sharding and the cross-rank reductions of the multi-GPU replicas, on CPU with gloo (world size 2)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from nanovllm_b200.replicas import shard_rows


@pytest.mark.parametrize("total,world", [(512, 1), (512, 2), (512, 8), (513, 4), (3, 8)])
def test_shards_cover_every_row_once(total, world):
    rows = [r for rank in range(world) for r in shard_rows(total, world, rank)]
    assert rows == list(range(total))
    sizes = [len(shard_rows(total, world, rank)) for rank in range(world)]
    assert max(sizes) - min(sizes) <= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist
    from nanovllm_b200 import replicas
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        replicas.barrier()
        rows = replicas.shard_rows(512, world, rank)
        out[rank] = (replicas.reduce_scalar(10.0 * (rank + 1), "max"), replicas.reduce_scalar(len(rows), "sum"))
    finally:
        dist.destroy_process_group()


def test_reductions_over_two_gloo_ranks():
    world, port = 2, _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    mp.start_processes(_worker, args=(world, port, out), nprocs=world, join=True, start_method="spawn")
    assert out[0] == out[1] == (20.0, 512.0)


def test_reductions_without_a_process_group():
    from nanovllm_b200 import replicas
    assert replicas.reduce_scalar(3.5, "max") == 3.5
