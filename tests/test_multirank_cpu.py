"""Cross-rank host logic on world_size-2 gloo process groups (CPU only).

The decode path shards value heads over ranks with no data-path collective;
what crosses ranks is the slot-count agreement (a MIN over the gloo CPU group,
sglang/runtime.py:310-317), the benchmark's max-over-ranks timing, and in the
layer stack (bench.py --workload gdn-stack) the all-gather of each layer's
readouts back into the global head order.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stepquant_b200.sglang.runtime import agree_min, shard_plan
        from stepquant_b200 import QuantizationPlan
        # Mixed-precision shards give each rank a different page size and slot count.
        count = agree_min([1000, 640][rank], dist.group.WORLD)
        gen = torch.Generator().manual_seed(0)
        bits = torch.tensor([4, 6, 8, 6])[:, None].expand(4, 8).clone()
        entry = dict(architecture="gdn", bits=bits, impact=torch.rand(4, 8, generator=gen) + 0.5, value_group_size=8)
        shard = shard_plan(entry, 2, rank, world)
        gathered = [torch.zeros(2, 8, dtype=torch.long) for _ in range(world)]
        dist.all_gather(gathered, shard.bits.contiguous())
        elapsed = torch.tensor([3.0, 7.5][rank], dtype=torch.float64)
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
        results[rank] = (count, torch.equal(torch.cat(gathered), bits), float(elapsed))
    finally:
        dist.destroy_process_group()


def test_two_rank_slot_agreement_sharding_and_timing():
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    assert dict(results) == {0: (640, True, 7.5), 1: (640, True, 7.5)}


def test_single_rank_agreement_is_identity():
    from stepquant_b200.sglang.runtime import agree_min
    assert agree_min(17, None) == 17


def _gather_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        tokens, heads, dim = 3, 4, 5
        full = torch.arange(tokens * heads * world * dim, dtype=torch.float32).reshape(tokens, heads * world, dim)
        local = full[:, rank * heads:(rank + 1) * heads].reshape(tokens, heads * dim)  # this rank's value heads
        gathered = bench.gather_heads(local, world)
        results[rank] = torch.equal(gathered, full.reshape(tokens, heads * world * dim))
    finally:
        dist.destroy_process_group()


def test_two_rank_readout_gather_keeps_global_head_order():
    world, port = 2, _free_port()
    results = mp.Manager().dict()
    mp.spawn(_gather_worker, args=(world, port, results), nprocs=world, join=True)
    assert results[0] and results[1]
