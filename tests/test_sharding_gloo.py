"""Batch sharding + final gather across 2 ranks (gloo, CPU).  The per-shard
compute is the CPU oracle; the test checks that shard bounds and the gather
reassemble exactly the unsharded result."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from tiktoktechjam2026_b200.sharding import gather_to_rank0, shard_bounds, sharded_forward


def test_shard_bounds_cover_batch():
    for batch in (1, 7, 16, 512):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(batch, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            for (s0, e0), (s1, e1) in zip(spans, spans[1:]):
                assert e0 == s1
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = oracle.Config(5, 12, 32, 2, 64, 2, True)
        sd = oracle.seeded_state_dict(cfg, 11)
        x, mask = oracle.generate_case(cfg, 3, padding_ratio=0.4)
        local = sharded_forward(lambda xs, ms: oracle.forward(sd, cfg, xs, ms), x, mask, rank, world)
        full = gather_to_rank0(local, x.shape[0], rank, world)
        if rank == 0:
            torch.save(full, result_path)
    finally:
        dist.destroy_process_group()


def test_two_rank_gather_equals_unsharded(tmp_path):
    path = str(tmp_path / "out.pt")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
    full = torch.load(path)
    cfg = oracle.Config(5, 12, 32, 2, 64, 2, True)
    sd = oracle.seeded_state_dict(cfg, 11)
    x, mask = oracle.generate_case(cfg, 3, padding_ratio=0.4)
    ref = oracle.forward(sd, cfg, x, mask)
    assert torch.equal(full, ref)
