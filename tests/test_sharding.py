"""Multi-GPU partitioning of the attention path, tested on CPU.

(batch, head) slices are independent, so N GPUs split them with no collective on the data
path (rocmkernels_b200.sharding). These tests check the plan covers every slice exactly once
and, with two gloo ranks on CPU, that per-rank oracle results on their shards reassemble into the
single-process result bit for bit.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from rocmkernels_b200.sharding import even_ranges, shard_plan


@pytest.mark.parametrize("batch,heads,world", [(8, 3, 1), (8, 3, 2), (8, 3, 8), (64, 12, 8), (2, 12, 8), (1, 5, 4), (3, 1, 8)])
def test_plan_covers_every_slice_once(batch, heads, world):
    seen = np.zeros((batch, heads), np.int32)
    for rank in range(world):
        for call in shard_plan(batch, heads, world, rank):
            assert 0 <= call.b0 < call.b1 <= batch and 0 <= call.h0 < call.h1 <= heads
            seen[call.b0:call.b1, call.h0:call.h1] += 1
    assert np.all(seen == 1)


def test_even_ranges_balance():
    ranges = even_ranges(10, 4)
    assert ranges == [(0, 3), (3, 6), (6, 8), (8, 10)]
    sizes = [b - a for a, b in even_ranges(64, 8)]
    assert sizes == [8] * 8


def _free_port() -> int:
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    from oracle import oracle

    batch, heads, seq, width = 3, 2, 24, 32
    q = oracle.normal(batch * heads * seq * width, 101).reshape(batch, heads, seq, width)
    k = oracle.normal(batch * heads * seq * width, 102).reshape(batch, heads, seq, width)
    v = oracle.normal(batch * heads * seq * width, 103).reshape(batch, heads, seq, width)
    u = oracle.normal(batch * heads * seq * width, 104).reshape(batch, heads, seq, width)
    mask = np.ones((batch, seq), np.uint8)
    mask[1, 5:] = 0
    out = np.zeros((batch, heads, seq, width), np.float32)
    for call in shard_plan(batch, heads, world, rank):
        part = oracle.attention(q[call.b0:call.b1, call.h0:call.h1], k[call.b0:call.b1, call.h0:call.h1],
                                v[call.b0:call.b1, call.h0:call.h1], mask[call.b0:call.b1], u[call.b0:call.b1, call.h0:call.h1], 3)
        out[call.b0:call.b1, call.h0:call.h1] = part["output"]
    total = torch.from_numpy(out)
    dist.all_reduce(total)  # test-only gather: each element is written by exactly one rank
    if rank == 0:
        whole = oracle.attention(q, k, v, mask, u, 3)["output"]
        queue.put(bool(np.array_equal(total.numpy().view(np.uint32), whole.view(np.uint32))))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_the_single_process_result():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(rank, world, port, queue)) for rank in range(world)]
    for proc in procs:
        proc.start()
    for proc in procs:
        proc.join(timeout=120)
    assert all(proc.exitcode == 0 for proc in procs)
    assert queue.get(timeout=5) is True
