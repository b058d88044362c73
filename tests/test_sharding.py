"""Multi-GPU partitioning of the attention path, tested on CPU.

(batch, head) slices are independent, so N GPUs split them with no collective on the data
path (rocmkernels_b200.sharding). These tests check the plan covers every slice exactly once
and, with two gloo ranks on CPU, that each rank's calls -- made by the same run_forward /
run_backward code a GPU rank runs, with the entry points replaced by the oracle on the
sub-problem each call's pointer offsets select -- reassemble into the single-process result
bit for bit (batch ranges, and head ranges inside one sequence).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
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


class _CpuEntries:
    """Stand-ins for the library's forward/backward entry points on the CPU: each "address" is a
    byte offset into one of the full problem's flat arrays (the base addresses are 0), and the
    call runs the oracle on the sub-problem found there. The offsets come from the same
    run_forward / run_backward / shard_offsets code a GPU rank runs."""

    def __init__(self, arrays):
        self.a = arrays  # role -> flat float32 / uint8 array

    def _view(self, role, offset_bytes, shape, strides_elements):
        flat = self.a[role]
        start = offset_bytes // flat.itemsize
        view = np.lib.stride_tricks.as_strided(flat[start:], shape=shape,
                                               strides=[s * flat.itemsize for s in strides_elements])
        return view

    def forward(self, q, k, v, mask, out, lse, batch, heads, queries, keys, radius, qs, ks, vs, os_, stream=None):
        width = 32
        sub = lambda role, off, n, s: np.ascontiguousarray(self._view(role, off, (batch, heads, n, width),
                                                                      (s.batch, s.head, s.token, 1)))
        m = self._view("mask", mask, (batch, keys), (keys, 1))
        result = oracle.attention(sub("q", q, queries, qs), sub("k", k, keys, ks), sub("v", v, keys, vs), m, None, radius,
                                  forward_only=True)
        self._view("out", out, (batch, heads, queries, width), (os_.batch, os_.head, os_.token, 1))[...] = result["output"]
        self._view("lse", lse, (batch, heads, queries, 2), (heads * queries * 2, queries * 2, 2, 1))[...] = result["lse"]
        return 0

    def backward(self, q, k, v, mask, out, lse, upstream, gq, gk, gv, delta, batch, heads, queries, keys, radius, qs, ks, vs,
                 os_, us, stream=None):
        width = 32
        sub = lambda role, off, n, s: np.ascontiguousarray(self._view(role, off, (batch, heads, n, width),
                                                                      (s.batch, s.head, s.token, 1)))
        m = self._view("mask", mask, (batch, keys), (keys, 1))
        result = oracle.attention(sub("q", q, queries, qs), sub("k", k, keys, ks), sub("v", v, keys, vs), m,
                                  sub("upstream", upstream, queries, us), radius)
        for role, off, n in (("grad_q", gq, queries), ("grad_k", gk, keys), ("grad_v", gv, keys)):
            self._view(role, off, (batch, heads, n, width), (heads * n * width, n * width, width, 1))[...] = result[role]
        return 0


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch

    from rocmkernels_b200.attention import Strides
    from rocmkernels_b200.sharding import run_backward, run_forward

    for batch, heads in ((3, 2), (1, 5)):  # batch ranges, then head ranges inside one sequence
        seq, width, radius = 24, 32, 3
        shape = (batch, heads, seq, width)
        q = oracle.normal(batch * heads * seq * width, 101).reshape(shape)
        k = oracle.normal(batch * heads * seq * width, 102).reshape(shape)
        v = oracle.normal(batch * heads * seq * width, 103).reshape(shape)
        u = oracle.normal(batch * heads * seq * width, 104).reshape(shape)
        mask = np.ones((batch, seq), np.uint8)
        mask[-1, 5:] = 0
        arrays = {"q": q.ravel(), "k": k.ravel(), "v": v.ravel(), "upstream": u.ravel(), "mask": mask.ravel(),
                  "out": np.zeros(q.size, np.float32), "lse": np.zeros(batch * heads * seq * 2, np.float32),
                  "grad_q": np.zeros(q.size, np.float32), "grad_k": np.zeros(q.size, np.float32),
                  "grad_v": np.zeros(q.size, np.float32), "delta": np.zeros(batch * heads * seq, np.float32)}
        entries = _CpuEntries(arrays)
        st = Strides(heads * seq * width, seq * width, width)
        strides = {role: st for role in ("q", "k", "v", "out", "upstream")}
        plan = shard_plan(batch, heads, world, rank)
        bases = {role: 0 for role in arrays}
        geometry = dict(heads=heads, queries=seq, keys=seq, width=width, radius=radius, strides=strides)
        assert run_forward(entries.forward, {r: bases[r] for r in ("q", "k", "v", "mask", "out", "lse")}, plan, **geometry) == 0
        assert run_backward(entries.backward, bases, plan, **geometry) == 0
        ok = True
        whole = oracle.attention(q, k, v, mask, u, radius)
        for role, expected in (("out", whole["output"]), ("lse", whole["lse"]), ("grad_q", whole["grad_q"]),
                               ("grad_k", whole["grad_k"]), ("grad_v", whole["grad_v"])):
            total = torch.from_numpy(arrays[role].copy())
            dist.all_reduce(total)  # test-only gather: each element is written by exactly one rank
            ok = ok and bool(np.array_equal(total.numpy().view(np.uint32), expected.ravel().view(np.uint32)))
        if rank == 0:
            queue.put(ok)
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
    assert queue.get(timeout=5) is True


@pytest.mark.parametrize("batch,heads,world,rank", [(64, 12, 8, 3), (8, 3, 2, 1), (3, 1, 8, 2)])
def test_forward_workspace_covers_every_call(batch, heads, world, rank):
    from rocmkernels_b200 import attention as api
    from rocmkernels_b200.sharding import forward_workspace_bytes

    plan = shard_plan(batch, heads, world, rank)
    size = api.attention_fp32_forward_flash_workspace_size
    need = forward_workspace_bytes(size, plan, 4096)
    assert need == max((size(c.batch, c.heads, 4096) for c in plan), default=0)
    assert all(size(c.batch, c.heads, 4096) <= need for c in plan)


@pytest.mark.parametrize("workspace", [None, 0x7000])
def test_run_forward_hands_the_workspace_to_every_call(workspace):
    from rocmkernels_b200.sharding import run_forward

    calls = []

    def entry(*args, **kwargs):
        calls.append(kwargs)
        return 0

    plan = shard_plan(8, 3, 2, 0)
    tensors = {name: 0x100000 for name in ("q", "k", "v", "mask", "out", "lse")}
    strides = {name: (3 * 1024 * 32, 1024 * 32, 32) for name in ("q", "k", "v", "out")}
    status = run_forward(entry, tensors, plan, heads=3, queries=1024, keys=1024, width=32, radius=-1, strides=strides,
                         workspace=workspace)
    assert status == 0 and len(calls) == len(plan)
    assert all(c == ({} if workspace is None else {"workspace": workspace}) for c in calls)
