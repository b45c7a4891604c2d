"""The N > 1 path on CPU: two gloo ranks shard requests, each runs its share of the GDN recurrence (oracle, CPU),
and the gathered results and the max-over-ranks timing equal the single-process run."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import __graft_entry__


def test_shard_is_a_balanced_partition():
    replicas = __graft_entry__.load_package().replicas
    for n in (0, 1, 7, 64, 255):
        for world in (1, 2, 3, 8):
            parts = [replicas.shard(n, world, r) for r in range(world)]
            assert [i for p in parts for i in p] == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import sys

        sys.path.insert(0, str(__graft_entry__.ROOT))
        from oracle import gdn as ogdn

        replicas = __graft_entry__.load_package().replicas
        n, H, d = 10, 2, 16
        gen = torch.Generator().manual_seed(0)
        q = torch.nn.functional.normalize(torch.randn(n, H, d, generator=gen), dim=-1)
        k = torch.nn.functional.normalize(torch.randn(n, H, d, generator=gen), dim=-1)
        v = torch.randn(n, H, d, generator=gen)
        g = -torch.rand(n, H, generator=gen)
        beta = torch.rand(n, H, generator=gen)
        state = torch.randn(n, H, d, d, generator=gen)
        mine = replicas.shard(n, world, rank)
        _, out = ogdn.recurrent_step(state[mine.start:mine.stop], q[mine.start:mine.stop], k[mine.start:mine.stop],
                                     v[mine.start:mine.stop], g[mine.start:mine.stop], beta[mine.start:mine.stop],
                                     d ** -0.5)
        gathered = replicas.gather_rows(out, n)
        slowest = replicas.max_over_ranks(1.0 + rank)
        if rank == 0:
            _, full = ogdn.recurrent_step(state, q, k, v, g, beta, d ** -0.5)
            result_queue.put((torch.equal(gathered, full), slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reproduce_the_single_process_result():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    equal, slowest = queue.get(timeout=10)
    assert equal and slowest == 2.0
