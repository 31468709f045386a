"""Head sharding across ranks (gloo, world size 2, CPU): the partition is
exact, every rank regenerates identical per-head inputs from the per-head
seeds, and the slowest-rank reduction works."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pasa_b200 import dist as pdist
from pasa_b200 import synth


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import dataclasses

        w = dataclasses.replace(synth.WORKLOADS["wan14b-720p"], heads=5, T=2 * 3600, frames=2)
        heads = pdist.shard_heads(w.heads, rank, world)
        sums = {}
        for h in heads:
            qh, kh, vh = synth.head_qkv(w, h, "cpu")
            sums[h] = float(qh.float().sum() + 2 * kh.float().sum() + 3 * vh.float().sum())
        t = pdist.max_over_ranks(float(rank + 1) * 1.5)
        pdist.barrier()
        q.put((rank, list(heads), sums, t))
    finally:
        dist.destroy_process_group()


def test_two_rank_head_sharding():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    heads = sorted(h for _, hs, _, _ in results for h in hs)
    assert heads == list(range(5))                      # exact partition
    assert all(t == 3.0 for *_, t in results)           # max over ranks
    import dataclasses

    w = dataclasses.replace(synth.WORKLOADS["wan14b-720p"], heads=5, T=2 * 3600, frames=2)
    for _, hs, sums, _ in results:                      # same per-head data as a single process
        for h in hs:
            qh, kh, vh = synth.head_qkv(w, h, "cpu")
            assert sums[h] == float(qh.float().sum() + 2 * kh.float().sum() + 3 * vh.float().sum())


def test_shard_sizes_differ_by_at_most_one():
    for total in (1, 5, 12, 24, 40):
        for world in (1, 2, 3, 4, 8):
            sizes = [len(pdist.shard_heads(total, r, world)) for r in range(world)]
            assert sum(sizes) == total and max(sizes) - min(sizes) <= 1


def test_block_sharding_partition():
    """(head, query-block) shards for head counts the world size does not
    divide: exact, disjoint, balanced within three blocks, and no pair of
    query blocks split inside a head."""
    for heads, NT in ((12, 512), (12, 511), (5, 37), (3, 1182)):
        for world in (1, 2, 3, 5, 8):
            ranges = [synth.shard_blocks(heads, NT, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == heads * NT
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [e - b for b, e in ranges]
            assert min(sizes) > 0 and max(sizes) - min(sizes) <= 3
            for b, e in ranges:
                for x in (b, e):
                    assert (x % NT) % 2 == 0 or x == heads * NT
