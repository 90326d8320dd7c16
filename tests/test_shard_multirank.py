"""Host-side multi-GPU logic on CPU: partitioning and max-over-ranks timing,
run as two gloo ranks (the data path exchanges nothing, so the CPU ranks
cover everything a multi-GPU run does outside the kernels)."""

import os
import random

import torch.distributed as dist
import torch.multiprocessing as mp

from evocompile_b200 import shard


def test_row_range_covers_exactly():
    for n in (0, 1, 7, 8192, 8193):
        for world in (1, 2, 3, 8):
            spans = [shard.row_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1


def test_balance_sequences_is_a_partition_and_balanced():
    rng = random.Random(0)
    lengths = [rng.randint(512, 8192) for _ in range(16)]
    for world in (1, 2, 4, 8):
        parts = shard.balance_sequences(lengths, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(16))
        loads = [sum(lengths[i] for i in p) for p in parts]
        # LPT bound: max load <= average + longest item
        assert max(loads) <= sum(lengths) / world + max(lengths)


def test_cu_seqlens():
    assert shard.cu_seqlens([3, 0, 5]) == [0, 3, 3, 8]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lengths = [100, 900, 40, 512, 7, 333]
        mine = shard.balance_sequences(lengths, world)[rank]
        got = [None] * world
        dist.all_gather_object(got, mine)
        t = shard.max_over_ranks(10.0 * (rank + 1))
        rows = shard.row_range(8192 * world, rank, world)
        q.put((rank, got, t, rows))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + random.Random().randint(0, 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    (_, g0, t0, r0), (_, g1, t1, r1) = res
    assert g0 == g1 and sorted(g0[0] + g0[1]) == list(range(6))
    assert t0 == t1 == 20.0
    assert r0 == (0, 8192) and r1 == (8192, 16384)
