"""The multi-GPU path of bench.py on CPU: two gloo ranks run the same
sharding and max/sum aggregation that the NCCL ranks run on B200s
(sequences sharded by global id, no collective on the data path)."""
import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import datetime
    import torch.distributed as dist
    import bench
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    first, n = bench.shard(rank, world, 8)
    prompts = bench.spec_prompts(first, n)
    # per-rank "timings" and "counters"
    t, c = bench.reduce_over_ranks(dist, [10.0 + rank, 1.0 * rank], [100 + rank, n], "cpu")
    q.put((rank, first, n, [p.tolist()[:4] for p in prompts], t, c))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharding_and_aggregation():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    sys.path.insert(0, ROOT)
    import bench
    ids = set()
    for rank, first, n, heads, t, c in res:
        assert n == 8 and first == 8 * rank
        ids.update(range(first, first + n))
        # a rank's prompts are the single-process prompts of the same global ids
        assert heads == [p.tolist()[:4] for p in bench.spec_prompts(first, n)]
        assert t == [11.0, 1.0]                 # max over ranks
        assert c == [201.0, 16.0]               # sum over ranks
    assert ids == set(range(16))                # disjoint shards cover all sequences
