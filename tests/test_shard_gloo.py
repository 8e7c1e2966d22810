"""The multi-GPU path's host logic on CPU: two gloo ranks, each with its own block of streams (no data-path
collective), give every stream the same words as one process running all of them; the job time is the max."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from oracle.oracle import Oracle
    from streaming_machine_b200 import convert, shard
    dist.init_process_group("gloo", rank=rank, world_size=world)
    r, w, _ = shard.rank_env()
    ids = shard.stream_ids(1, 2, 8, r, w, 50257)
    orc = Oracle(convert.load_gpt2(0))
    words = orc.generate(ids, 2, threads=1)
    # a fixed total split by stream (strong scaling, as C5 is): 5 streams over the ranks
    total = np.random.default_rng(4).integers(0, 50257, (5, 8))
    lo, hi = shard.partition(len(total), r, w)
    part = orc.generate(total[lo:hi], 2, threads=1)
    got = [None] * w
    dist.all_gather_object(got, (ids.tolist(), words.tolist(), lo, hi, part.tolist()))
    t = shard.max_over_ranks(1.0 + r, dist)
    if r == 0:
        q.put((got, t))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.slow
def test_two_ranks_match_one_process(M):
    from oracle.oracle import Oracle
    from streaming_machine_b200 import shard
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got, t = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert t == 2.0
    all_ids = shard.stream_ids(1, 4, 8, 0, 1, 50257)
    assert np.array_equal(np.concatenate([np.asarray(g[0]) for g in got]), all_ids)     # disjoint, complete
    want = Oracle(M).generate(all_ids, 2)
    assert np.array_equal(np.concatenate([np.asarray(g[1]) for g in got]), want)
    # rank 0 of any world size holds the single-GPU configuration's streams
    assert np.array_equal(shard.stream_ids(1, 2, 8, 0, 4, 50257), shard.stream_ids(1, 2, 8, 0, 1, 50257))
    # the partitioned total: blocks in rank order cover every stream once and give one process's words
    assert [(g[2], g[3]) for g in got] == [(0, 3), (3, 5)]
    total = np.random.default_rng(4).integers(0, 50257, (5, 8))
    assert np.array_equal(np.concatenate([np.asarray(g[4]) for g in got]), Oracle(M).generate(total, 2))


@pytest.mark.parametrize("n,world", [(512, 1), (512, 2), (512, 8), (5, 2), (7, 3), (3, 4)])
def test_partition_covers_every_stream_once(n, world):
    from streaming_machine_b200 import shard
    blocks = [shard.partition(n, r, world) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
    sizes = [hi - lo for lo, hi in blocks]
    assert max(sizes) - min(sizes) <= 1
