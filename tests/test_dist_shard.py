"""The multi-GPU plumbing of bench.py on CPU: two gloo ranks take disjoint
document shards, and the reductions give the max time and the total count.
Chunks are independent, so the per-rank chunk bytes (CPU oracle) concatenated
in rank order equal the bytes of the whole set compressed by one process."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bench
    from oracle import oracle as O

    seeds = list(bench.shard_seeds(rank, 2))
    mf = bench.czm.ModelFile.load(os.path.join(ROOT, "models", "v001_eng.czm"))
    tokens, starts, nbytes, _ = bench.workload(mf, seeds, 64)
    om = O.load_model(os.path.join(ROOT, "models", "v001_eng.czm"))
    chunks = O.compress_chunks(om, tokens[:400], starts[starts <= 400], nthreads=2)
    tmax, nsum = bench.reduce_over_ranks([1.0 + rank], [float(len(tokens))], "cpu")
    q.put((rank, seeds, tmax, nsum, len(tokens), chunks))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_sharding():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (_, s0, t0, n0, k0, c0), (_, s1, t1, n1, k1, c1) = res
    assert set(s0).isdisjoint(s1) and s0 == [1, 2] and s1 == [3, 4]
    assert t0 == t1 == [2.0]
    assert n0 == n1 == [float(k0 + k1)]

    sys.path.insert(0, ROOT)
    import bench
    from oracle import oracle as O

    mf = bench.czm.ModelFile.load(os.path.join(ROOT, "models", "v001_eng.czm"))
    om = O.load_model(os.path.join(ROOT, "models", "v001_eng.czm"))
    for seeds, chunks in (([1, 2], c0), ([3, 4], c1)):
        tokens, starts, _, _ = bench.workload(mf, seeds, 64)
        assert chunks == O.compress_chunks(om, tokens[:400], starts[starts <= 400], nthreads=4)
