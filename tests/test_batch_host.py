"""Batch data-parallel split, host side (no GPU): the compressed-x4 batch of
independent images is divided among ranks with no exchange between them
(bench.py --mode batch). Each rank must take a contiguous, equal shard in rank
order, so that the ranks' outputs concatenate to the batch's; run here on CPU
ranks over gloo with the same input recipe the bench uses.
"""
import os
import socket

import numpy as np
import pytest

from s2s_testlib import pkg


def workloads():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.workloads")


@pytest.mark.parametrize("batch,world", [(256, 1), (256, 2), (256, 4), (256, 8), (6, 3)])
def test_shards_cover_the_batch_in_rank_order(batch, world):
    W = workloads()
    shards = [W.batch_shard(batch, world, r) for r in range(world)]
    assert shards[0][0] == 0 and shards[-1][1] == batch
    for (lo, hi), (lo2, _) in zip(shards, shards[1:]):
        assert hi == lo2
    assert len({hi - lo for lo, hi in shards}) == 1


@pytest.mark.parametrize("batch,world,rank", [(256, 3, 0), (5, 2, 1), (8, 2, 2), (8, 0, 0)])
def test_uneven_batches_and_bad_ranks_are_refused(batch, world, rank):
    with pytest.raises(ValueError):
        workloads().batch_shard(batch, world, rank)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, batch, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = workloads()
        P = pkg()
        wt = P.weights.Weights.seeded("compressed_sr", 0)
        x = W.make_input("compressed-x4", batch)
        lo, hi = W.batch_shard(batch, world, rank)
        mine = torch.from_numpy(W.adjust(x[lo:hi], wt))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        # the bench's job time is the slowest rank's: a MAX all-reduce of each rank's time
        t = torch.tensor([float(rank + 1)])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        whole = torch.cat(parts).numpy()
        ok = bool(np.array_equal(whole, W.adjust(x, wt))) and float(t.item()) == float(world)
        q.put((rank, ok, hi - lo, None))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, False, 0, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_rank_shards_reassemble_the_batch_over_gloo(world):
    import torch.multiprocessing as mp
    batch = 8
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, batch, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, ok, n, err = q.get(timeout=120)
        results[rank] = (ok, n, err)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok and n == batch // world for ok, n, _ in results.values()), results
