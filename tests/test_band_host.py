"""Row-band sharding, host side (no GPU): the split of the padded plane's window
rows among ranks and the halo schedule, run on CPU ranks over gloo.

The library's own schedule (s2s_band_halo_ops, the function its exchange uses)
is executed with torch.distributed send/recv between world-size-2/3/4 gloo ranks,
on float planes that hold each global row's index. Messages between a pair of
ranks are matched in issue order, as NCCL matches point-to-point operations of a
group. Afterwards every halo row must hold the global row the shifted windows (4
rows, cyclic wrap) or a 3x3 convolution (1 row, nothing beyond the true edges)
read there.
"""
import os
import socket

import numpy as np
import pytest

from s2s_testlib import pkg

HALO = 8


def capi():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.capi")


@pytest.mark.parametrize("window_rows,world", [(31, 8), (65, 8), (31, 2), (3, 3), (7, 4), (5, 1)])
def test_partition_covers_the_plane_in_order(window_rows, world):
    C = capi()
    bands = [C.band_partition(window_rows, world, r) for r in range(world)]
    assert bands[0][0] == 0 and bands[-1][1] == window_rows
    for (a0, a1), (b0, b1) in zip(bands, bands[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in bands]
    assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)   # the larger bands come first


def test_partition_rejects_more_bands_than_window_rows():
    C = capi()
    with pytest.raises(C.S2SError):
        C.band_partition(3, 4, 0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, window_rows, wp, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        C = capi()
        hp = 8 * window_rows
        w0, w1 = C.band_partition(window_rows, world, rank)
        own = 8 * (w1 - w0)
        errors = []
        for rows, cyclic in ((4, True), (1, False), (4, False)):
            # local plane: row i of the band holds global row R0 - 8 + i; halos start at -1
            local = torch.full((own + 2 * HALO, wp), -1.0)
            g = torch.arange(8 * w0, 8 * w1, dtype=torch.float32)
            local[HALO:HALO + own] = g[:, None].expand(own, wp)
            ops = C.band_halo_ops(rank, world, own, rows, cyclic)
            seq = {}
            reqs = []
            for kind, peer, r0, n in ops:
                tag = seq.get((kind, peer), 0)
                seq[(kind, peer)] = tag + 1
                buf = local[r0:r0 + n]
                if kind == 0:
                    reqs.append(dist.isend(buf.contiguous(), peer, tag=tag))
                else:
                    recv = torch.empty_like(buf)
                    reqs.append((dist.irecv(recv, peer, tag=tag), r0, n, recv))
            for r in reqs:
                if isinstance(r, tuple):
                    r[0].wait()
                    local[r[1]:r[1] + r[2]] = r[3]
                else:
                    r.wait()
            dist.barrier()
            for i in range(HALO - rows, HALO):               # top halo
                gr = 8 * w0 - HALO + i
                want = gr % hp if cyclic else (gr if gr >= 0 else -1)
                if int(local[i, 0]) != want:
                    errors.append((rows, cyclic, "top", i, float(local[i, 0]), want))
            for i in range(HALO + own, HALO + own + rows):   # bottom halo
                gr = 8 * w0 - HALO + i
                want = gr % hp if cyclic else (gr if gr < hp else -1)
                if int(local[i, 0]) != want:
                    errors.append((rows, cyclic, "bottom", i, float(local[i, 0]), want))
            assert bool((local[:, 0:1] == local).all()), "a row arrived torn"
        q.put((rank, errors))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, [repr(e)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,window_rows", [(2, 5), (3, 7), (4, 31)])
def test_halo_schedule_delivers_the_neighbours_rows_over_gloo(world, window_rows):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, window_rows, 16, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, errs = q.get(timeout=120)
        results[rank] = errs
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(not e for e in results.values()), results


def test_halo_ops_pair_up_between_two_ranks():
    """With two ranks prev == next: my last rows must land in the peer's top halo."""
    C = capi()
    a = C.band_halo_ops(0, 2, 24, 4, True)
    b = C.band_halo_ops(1, 2, 16, 4, True)
    sends_a = [op for op in a if op[0] == 0]
    recvs_b = [op for op in b if op[0] == 1]
    assert sends_a[0][2] == HALO + 24 - 4 and recvs_b[0][2] == HALO - 4   # last -> top
    assert sends_a[1][2] == HALO and recvs_b[1][2] == HALO + 16           # first -> bottom
    # no wrap for convolutions: the first rank receives nothing from above
    assert all(op[2] >= HALO for op in C.band_halo_ops(0, 2, 24, 1, False))
