"""Row-band sharded forward across processes, one per GPU (skipped below 2 GPUs).

Each rank is a spawned process on its own GPU; the communicator id comes from
s2s_band_unique_id in the parent. Both halo transports run: peer stores into the
neighbours' IPC-mapped planes (the default) and NCCL send/recv (S2S_HALO=nccl).
The concatenated bands must equal the whole-image forward on one GPU exactly (the
arithmetic per row is identical).
"""
import numpy as np
import pytest

from s2s_testlib import adjust, pkg

pytestmark = pytest.mark.gpu


def _ngpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _rank(rank, world, uid, task, h, w, transport, q):
    import importlib
    import os
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["S2S_HALO"] = transport
    try:
        import torch
        torch.cuda.set_device(rank)
        P = pkg()
        C = importlib.import_module("swin2sr_b200.capi")
        wt = P.weights.Weights.seeded(task, 0, True)
        x = adjust(wt, np.random.default_rng(21).random((3, h, w), dtype=np.float32))
        H = C.Handle(wt, device=rank)
        try:
            H.band_init(rank, world, uid)
            out = H.forward_band(x)
            out2 = H.forward_band(x)          # a second forward reuses plan and communicator
            q.put((rank, H.band_rows(h), out, bool(np.array_equal(out, out2)), None))
        finally:
            H.close()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, None, None, False, repr(e)))


@pytest.mark.parametrize("transport", ["ipc", "nccl"])
@pytest.mark.parametrize("task,h,w", [("classical_sr", 70, 52), ("real_sr", 45, 33)])
def test_bands_equal_the_whole_image_forward(task, h, w, transport):
    world = min(_ngpus(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import importlib

    import torch.multiprocessing as mp
    P = pkg()
    C = importlib.import_module("swin2sr_b200.capi")
    uid = C.band_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, task, h, w, transport, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, rows, out, same, err = q.get(timeout=600)
        res[r] = (rows, out, same, err)
    for p in procs:
        p.join(timeout=120)
    assert all(v[3] is None for v in res.values()), {r: v[3] for r, v in res.items()}
    assert all(v[2] for v in res.values()), "a second band forward differed from the first"
    wt = P.weights.Weights.seeded(task, 0, True)
    x = adjust(wt, np.random.default_rng(21).random((3, h, w), dtype=np.float32))
    H = C.Handle(wt, device=0)
    try:
        whole = H.forward_batch(x[None])[0][0]
    finally:
        H.close()
    got = np.concatenate([res[r][1] for r in range(world)], axis=1)
    err = float(np.abs(got - whole).max())
    print(f"{task} {h}x{w} {transport} world {world}: bands vs whole max-abs {err:.3e}")
    assert err == 0.0
