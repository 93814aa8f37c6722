"""Row-band sharded forward against the whole-image forward, on one GPU.

The bands of an in-process group (s2s_band_init_local) run concurrently, one host
thread per band, and swap halos by device-to-device copies; the same forward code
runs under NCCL between processes (test_gpu_band_nccl.py). Every row of the output
depends only on the rows the halos carry, and the per-row arithmetic is the same
kernels on the same operands, so the bands' output must equal the whole-image
forward's exactly.
"""
import threading

import numpy as np
import pytest

from s2s_testlib import TOL, adjust, oracle, pkg

pytestmark = pytest.mark.gpu


def capi():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.capi")


def run_bands(wt, x, world):
    C = capi()
    hs = [C.Handle(wt) for _ in range(world)]
    try:
        C.band_init_local(hs)
        outs = [None] * world
        errs = []

        def go(r):
            try:
                outs[r] = hs[r].forward_band(x)
            except Exception as e:  # noqa: BLE001
                errs.append((r, e))

        ts = [threading.Thread(target=go, args=(r,)) for r in range(world)]
        for t in ts:
            t.start()
        for t in ts:
            t.join(timeout=300)
        assert not errs, errs
        rows = [hs[r].band_rows(x.shape[1]) for r in range(world)]
        return outs, rows
    finally:
        for h in hs:
            h.close()


@pytest.mark.parametrize("task,h,w,world,attn", [
    ("classical_sr", 61, 45, 2, None),      # x4 pixelshuffle, 8 window rows
    ("classical_sr_x2", 61, 45, 3, None),   # x2 pixelshuffle
    ("lightweight_sr", 40, 30, 4, None),    # pixelshuffledirect
    ("real_sr", 37, 21, 2, None),           # nearest+conv x4
    ("classical_sr", 16, 30, 3, None),      # one window row per band; the last band is all padding
    ("classical_sr", 61, 45, 3, "fused"),   # the fused QKV + attention kernel on bands
    ("real_sr", 37, 21, 2, "fused"),
])
def test_bands_equal_the_whole_image_forward(task, h, w, world, attn, monkeypatch):
    if attn:
        monkeypatch.setenv("S2S_ATTN", attn)
    C = capi()
    P = pkg()
    wt = P.weights.Weights.seeded(task, 0, True)
    x = adjust(wt, np.random.default_rng(11).random((3, h, w), dtype=np.float32))
    H = C.Handle(wt)
    try:
        whole = H.forward_batch(x[None])[0][0]
    finally:
        H.close()
    outs, rows = run_bands(wt, x, world)
    s = wt.scale
    assert rows[0][0] == 0 and rows[-1][1] == h
    for (a0, a1), (b0, b1) in zip(rows, rows[1:]):
        assert a1 == b0
    for r, (r0, r1) in enumerate(rows):
        assert outs[r].shape == (3, (r1 - r0) * s, w * s)
    got = np.concatenate(outs, axis=1)
    err = float(np.abs(got - whole).max())
    print(f"{task} {h}x{w} world {world}: bands vs whole max-abs {err:.3e}")
    assert err == 0.0


def test_bands_match_the_oracle():
    P = pkg()
    wt = P.weights.Weights.seeded("classical_sr", 0, True)
    h, w = 44, 37
    x = adjust(wt, np.random.default_rng(12).random((3, h, w), dtype=np.float32))
    outs, _ = run_bands(wt, x, 3)
    got = np.concatenate(outs, axis=1)
    ref = oracle().forward(wt, h, w, x)[0]
    err = float(np.abs(got - ref.reshape(got.shape)).max())
    print(f"bands vs oracle max-abs {err:.3e}")
    assert err <= TOL


def test_band_mode_rejects_the_aux_head_and_whole_image_calls():
    C = capi()
    P = pkg()
    wt = P.weights.Weights.seeded("compressed_sr", 0, False)
    hs = [C.Handle(wt) for _ in range(2)]
    try:
        with pytest.raises(C.S2SError) as ei:
            C.band_init_local(hs)
        assert ei.value.code == C.S2S_ERR_UNSUPPORTED
    finally:
        for h in hs:
            h.close()
    wt = P.weights.Weights.seeded("lightweight_sr", 0, False)
    hs = [C.Handle(wt) for _ in range(2)]
    try:
        C.band_init_local(hs)
        x = np.zeros((3, 16, 16), np.float32)
        with pytest.raises(C.S2SError) as ei:
            hs[0].forward_batch(x[None])
        assert ei.value.code == C.S2S_ERR_INVALID and "s2s_forward_band" in str(ei.value)
    finally:
        for h in hs:
            h.close()


@pytest.mark.parametrize("rows", [1, 4, 8])
def test_peer_store_halo_kernel_in_loopback(rows):
    """The peer-store exchange kernel on one GPU, its neighbours being the plane itself:
    the last `rows` owned rows land in the top halo, the first in the bottom halo, and
    the device-side exchange epoch advances once per exchange (checked inside
    s2s_debug_halo_loopback)."""
    C = capi()
    H = C.Handle(pkg().weights.Weights.seeded("lightweight_sr", 0, True))
    try:
        H.debug_halo_loopback(rows)
    finally:
        H.close()


def test_peer_store_halo_wait_runs_out_without_a_neighbour():
    """No neighbour ever signals: the kernel's bounded waits give up after about a
    second, the call reports S2S_ERR_TIMEOUT, and the handle (and its context) still
    works afterwards."""
    import time
    C = capi()
    H = C.Handle(pkg().weights.Weights.seeded("lightweight_sr", 0, True))
    try:
        t0 = time.time()
        with pytest.raises(C.S2SError) as ei:
            H.debug_halo_loopback(4, missing=True)
        assert "S2S_ERR_TIMEOUT" in str(ei.value) or ei.value.code == 5, ei.value
        assert time.time() - t0 < 30.0
        H.debug_halo_loopback(4)
    finally:
        H.close()

