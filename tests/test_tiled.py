"""The tiled driver over the backend (src/backend.rs:92-259, src/main.rs:579-662):
crop geometry, the budget-driven tile choice, the halve-on-out-of-memory retry
(host logic with fake backends, no GPU), and the tiled forward on the GPU against
the oracle run through the same tiling."""
import numpy as np
import pytest

from s2s_testlib import TOL, oracle, pkg


def backend_mod():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.backend")


class FakeWeights:
    window, scale, embed, img_range = 8, 2, 60, 1.0
    mean = (0.0, 0.0, 0.0)


class Echo:
    """A backend whose forward is a nearest-neighbour upscale of its input and
    which fails with the driver's out-of-memory message above `limit` pixels."""

    def __init__(self, limit=None):
        self.limit, self.calls = limit, []

    def forward(self, h, w, inp):
        self.calls.append((h, w))
        if self.limit is not None and h * w > self.limit:
            raise RuntimeError("S2S_ERR_OOM: workspace: CUDA_ERROR_OUT_OF_MEMORY (out of memory)")
        x = np.asarray(inp, np.float32).reshape(3, h, w)
        return x.repeat(2, axis=1).repeat(2, axis=2)

    def workspace_bytes(self, h, w):
        return 1000 * ((h // 8 + 1) * 8) * ((w // 8 + 1) * 8)


def test_crop_side_follows_the_reference_padding():
    B = backend_mod()
    assert B.crop_side(640, 640, 0, 32, 8) == 648        # whole image: next multiple + 1 window
    assert B.crop_side(1000, 700, 256, 20, 8) == 312     # tile 256 + 2 x 24 pad = 304 -> 312
    assert B.crop_side(100, 100, 256, 32, 8) == 104      # the crop is clamped to the image


def test_tiled_echo_reassembles_the_image_exactly():
    B = backend_mod()
    img = np.random.default_rng(0).random((3, 45, 67), dtype=np.float32)
    out = B.run_tiled(FakeWeights, Echo(), img, 16, 8)
    want = img.repeat(2, axis=1).repeat(2, axis=2)
    assert np.array_equal(out, want)


def test_auto_tile_uses_the_exact_workspace_figure():
    B = backend_mod()
    be = Echo()
    # whole 100x100 (plane 104^2) fits 1000 * 104^2 bytes
    assert B.auto_tile(FakeWeights, be, 1000 * 104 * 104, 100, 100, 16) == 0
    t = B.auto_tile(FakeWeights, be, 1000 * 104 * 104 - 1, 100, 100, 16)
    assert t > 0 and t % 8 == 0
    side = B.crop_side(100, 100, t, 16, 8)
    assert be.workspace_bytes(side - 8, side - 8) <= 1000 * 104 * 104 - 1


def test_run_with_fallback_halves_on_out_of_memory_only():
    B = backend_mod()
    img = np.random.default_rng(1).random((3, 70, 90), dtype=np.float32)
    notes = []
    be = Echo(limit=40 * 40)
    out, tile = B.run_with_fallback(FakeWeights, be, img, 0, 8, notes.append)
    assert tile in (8, 16) and notes and "OUT_OF_MEMORY" in notes[0]
    assert np.array_equal(out, img.repeat(2, axis=1).repeat(2, axis=2))
    # nothing fits: at a one-window tile the driver's own error comes back
    with pytest.raises(RuntimeError, match="OUT_OF_MEMORY"):
        B.run_with_fallback(FakeWeights, Echo(limit=10), img, 64, 8)

    class Broken(Echo):
        def forward(self, h, w, inp):
            raise RuntimeError("S2S_ERR_CUDA: an illegal memory access")
    with pytest.raises(RuntimeError, match="illegal"):   # not retried
        B.run_with_fallback(FakeWeights, Broken(), img, 64, 8)


class OracleBackend:
    """The CPU oracle behind the same interface (test infrastructure only)."""

    def __init__(self, wt):
        self.wt = wt

    def forward(self, h, w, inp):
        return oracle().forward(self.wt, h, w, np.ascontiguousarray(inp, np.float32))[0].reshape(
            3, h * self.wt.scale, w * self.wt.scale)


@pytest.mark.gpu
def test_tiled_gpu_forward_matches_the_tiled_oracle():
    P = pkg()
    B = backend_mod()
    wt = P.weights.Weights.seeded("classical_sr", 0, True)
    img = np.random.default_rng(5).random((3, 52, 70), dtype=np.float32)
    gpu = B.Gpu(wt)
    try:
        got = B.run_tiled(wt, gpu, img, 24, 8)
        ws = gpu.workspace_bytes(40, 40)
        assert B.auto_tile(wt, gpu, ws, 52, 70, 8) > 0      # the whole image does not fit
    finally:
        gpu.close()
    want = B.run_tiled(wt, OracleBackend(wt), img, 24, 8)
    err = float(np.abs(got - want).max())
    print(f"tiled GPU vs tiled oracle max-abs {err:.3e}")
    assert err <= TOL
