"""Stage-by-stage comparison of the CUDA forward with the oracle's activation dumps.

The reference names every activation for bisection (src/cpu.rs:1405, 1453-1459 and
tools/make_fixture.py --dump); here the forward is stopped after a given launch
(s2s_debug_stop_after) and a workspace buffer is read back (s2s_debug_read) and
compared with the oracle's dump of the same activation, so a failure names the
first op that diverges. Device buffers are token rows [T][Cp]; the oracle's are
NCHW planes.
"""
import importlib

import numpy as np
import pytest

from s2s_testlib import adjust, block_launches, oracle, pkg

pytestmark = pytest.mark.gpu


def rows_to_plane(buf, T, Cp, C, hp, wp, order=None):
    """[T][Cp] rows (image order, or window order given token_pixels) -> [C][hp][wp]."""
    rows = buf.reshape(T, Cp)[:, :C]
    if order is not None:
        img = np.empty_like(rows)
        img[order] = rows
        rows = img
    return rows.T.reshape(C, hp, wp)


@pytest.mark.parametrize("task", ["lightweight_sr", "classical_sr"])
def test_stages_track_the_oracle(task):
    P = pkg()
    capi = importlib.import_module("swin2sr_b200.capi")
    wt = P.weights.Weights.seeded(task, 0, True)
    h, w = 21, 30
    x = adjust(wt, np.random.default_rng(0).random((3, h, w), dtype=np.float32))
    _, _, dumps = oracle().forward(wt, h, w, x, dump=True)
    pl = P.plan.Plan.new(h, w, wt.window, wt.embed)
    C, Cp, T = wt.embed, -(-wt.embed // 64) * 64, pl.plane()
    hd = wt.head_dim
    H = capi.Handle(wt)
    depth0 = wt.depths[0]

    def run_until(n):
        H.debug_stop_after(n)
        H.forward_batch(x[None])

    def cmp(name, got, tol):
        want = dumps[name].reshape(got.shape)
        err = float(np.abs(got - want).max())
        scale = float(np.abs(want).max())
        print(f"{task} {name}: max-abs {err:.3e} (|ref| max {scale:.3f})")
        assert err <= tol * max(1.0, scale), f"{name} diverges: {err:.3e}"

    run_until(2)                                            # pad, conv_first
    cmp("conv_first", rows_to_plane(H.debug_read("F0"), T, Cp, C, pl.hp, pl.wp), 1e-4)
    run_until(3)                                            # + patch_embed
    cmp("patch_embed", rows_to_plane(H.debug_read("S"), T, Cp, C, pl.hp, pl.wp), 2e-2)
    # block 0 (unshifted) and block 1 (shifted) of stage 0; the residual stream is
    # kept in image order, windows exist only inside the attention kernel
    nb = block_launches(wt)
    run_until(3 + nb)
    cmp("layers.0.blocks.0", rows_to_plane(H.debug_read("X"), T, Cp, C, pl.hp, pl.wp), 2e-2)
    run_until(3 + 2 * nb)
    cmp("layers.0.blocks.1", rows_to_plane(H.debug_read("X"), T, Cp, C, pl.hp, pl.wp), 2e-2)
    # the whole first stage (blocks, conv, patch_embed, + stage input)
    run_until(3 + nb * depth0 + 2)
    cmp("layers.0", rows_to_plane(H.debug_read("S"), T, Cp, C, pl.hp, pl.wp), 3e-2)
    H.debug_stop_after(-1)
    H.close()
    del hd
