"""s2s_window_attention_noalloc against the forward's own window attention.

The forward (s2s_forward_batch) is stopped right after the attention launch of a
block (s2s_debug_stop_after); its QKV input and attention output are read back
(s2s_debug_read). The non-allocating entry point then runs on the same QKV, in
device buffers the test owns, for an unshifted and a shifted block back to back on
one stream, so the second call rebuilds the fixed row table the first one used.
Both results must match the forward's. The file is named to be collected last.
"""
import importlib

import numpy as np
import pytest

from s2s_testlib import adjust, block_launches, pkg

pytestmark = pytest.mark.gpu

# The same kernel on the same fp16 inputs: identical results are expected; the
# tolerance is one fp16 step at |x| <= 1.
TOL = 1e-3


@pytest.mark.parametrize("task", ["lightweight_sr", "classical_sr"])
def test_noalloc_attention_matches_forward(task, monkeypatch):
    import torch

    # the entry point reads the single-term QKV layout that the QKV GEMM writes: the
    # forward it is compared with runs single-term operands (S2S_SPLIT=0; the 60-wide
    # network otherwise carries two-term ones) and the QKV GEMM + attention kernel pair
    # (S2S_ATTN=mma; the 180-wide network otherwise fuses them), both read at create
    monkeypatch.setenv("S2S_SPLIT", "0")
    monkeypatch.setenv("S2S_ATTN", "mma")
    P = pkg()
    capi = importlib.import_module("swin2sr_b200.capi")
    wt = P.weights.Weights.seeded(task, 0, True)
    B, h, w = 2, 21, 30
    x = adjust(wt, np.random.default_rng(4).random((B, 3, h, w), dtype=np.float32))
    pl = P.plan.Plan.new(h, w, wt.window, wt.embed)
    hp, wp = pl.hp, pl.wp
    T, Cp, C = B * hp * wp, -(-wt.embed // 64) * 64, wt.embed
    H = capi.Handle(wt)
    try:
        want = {}
        for block, stop in ((0, 3 + 2), (1, 3 + block_launches(wt) + 2)):
            H.debug_stop_after(stop)  # pad, conv_first, patch_embed, [block 0,] qkv, attention
            H.forward_batch(x)
            qkv = H.debug_read("QKV")
            ao = H.debug_read("AO").reshape(T, Cp)
            want[block] = (qkv, ao)
        H.debug_stop_after(-1)

        dev = torch.device("cuda:0")
        st = torch.cuda.Stream(dev)
        d_qkv = {b: torch.from_numpy(q).to(dev, torch.float16).contiguous()
                 for b, (q, _) in want.items()}
        d_out = {b: torch.zeros((T, Cp), dtype=torch.float16, device=dev) for b in want}
        torch.cuda.synchronize()
        for block in (1, 0):  # two calls in a row on one stream: shifted, then unshifted
            H.window_attention_noalloc(0, block, B, hp, wp, d_qkv[block].data_ptr(),
                                       d_out[block].data_ptr(), Cp, st.cuda_stream)
        st.synchronize()
        for block in (0, 1):
            got = d_out[block].float().cpu().numpy()
            ref = want[block][1]
            err = float(np.abs(got[:, :C] - ref[:, :C]).max())
            print(f"{task} block {block}: max-abs {err:.3e}")
            assert err <= TOL, f"block {block}: {err:.3e}"
            assert np.all(got[:, C:] == 0), "columns past embed must stay untouched"

        # beyond the fixed scratch: rejected before anything is enqueued
        side = 1032  # 1032 x 1032 > S2S_NOALLOC_MAX_TOKENS = 1048576
        with pytest.raises(capi.S2SError) as ei:
            H.window_attention_noalloc(0, 0, 1, side, side, d_qkv[0].data_ptr(),
                                       d_out[0].data_ptr(), Cp, st.cuda_stream)
        assert ei.value.code == capi.S2S_ERR_INVALID
        assert "S2S_NOALLOC_MAX_TOKENS" in str(ei.value)
        # the handle still works after the rejection
        H.window_attention_noalloc(0, 0, B, hp, wp, d_qkv[0].data_ptr(), d_out[1].data_ptr(),
                                   Cp, st.cuda_stream)
        st.synchronize()
        assert torch.equal(d_out[1], d_out[0])
    finally:
        H.close()
