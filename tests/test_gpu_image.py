"""The device image path against the host pipeline, byte for byte.

s2s_forward_image runs load_rgb's sample scaling + Pre::adjust (k_samples_in), the
forward, and Image::to_rgb8 (k_rgb8) or the PNG scanline filter (k_png_rows) on the
device. Each float step rounds once, as the reference's host code does, so the bytes
must equal oracle.to_rgb8(s2s_forward_batch(oracle.adjust(oracle.load_samples(...))))
exactly: the forward in between is the same deterministic kernel sequence.
"""
import io

import numpy as np
import pytest
from PIL import Image as PILImage

from s2s_testlib import oracle, pkg

pytestmark = pytest.mark.gpu


def capi():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.capi")


def host_path(H, wt, samples, channels, depth):
    """The reference's host pipeline around the library's float forward."""
    O = oracle()
    xs = np.stack([O.adjust(O.load_samples(s, channels, depth), wt.mean, wt.img_range)
                   for s in samples])
    out, aux = H.forward_batch(xs)
    rgb = np.stack([O.to_rgb8(o) for o in out])
    arg = np.stack([O.to_rgb8(a) for a in aux]) if aux is not None else None
    return rgb, arg


def host_filter_choice(rgb):
    from test_png import host_filter_choice as f
    return f(rgb)


@pytest.mark.parametrize("task,B,h,w", [
    ("classical_sr", 1, 37, 29),
    ("classical_sr_x2", 2, 24, 31),
    ("lightweight_sr", 1, 40, 24),
    ("real_sr", 1, 21, 37),
    ("compressed_sr", 3, 16, 16),
])
def test_forward_image_equals_the_host_pipeline(task, B, h, w):
    C = capi()
    P = pkg()
    wt = P.weights.Weights.seeded(task, 0, True)
    samples = np.random.default_rng(h * w + B).integers(0, 256, (B, h, w, 3), dtype=np.uint8)
    H = C.Handle(wt)
    try:
        got, aux = H.forward_image(samples)
        want, want_aux = host_path(H, wt, samples, 3, 8)
        assert got.shape == (B, h * wt.scale, w * wt.scale, 3)
        diff = int((got != want).sum())
        print(f"{task} B={B} {h}x{w}: {diff} bytes differ of {got.size}")
        assert diff == 0
        if task == "compressed_sr":
            assert aux is not None and np.array_equal(aux, want_aux)
        else:
            assert aux is None
        # the PNG scanline form: the filter each row chose and the pixels it encodes
        rows, aux_rows = H.forward_image(samples, png_rows=True)
        Hs, Ws = h * wt.scale, w * wt.scale
        assert rows.shape == (B, Hs, 1 + 3 * Ws)
        for b in range(B):
            assert rows[b, :, 0].tolist() == host_filter_choice(want[b])
            f = C.png_encode_rows(rows[b])
            assert np.array_equal(np.array(PILImage.open(io.BytesIO(f))), want[b])
        if task == "compressed_sr":
            f = C.png_encode_rows(aux_rows[0])
            assert np.array_equal(np.array(PILImage.open(io.BytesIO(f))), want_aux[0])
    finally:
        H.close()


@pytest.mark.parametrize("channels,depth", [(1, 8), (2, 8), (4, 8), (1, 16), (3, 16), (4, 16)])
def test_forward_image_takes_every_decodable_sample_format(channels, depth):
    C = capi()
    P = pkg()
    wt = P.weights.Weights.seeded("lightweight_sr", 0, True)
    h, w = 19, 26
    samples = np.random.default_rng(channels * depth).integers(
        0, 256, (1, h, w, channels * depth // 8), dtype=np.uint8)
    H = C.Handle(wt)
    try:
        got, _ = H.forward_image(samples, depth)
        want, _ = host_path(H, wt, samples, channels, depth)
        assert np.array_equal(got, want)
    finally:
        H.close()


def test_adjust_and_rgb8_device_match_the_oracle_bit_for_bit():
    import torch
    C = capi()
    O = oracle()
    P = pkg()
    wt = P.weights.Weights.seeded("classical_sr", 0, False)
    H = C.Handle(wt)
    st = torch.cuda.current_stream()
    try:
        for channels, depth in [(1, 8), (2, 8), (3, 8), (4, 8), (1, 16), (2, 16), (3, 16),
                                (4, 16)]:
            B, h, w = 2, 13, 17
            s = np.random.default_rng(channels + depth).integers(
                0, 256, (B, h, w, channels * depth // 8), dtype=np.uint8)
            s[0, 0, 0] = 255
            s[0, 0, 1] = 0
            d_s = torch.from_numpy(s).cuda()
            d_x = torch.empty((B, 3, h, w), dtype=torch.float32, device="cuda")
            H.adjust_device(B, h, w, d_s.data_ptr(), channels, depth, d_x.data_ptr(),
                            st.cuda_stream)
            torch.cuda.synchronize()
            want = np.stack([O.adjust(O.load_samples(x, channels, depth), wt.mean, wt.img_range)
                             for x in s])
            got = d_x.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (channels, depth)
    finally:
        H.close()
    # quantisation: special values, both sides of every rounding boundary, random
    k = np.arange(256, dtype=np.float32)
    edges = np.concatenate([(k + np.float32(0.5)) / np.float32(255),
                            np.nextafter((k + np.float32(0.5)) / np.float32(255), np.float32(0)),
                            np.nextafter((k + np.float32(0.5)) / np.float32(255), np.float32(2))])
    special = np.array([np.nan, np.inf, -np.inf, -0.0, 0.0, 1.0, -1e-30, 1.0000001, 3e38],
                       np.float32)
    rnd = np.random.default_rng(3).uniform(-0.5, 1.5, 4000).astype(np.float32)
    vals = np.concatenate([edges, special, rnd])
    B, h, w = 2, 7, 211
    x = np.resize(vals, B * 3 * h * w).astype(np.float32).reshape(B, 3, h, w)
    d_x = torch.from_numpy(x).cuda()
    d_o = torch.empty((B, h, w, 3), dtype=torch.uint8, device="cuda")
    C.rgb8_device(B, h, w, d_x.data_ptr(), d_o.data_ptr(), False, st.cuda_stream)
    d_r = torch.empty((B, h, 1 + 3 * w), dtype=torch.uint8, device="cuda")
    C.rgb8_device(B, h, w, d_x.data_ptr(), d_r.data_ptr(), True, st.cuda_stream)
    torch.cuda.synchronize()
    want = np.stack([O.to_rgb8(i) for i in x])
    assert np.array_equal(d_o.cpu().numpy(), want)
    rows = d_r.cpu().numpy()
    for b in range(B):
        assert rows[b, :, 0].tolist() == host_filter_choice(want[b])
        f = C.png_encode_rows(rows[b])
        assert np.array_equal(np.array(PILImage.open(io.BytesIO(f))), want[b])


def test_png_rows_of_a_wide_image_use_the_large_shared_memory_path():
    import torch
    C = capi()
    O = oracle()
    B, h, w = 1, 3, 9001                                # 54 KB of rows in shared memory
    x = np.random.default_rng(4).uniform(-0.1, 1.1, (B, 3, h, w)).astype(np.float32)
    d_x = torch.from_numpy(x).cuda()
    d_r = torch.empty((B, h, 1 + 3 * w), dtype=torch.uint8, device="cuda")
    C.rgb8_device(B, h, w, d_x.data_ptr(), d_r.data_ptr(), True,
                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = O.to_rgb8(x[0])
    f = C.png_encode_rows(d_r.cpu().numpy()[0])
    assert np.array_equal(np.array(PILImage.open(io.BytesIO(f))), want)
    with pytest.raises(C.S2SError, match="shared memory"):
        C.rgb8_device(1, 1, 40000, d_x.data_ptr(), d_r.data_ptr(), True)


def test_upscale_pngs_batches_mixed_sizes_and_keeps_input_order(tmp_path):
    import importlib
    import subprocess
    import sys
    C = capi()
    P = pkg()
    cli = importlib.import_module("swin2sr_b200.cli")
    from test_png import pil_png, smooth_rgb
    wt = P.weights.Weights.seeded("compressed_sr", 0, True)
    imgs = [smooth_rgb(16, 16, 1), smooth_rgb(24, 17, 2), smooth_rgb(16, 16, 3),
            smooth_rgb(16, 16, 4), smooth_rgb(24, 17, 5)]
    pngs = [pil_png(a, "RGB") for a in imgs]
    H = C.Handle(wt)
    try:
        stats = {}
        outs, auxs = cli.upscale_pngs([H], pngs, batch=2, threads=4, want_aux=True, stats=stats)
        assert stats["images"] == 5 and stats["batches"] == 3
        for a, o, x in zip(imgs, outs, auxs):
            want, want_aux = H.forward_image(a[None])
            assert np.array_equal(np.array(PILImage.open(io.BytesIO(o))), want[0])
            assert np.array_equal(np.array(PILImage.open(io.BytesIO(x))), want_aux[0])
    finally:
        H.close()
    # the same through the script, files in and out
    ck = tmp_path / "cx.safetensors"
    P.weights.save_safetensors(str(ck), wt.tensors, wt.meta)
    src = []
    for k, p in enumerate(pngs[:3]):
        f = tmp_path / f"in{k}.png"
        f.write_bytes(p)
        src.append(str(f))
    r = subprocess.run([sys.executable, str(pkg().__path__[0] + "/cli.py"), "-m", str(ck), "-i",
                        *src, "-o", str(tmp_path / "out"), "--aux", str(tmp_path / "aux"),
                        "--batch", "4"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    for k in range(3):
        got = np.array(PILImage.open(tmp_path / "out" / f"in{k}.png"))
        assert np.array_equal(np.array(PILImage.open(io.BytesIO(outs[k]))), got)
        assert (tmp_path / "aux" / f"in{k}.png").exists()
