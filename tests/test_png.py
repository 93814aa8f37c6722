"""The image path's host side (no GPU): the PNG codec of libs2s.so, the Image mirror
of src/image.rs and the oracle's to_rgb8 / sample scaling.

The decoder is pinned against PIL (an independent PNG implementation) and against a
PNG writer restated here from the PNG specification, which exercises what PIL does
not write: every filter type, Adam7 interlacing, 16-bit colour. The encoder is
pinned by decoding its files with PIL and zlib. The reference's own tests hold no
image vectors; its decode contract (src/image.rs:48-96) is restated in the oracle.
"""
import io
import struct
import zlib

import numpy as np
import pytest
from PIL import Image as PILImage

from s2s_testlib import oracle, pkg


def capi():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.capi")


def image_mod():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.image")


# ---------------------------------------------------------------- a spec-level writer

ADAM7 = [(0, 0, 8, 8), (0, 4, 8, 8), (4, 0, 8, 4), (0, 2, 4, 4), (2, 0, 4, 2), (0, 1, 2, 2),
         (1, 0, 2, 1)]
CHANNELS = {0: 1, 2: 3, 3: 1, 4: 2, 6: 4}


def paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
    return a if pa <= pb and pa <= pc else (b if pb <= pc else c)


def filter_row(ft, cur, prev, bpp):
    out = bytearray(len(cur))
    for i in range(len(cur)):
        a = cur[i - bpp] if i >= bpp else 0
        b = prev[i] if prev is not None else 0
        c = prev[i - bpp] if (prev is not None and i >= bpp) else 0
        pred = [0, a, b, (a + b) >> 1, paeth(a, b, c)][ft]
        out[i] = (cur[i] - pred) & 255
    return bytes(out)


def chunk(t, body):
    return struct.pack(">I", len(body)) + t + body + struct.pack(">I", zlib.crc32(t + body))


def spec_png(rows_bytes, w, h, ctype, depth, interlace=0, filters=None, rng=None):
    """A PNG whose image is `rows_bytes` [h][w * bpp] (bytes per row as stored, 16-bit
    big-endian), each scanline filtered with `filters` (a type, 'random', or None=0)."""
    bpp = max(1, CHANNELS[ctype] * depth // 8)
    raw = bytearray()

    def emit(sub):  # sub: list of row byte strings
        prev = None
        for r in sub:
            ft = filters if isinstance(filters, int) else (
                int(rng.integers(0, 5)) if filters == "random" else 0)
            raw.append(ft)
            raw.extend(filter_row(ft, r, prev, bpp) if ft < 5 else r)
            prev = r
    if not interlace:
        emit([bytes(rows_bytes[y]) for y in range(h)])
    else:
        for y0, x0, dy, dx in ADAM7:
            sub = []
            for y in range(y0, h, dy):
                row = rows_bytes[y]
                sub.append(b"".join(bytes(row[x * bpp:(x + 1) * bpp]) for x in range(x0, w, dx)))
            if sub and sub[0]:
                emit(sub)
    ihdr = struct.pack(">IIBBBBB", w, h, depth, ctype, 0, 0, interlace)
    z = zlib.compress(bytes(raw), 6)
    return b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", z[:len(z) // 2]) + \
        chunk(b"tEXt", b"k\x00v") + chunk(b"IDAT", z[len(z) // 2:]) + chunk(b"IEND", b"")


def pil_png(arr, mode):
    buf = io.BytesIO()
    PILImage.fromarray(arr, mode=mode).save(buf, format="PNG")
    return buf.getvalue()


# ---------------------------------------------------------------- decoder

@pytest.mark.parametrize("mode,ch", [("L", 1), ("LA", 2), ("RGB", 3), ("RGBA", 4)])
def test_decoder_matches_pil_8bit(mode, ch):
    C = capi()
    rng = np.random.default_rng(ch)
    shape = (23, 41) if ch == 1 else (23, 41, ch)
    a = rng.integers(0, 256, shape, dtype=np.uint8)
    f = pil_png(a, mode)
    assert C.png_header(f) == (41, 23, ch, 8)
    s, d = C.png_decode(f)
    assert d == 8 and s.shape == (23, 41, ch)
    assert np.array_equal(s.reshape(shape), a)


def test_decoder_matches_pil_16bit_grey():
    C = capi()
    a = np.random.default_rng(5).integers(0, 65536, (19, 33), dtype=np.uint16)
    buf = io.BytesIO()
    PILImage.fromarray(a.astype(np.uint16)).save(buf, format="PNG")   # mode I;16
    s, d = C.png_decode(buf.getvalue())
    assert d == 16 and s.shape == (19, 33, 2)
    got = (s[..., 0].astype(np.uint16) << 8) | s[..., 1]
    assert np.array_equal(got, np.array(PILImage.open(io.BytesIO(buf.getvalue()))).astype(np.uint16))
    assert np.array_equal(got, a)


@pytest.mark.parametrize("ctype", [0, 2, 4, 6])
@pytest.mark.parametrize("depth", [8, 16])
@pytest.mark.parametrize("interlace", [0, 1])
@pytest.mark.parametrize("hw", [(1, 1), (3, 5), (9, 17), (16, 13)])
def test_decoder_unfilters_every_filter_type_and_adam7(ctype, depth, interlace, hw):
    C = capi()
    h, w = hw
    rng = np.random.default_rng(ctype * 100 + depth + interlace + h * w)
    bpp = CHANNELS[ctype] * depth // 8
    # smooth-ish rows so every predictor matters, plus noise
    base = (np.arange(w * bpp)[None, :] * 3 + np.arange(h)[:, None] * 7) % 256
    rows = ((base + rng.integers(0, 40, (h, w * bpp))) % 256).astype(np.uint8)
    f = spec_png(rows, w, h, ctype, depth, interlace, "random", rng)
    s, d = C.png_decode(f)
    assert d == depth and s.shape == (h, w, bpp)
    assert np.array_equal(s.reshape(h, w * bpp), rows)


def test_decoder_refusals_follow_the_reference():
    C = capi()
    # src/image.rs:55-65: indexed colour and sub-byte depths are refused
    with pytest.raises(C.S2SError, match="unsupported png colour type Indexed") as ei:
        C.png_header(pil_png(np.zeros((8, 8), np.uint8), "P"))
    assert ei.value.code == C.S2S_ERR_INVALID
    with pytest.raises(C.S2SError, match="unsupported png bit depth One"):
        C.png_decode(pil_png(np.zeros((8, 8), bool), "1"))
    rows4 = np.zeros((4, 2), np.uint8)  # 4 pixels of 4 bits = 2 bytes a row
    ihdr = struct.pack(">IIBBBBB", 4, 4, 4, 0, 0, 0, 0)
    f4 = b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + \
        chunk(b"IDAT", zlib.compress(b"".join(b"\x00" + r.tobytes() for r in rows4))) + \
        chunk(b"IEND", b"")
    with pytest.raises(C.S2SError, match="unsupported png bit depth Four"):
        C.png_decode(f4)


def test_decoder_rejects_damaged_files():
    C = capi()
    rows = np.random.default_rng(1).integers(0, 256, (12, 10 * 3), dtype=np.uint8)
    good = spec_png(rows, 10, 12, 2, 8)
    assert np.array_equal(C.png_decode(good)[0].reshape(12, 30), rows)
    with pytest.raises(C.S2SError, match="signature"):
        C.png_decode(b"GIF89a" + good[6:])
    bad = bytearray(good)
    bad[60] ^= 0x55                       # inside the first IDAT: CRC no longer matches
    with pytest.raises(C.S2SError, match="CRC mismatch"):
        C.png_decode(bytes(bad))
    with pytest.raises(C.S2SError, match="truncated"):
        C.png_decode(good[:50])
    with pytest.raises(C.S2SError, match="filter type 5"):
        C.png_decode(spec_png(rows, 10, 12, 2, 8, 0, 5))
    # image data that ends early
    ihdr = struct.pack(">IIBBBBB", 10, 12, 8, 2, 0, 0, 0)
    short = zlib.compress(b"\x00" * 31 * 5)
    f = b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", short) + chunk(b"IEND", b"")
    with pytest.raises(C.S2SError, match="truncated PNG image data"):
        C.png_decode(f)
    s = np.empty(10, np.uint8)
    L = C.load()
    rc = L.s2s_png_decode(good, len(good), s.ctypes.data, s.nbytes)
    assert rc == C.S2S_ERR_INVALID and b"sample buffer" in L.s2s_last_error(None)


# ---------------------------------------------------------------- encoder

def host_filter_choice(rgb):
    """The per-row choice the encoder (host and device) makes: least sum of
    |filtered byte| read as a signed byte, ties to the lower type."""
    h, w, _ = rgb.shape
    cur = rgb.reshape(h, w * 3).astype(np.int32)
    out = []
    for y in range(h):
        x = cur[y]
        p = cur[y - 1] if y else np.zeros_like(x)
        a = np.concatenate([[0, 0, 0], x[:-3]])
        c = np.concatenate([[0, 0, 0], p[:-3]])
        pp = a + p - c
        pa, pb, pc = np.abs(pp - a), np.abs(pp - p), np.abs(pp - c)
        pae = np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, p, c))
        preds = [0, a, p, (a + p) >> 1, pae]
        costs = [int(np.abs(((x - q) & 255).astype(np.uint8).astype(np.int8).astype(np.int32)).sum())
                 for q in preds]
        out.append(int(np.argmin(costs)))
    return out


def idat_of(f):
    off, z = 8, b""
    while off < len(f):
        n = struct.unpack(">I", f[off:off + 4])[0]
        t = f[off + 4:off + 8]
        if t == b"IDAT":
            z += f[off + 8:off + 8 + n]
        off += 12 + n
    return z


def smooth_rgb(h, w, seed):
    rng = np.random.default_rng(seed)
    y, x = np.mgrid[0:h, 0:w]
    ch = [127 + 100 * np.sin(x / (7 + 3 * k) + y / (11 + k)) for k in range(3)]
    a = np.stack(ch, -1) + rng.normal(0, 6, (h, w, 3))
    return np.clip(a, 0, 255).astype(np.uint8)


@pytest.mark.parametrize("h,w,level,threads", [
    (1, 1, -1, 0), (7, 3, 0, 1), (31, 47, 1, 2), (240, 320, 6, 0), (700, 500, 9, 8),
    (513, 1025, -1, 3),
])
def test_encoder_roundtrips_through_pil_and_zlib(h, w, level, threads):
    C = capi()
    a = smooth_rgb(h, w, h + w)
    f = C.png_encode_rgb8(a, level, threads)
    assert f[:8] == b"\x89PNG\r\n\x1a\n"
    im = PILImage.open(io.BytesIO(f))
    assert im.mode == "RGB" and im.size == (w, h)
    assert np.array_equal(np.array(im), a)
    raw = zlib.decompress(idat_of(f))           # checks the combined Adler-32
    assert len(raw) == h * (1 + 3 * w)
    assert [raw[y * (1 + 3 * w)] for y in range(h)] == host_filter_choice(a)
    s, d = C.png_decode(f)
    assert d == 8 and np.array_equal(s, a)


def test_parallel_deflate_is_one_valid_stream_and_compresses():
    C = capi()
    a = smooth_rgb(900, 700, 3)                 # 1.9 MB of scanlines: several segments
    one = C.png_encode_rgb8(a, 6, 1)
    many = C.png_encode_rgb8(a, 6, 16)
    assert np.array_equal(np.array(PILImage.open(io.BytesIO(many))), a)
    assert zlib.decompress(idat_of(many)) == zlib.decompress(idat_of(one))
    # primed segments cost little against one serial stream
    assert len(many) <= 1.02 * len(one) + 4096
    assert len(one) < a.nbytes


def test_encode_rows_takes_prefiltered_scanlines():
    C = capi()
    rng = np.random.default_rng(9)
    a = smooth_rgb(37, 29, 4)
    rows = []
    prev = None
    for y in range(37):
        ft = int(rng.integers(0, 5))
        cur = a[y].tobytes()
        rows.append(bytes([ft]) + filter_row(ft, cur, prev, 3))
        prev = cur
    buf = np.frombuffer(b"".join(rows), np.uint8).reshape(37, 1 + 29 * 3)
    f = C.png_encode_rows(buf, 1, 2)
    assert np.array_equal(np.array(PILImage.open(io.BytesIO(f))), a)
    bad = buf.copy()
    bad[5, 0] = 7
    with pytest.raises(C.S2SError, match="scanline 5 has filter type 7"):
        C.png_encode_rows(bad)


# ---------------------------------------------------------------- to_rgb8 and samples

def test_to_rgb8_known_answers():
    O = oracle()
    M = image_mod()
    v = np.array([-np.inf, -1.0, -0.0, 0.0, 0.25, 0.5, 0.998, 1.0, 1.5, np.inf, np.nan,
                  1.0 / 255.0, 254.5 / 255.0], np.float32)
    want = [0, 0, 0, 0, 64, 128, 254, 255, 255, 255, 255, 1, 255]
    img = np.stack([v, v[::-1], v]).reshape(3, 1, -1)
    got = O.to_rgb8(img)
    assert got.shape == (1, v.size, 3)
    assert got[0, :, 0].tolist() == want
    assert got[0, :, 1].tolist() == want[::-1]
    assert np.array_equal(M.Image(v.size, 1, img).to_rgb8(), got)
    # every output level is reached from its own centre and rounds half up
    k = np.arange(256, dtype=np.float32)
    assert O.to_rgb8(np.stack([k / np.float32(255)] * 3)[:, None, :])[0, :, 0].tolist() == \
        list(range(256))


@pytest.mark.parametrize("channels,depth", [(1, 8), (2, 8), (3, 8), (4, 8), (1, 16), (3, 16),
                                            (4, 16)])
def test_samples_to_image_matches_the_oracle(channels, depth):
    O = oracle()
    M = image_mod()
    s = np.random.default_rng(channels + depth).integers(
        0, 256, (6, 11, channels * depth // 8), dtype=np.uint8)
    img = M.samples_to_image(s, depth)
    ref = O.load_samples(s, channels, depth)
    assert img.data.dtype == np.float32 and np.array_equal(img.data, ref)
    # the extremes map to exactly 0 and 1
    z = np.zeros_like(s)
    f = np.full_like(s, 255)
    assert O.load_samples(z, channels, depth).max() == 0.0
    assert np.all(O.load_samples(f, channels, depth) == 1.0)


def test_image_load_save_roundtrip(tmp_path):
    M = image_mod()
    a = smooth_rgb(21, 34, 2)
    p = str(tmp_path / "x.png")
    M.save_rgb(p, 34, 21, a.tobytes())
    img = M.load_rgb(p)
    assert (img.w, img.h) == (34, 21)
    assert np.array_equal(img.to_rgb8(), a)
    with pytest.raises(ValueError):
        M.save_rgb(p, 35, 21, a.tobytes())
    (tmp_path / "bad.png").write_bytes(b"nope")
    with pytest.raises(RuntimeError, match="bad.png: .*signature"):
        M.load_rgb(str(tmp_path / "bad.png"))


# ---------------------------------------------------------------- the multi-image driver

def cli_mod():
    pkg()
    import importlib
    return importlib.import_module("swin2sr_b200.cli")


def test_batches_group_same_size_images_in_input_order():
    cli = cli_mod()
    hd = [(16, 16, 3, 8), (20, 16, 3, 8), (16, 16, 3, 8), (16, 16, 1, 8), (16, 16, 3, 8),
          (16, 16, 3, 8)]
    assert cli.plan_batches(hd, 2) == [((16, 16, 3, 8), [0, 2]), ((16, 16, 3, 8), [4, 5]),
                                       ((20, 16, 3, 8), [1]), ((16, 16, 1, 8), [3])]
    assert cli.plan_batches(hd, 8)[0] == ((16, 16, 3, 8), [0, 2, 4, 5])
    assert cli.plan_batches([], 4) == []
    with pytest.raises(ValueError):
        cli.plan_batches(hd, 0)


def test_cli_refuses_aux_for_a_single_output_head(tmp_path, capsys):
    cli = cli_mod()
    P = pkg()
    wt = P.weights.Weights.seeded("lightweight_sr", 0)
    ck = tmp_path / "lw.safetensors"
    P.weights.save_safetensors(str(ck), wt.tensors, wt.meta)
    src = tmp_path / "in.png"
    src.write_bytes(pil_png(smooth_rgb(16, 16, 1), "RGB"))
    rc = cli.main(["-m", str(ck), "-i", str(src), "-o", str(tmp_path / "o.png"),
                   "--aux", str(tmp_path / "a.png"), "-q"])
    assert rc == 1
    assert "only the compressed_sr head" in capsys.readouterr().err


class _FakeWeights:
    window, scale = 8, 2

    def __init__(self, upsampler):
        self.upsampler = upsampler


class _FakeHandle:
    """Stands in for capi.Handle in the driver's host logic: "upscales" by pixel
    repetition and returns PNG scanlines with filter type 0 (no GPU involved)."""

    def __init__(self, upsampler="pixelshuffle", fail_on=None):
        self.wt = _FakeWeights(upsampler)
        self.calls = []
        self.fail_on = fail_on

    def forward_image(self, samples, bit_depth=8, png_rows=False):
        assert png_rows
        B, h, w, cb = samples.shape
        self.calls.append((B, h, w, cb, bit_depth))
        if self.fail_on is not None and (h, w) == self.fail_on:
            raise RuntimeError("fake device failure")
        ch = cb // (bit_depth // 8)
        px = samples[..., ::bit_depth // 8][..., :ch]          # high bytes of 16-bit samples
        rgb = px if ch >= 3 else np.repeat(px[..., :1], 3, axis=-1)
        rgb = np.ascontiguousarray(rgb[..., :3])
        up = rgb.repeat(2, axis=1).repeat(2, axis=2)
        rows = np.zeros((B, 2 * h, 1 + 6 * w), np.uint8)
        rows[:, :, 1:] = up.reshape(B, 2 * h, 6 * w)
        aux = None
        if self.wt.upsampler == "pixelshuffle_aux":
            aux = np.zeros((B, h, 1 + 3 * w), np.uint8)
            aux[:, :, 1:] = rgb.reshape(B, h, 3 * w)
        return rows, aux


def test_upscale_pngs_orders_batches_and_aux_on_the_host():
    cli = cli_mod()
    imgs = [smooth_rgb(16, 16, 1), smooth_rgb(16, 24, 2), smooth_rgb(16, 16, 3),
            smooth_rgb(16, 16, 4), smooth_rgb(16, 24, 5)]
    pngs = [pil_png(a, "RGB") for a in imgs]
    grey = np.random.default_rng(6).integers(0, 65536, (16, 16), dtype=np.uint16)
    buf = io.BytesIO()
    PILImage.fromarray(grey).save(buf, format="PNG")            # 16-bit grey
    pngs.append(buf.getvalue())
    hs = [_FakeHandle("pixelshuffle_aux"), _FakeHandle("pixelshuffle_aux")]
    stats = {}
    outs, auxs = cli.upscale_pngs(hs, pngs, batch=2, threads=3, want_aux=True, stats=stats)
    assert stats["images"] == 6 and stats["batches"] == 4
    assert stats["output_mpix"] == pytest.approx(sum(a.shape[0] * a.shape[1] * 4 for a in imgs
                                                     + [grey]) / 1e6)
    calls = sorted(c for h in hs for c in h.calls)
    assert calls == sorted([(2, 16, 16, 3, 8), (1, 16, 16, 3, 8), (2, 16, 24, 3, 8),
                            (1, 16, 16, 2, 16)])
    for a, o, x in zip(imgs, outs, auxs):
        assert np.array_equal(np.array(PILImage.open(io.BytesIO(o))),
                              a.repeat(2, axis=0).repeat(2, axis=1))
        assert np.array_equal(np.array(PILImage.open(io.BytesIO(x))), a)
    g8 = (grey >> 8).astype(np.uint8)
    assert np.array_equal(np.array(PILImage.open(io.BytesIO(outs[-1]))),
                          np.repeat(g8[..., None], 3, -1).repeat(2, axis=0).repeat(2, axis=1))
    # without --aux nothing is encoded for it
    outs2, auxs2 = cli.upscale_pngs([_FakeHandle("pixelshuffle_aux")], pngs[:2], batch=4)
    assert auxs2 == [None, None] and outs2[0] == outs[0]


def test_upscale_pngs_reports_device_errors_and_small_images():
    cli = cli_mod()
    pngs = [pil_png(smooth_rgb(16, 16, 1), "RGB"), pil_png(smooth_rgb(16, 24, 2), "RGB")]
    with pytest.raises(RuntimeError, match="fake device failure"):
        cli.upscale_pngs([_FakeHandle(fail_on=(16, 24))], pngs, batch=1, threads=2)
    with pytest.raises(ValueError, match="smaller than one 8x8 window"):
        cli.upscale_pngs([_FakeHandle()], [pil_png(smooth_rgb(7, 16, 3), "RGB")])
    with pytest.raises(ValueError):
        cli.upscale_pngs([], pngs)


def test_decoder_survives_corrupt_and_hostile_files():
    """Random byte flips (with the CRCs recomputed, so the damage reaches inflate and
    the unfilter), truncation at every chunk boundary and absurd dimensions end in
    S2SError, never a crash or a read or write outside the buffers."""
    C = capi()
    rng = np.random.default_rng(31)
    rows = rng.integers(0, 256, (13, 11 * 4), dtype=np.uint8)
    base = spec_png(rows, 11, 13, 6, 8, 1, "random", rng)

    def rechunk(data):  # recompute every chunk's CRC
        out, off = bytearray(data[:8]), 8
        while off + 12 <= len(data):
            n = struct.unpack(">I", data[off:off + 4])[0]
            if off + 12 + n > len(data):
                break
            body = data[off + 4:off + 8 + n]
            out += data[off:off + 8 + n] + struct.pack(">I", zlib.crc32(body))
            off += 12 + n
        return bytes(out)

    outcomes = {"ok": 0, "error": 0}
    for _ in range(300):
        b = bytearray(base)
        for _ in range(int(rng.integers(1, 6))):
            b[int(rng.integers(8, len(b)))] = int(rng.integers(0, 256))
        try:
            C.png_decode(rechunk(bytes(b)))
            outcomes["ok"] += 1
        except (C.S2SError, MemoryError, ValueError):
            outcomes["error"] += 1
    assert outcomes["error"] > 0
    # a cut before the last IDAT chunk is complete loses image data (one after it, a
    # missing IEND, decodes: the image is all there)
    last_idat_end = base.rindex(b"IDAT") - 4 + 12 + struct.unpack(
        ">I", base[base.rindex(b"IDAT") - 4:base.rindex(b"IDAT")])[0]
    for cut in range(8, last_idat_end, 7):
        with pytest.raises(C.S2SError):
            C.png_decode(base[:cut])
    assert np.array_equal(C.png_decode(base[:last_idat_end])[0].reshape(13, 44), rows)
    for w, h in [((1 << 31) - 1, (1 << 31) - 1), (1 << 20, 1 << 20), (1 << 17, (1 << 17) + 1),
                 (0, 5), (5, 0)]:
        ihdr = struct.pack(">IIBBBBB", w, h, 8, 6, 0, 0, 0)
        f = b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", zlib.compress(b"\0" * 64)) \
            + chunk(b"IEND", b"")
        with pytest.raises(C.S2SError, match="too large|invalid PNG header"):
            C.png_header(f)
        L = C.load()
        assert L.s2s_png_decode(f, len(f), None, 0) == C.S2S_ERR_INVALID
    # exactly 2^34 pixels passes the dimension check, but 16-bit RGBA of that size
    # (128 GiB of filtered rows) cannot come out of a tiny zlib stream: the header query
    # refuses it, so no caller sizes a sample buffer from it (png_decode would
    # otherwise allocate the output before the decoder runs)
    for depth, ctype in [(16, 6), (8, 0)]:
        ihdr = struct.pack(">IIBBBBB", 1 << 17, 1 << 17, depth, ctype, 0, 0, 0)
        f = b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", zlib.compress(b"\0" * 64)) \
            + chunk(b"IEND", b"")
        with pytest.raises(C.S2SError, match="truncated PNG image data"):
            C.png_header(f)
        with pytest.raises(C.S2SError, match="truncated PNG image data"):
            C.png_decode(f)
        assert L.s2s_png_decode(f, len(f), None, 0) == C.S2S_ERR_INVALID
    # a header-only prefix (no image data yet) still answers the header query
    ihdr = struct.pack(">IIBBBBB", 1 << 17, 1 << 17, 8, 2, 0, 0, 0)
    assert C.png_header(b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr)) == (1 << 17, 1 << 17, 3, 8)


class _FakeFloatHandle:
    """Stands in for capi.Handle in the tiled path: forward_batch undoes the mean
    adjustment and repeats each pixel `scale` times (a local operation, so every
    tiling gives the whole-image result); it runs out of memory above `limit` pixels."""

    def __init__(self, wt, limit=None):
        self.wt, self.limit, self.sizes = wt, limit, []

    def forward_batch(self, x):
        B, _, h, w = x.shape
        self.sizes.append((h, w))
        if self.limit is not None and h * w > self.limit:
            capi_mod = cli_mod().capi
            raise capi_mod.S2SError(capi_mod.S2S_ERR_OOM,
                                    "cudaMalloc: CUDA_ERROR_OUT_OF_MEMORY (fake)")
        m = np.asarray(self.wt.mean, np.float32).reshape(1, 3, 1, 1)
        img = x / np.float32(self.wt.img_range) + m
        s = self.wt.scale
        return img.repeat(s, axis=2).repeat(s, axis=3), None

    def workspace_bytes(self, B, h, w):
        return B * h * w * 1000


def test_tiled_cli_path_matches_the_whole_image_and_recovers_from_oom():
    cli = cli_mod()
    P = pkg()
    wt = P.weights.Weights.seeded("classical_sr", 0)
    imgs = [smooth_rgb(40, 56, 1), smooth_rgb(33, 20, 2)]
    pngs = [pil_png(a, "RGB") for a in imgs]
    want = [np.array(a).repeat(4, axis=0).repeat(4, axis=1) for a in imgs]
    for tile in (16, 0):
        outs, ran = cli.upscale_pngs_tiled([_FakeFloatHandle(wt), _FakeFloatHandle(wt)], pngs,
                                           tile, 8)
        assert ran == [tile, tile]
        for o, w_ in zip(outs, want):
            assert np.array_equal(np.array(PILImage.open(io.BytesIO(o))), w_)
    notes = []
    h = _FakeFloatHandle(wt, limit=40 * 40)
    outs, ran = cli.upscale_pngs_tiled([h], pngs[:1], 0, 8, note=notes.append)
    # 40x56 (2240 px) is over the limit; half the long side, a 24-pixel tile with 8 of
    # context, makes crops of at most 40x40 = 1600 px, which fit
    assert ran == [24] and len(notes) == 1 and "retrying with a 24x24 tile" in notes[0]
    assert np.array_equal(np.array(PILImage.open(io.BytesIO(outs[0]))), want[0])
    assert max(a * b for a, b in h.sizes[1:]) <= 40 * 40


class _FakeImageHandle(_FakeFloatHandle):
    """The batched (whole-image) CLI path's handle: its image forward runs out of
    memory, as a batch too large for the device would."""

    def forward_image(self, samples, depth, png_rows=True):
        capi_mod = cli_mod().capi
        raise capi_mod.S2SError(capi_mod.S2S_ERR_OOM,
                                "cudaMalloc: CUDA_ERROR_OUT_OF_MEMORY (fake)")


def test_whole_image_cli_path_falls_back_to_tiles_and_says_so_under_quiet():
    """--tile 0 (the default, batched path): a batch that runs out of device memory is
    redone image by image from tile 0 - the whole image alone, then halving tiles - as
    the reference retries (src/main.rs:579-657). The note for leaving the exact
    whole-image mode goes to note_exact, which the CLI prints even under -q."""
    cli = cli_mod()
    P = pkg()
    wt = P.weights.Weights.seeded("classical_sr", 0)
    imgs = [smooth_rgb(40, 56, 1), smooth_rgb(33, 20, 2)]
    pngs = [pil_png(a, "RGB") for a in imgs]
    want = [np.array(a).repeat(4, axis=0).repeat(4, axis=1) for a in imgs]
    exact = []
    outs, aux = cli.upscale_pngs([_FakeImageHandle(wt, limit=40 * 40)], pngs, batch=2, pad=8,
                                 note=None, note_exact=exact.append)
    for o, w_ in zip(outs, want):
        assert np.array_equal(np.array(PILImage.open(io.BytesIO(o))), w_)
    assert aux == [None, None]
    # only the 40x56 image needs tiles (33x20 fits whole)
    assert len(exact) == 1 and "--tile 0 is the only exact mode" in exact[0]
    assert "retrying with a 24x24 tile" in exact[0]


def test_cli_refuses_aux_with_tiling(tmp_path, capsys):
    cli = cli_mod()
    P = pkg()
    wt = P.weights.Weights.seeded("compressed_sr", 0)
    ck = tmp_path / "cx.safetensors"
    P.weights.save_safetensors(str(ck), wt.tensors, wt.meta)
    src = tmp_path / "in.png"
    src.write_bytes(pil_png(smooth_rgb(16, 16, 1), "RGB"))
    rc = cli.main(["-m", str(ck), "-i", str(src), "-o", str(tmp_path / "o.png"), "--aux",
                   str(tmp_path / "a.png"), "--tile", "64", "-q"])
    assert rc == 1 and "only for a single pass" in capsys.readouterr().err
    rc = cli.main(["-m", str(ck), "-i", str(src), "-o", str(tmp_path / "o.png"), "--tile", "x"])
    assert rc == 1 and "--tile takes a number" in capsys.readouterr().err
