"""ctypes binding of the C ABI in include/s2s.h (libs2s.so, built by build.py).

This is the same binding a Rust maintainer writes with `extern "C"` blocks: plain
structs, plain pointers. The library MUST be present: there is no CPU fallback,
and loading fails loudly when libs2s.so has not been built.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libs2s.so"

S2S_OK, S2S_ERR_OOM, S2S_ERR_INVALID, S2S_ERR_CUDA, S2S_ERR_NCCL, S2S_ERR_TIMEOUT, \
    S2S_ERR_UNSUPPORTED, S2S_ERR_SELFTEST = range(8)
STATUS_NAMES = {0: "S2S_OK", 1: "S2S_ERR_OOM", 2: "S2S_ERR_INVALID", 3: "S2S_ERR_CUDA",
                4: "S2S_ERR_NCCL", 5: "S2S_ERR_TIMEOUT", 6: "S2S_ERR_UNSUPPORTED",
                7: "S2S_ERR_SELFTEST"}
UPSAMPLER_CODE = {"pixelshuffle": 0, "pixelshuffledirect": 1, "nearest+conv": 2,
                  "pixelshuffle_aux": 3}

# Every entry point include/s2s.h declares.
EXPORTS = ("s2s_create", "s2s_forward", "s2s_forward_batch", "s2s_forward_device",
           "s2s_aux_dims", "s2s_uploaded_bytes", "s2s_workspace_bytes", "s2s_last_error",
           "s2s_profile_enable", "s2s_profile_report", "s2s_launch_count", "s2s_destroy",
           "s2s_version", "s2s_debug_stop_after", "s2s_debug_read", "s2s_debug_halo_loopback",
           "s2s_window_attention_noalloc", "s2s_band_unique_id", "s2s_band_init",
           "s2s_band_init_local", "s2s_band_rows", "s2s_forward_band", "s2s_forward_band_host",
           "s2s_band_partition", "s2s_band_halo_ops", "s2s_png_header", "s2s_png_decode",
           "s2s_png_encode_rgb8", "s2s_png_encode_rows", "s2s_free", "s2s_adjust_device",
           "s2s_rgb8_device", "s2s_forward_image", "s2s_selftest")
BAND_ID_BYTES = 128


class S2SConfig(ctypes.Structure):
    _fields_ = [("upsampler", ctypes.c_int), ("scale", ctypes.c_int), ("window", ctypes.c_int),
                ("embed", ctypes.c_int), ("heads", ctypes.c_int), ("mlp_ratio", ctypes.c_int),
                ("n_depths", ctypes.c_int), ("depths", ctypes.c_int * 16),
                ("img_range", ctypes.c_float), ("mean", ctypes.c_float * 3)]


class S2STensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.POINTER(ctypes.c_float)),
                ("ndim", ctypes.c_int), ("shape", ctypes.c_int64 * 4)]


class S2SError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None


def load() -> ctypes.CDLL:
    """Load libs2s.so, declaring every prototype. Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise FileNotFoundError(
            f"{LIB_PATH} is missing: build it with `python swin2sr-rs_b200/build.py` "
            f"(there is no CPU fallback for the forward pass)")
    L = ctypes.CDLL(str(LIB_PATH))
    fp = ctypes.POINTER(ctypes.c_float)
    vp = ctypes.c_void_p
    L.s2s_create.argtypes = [ctypes.POINTER(S2SConfig), ctypes.POINTER(S2STensor), ctypes.c_int,
                             ctypes.c_int, ctypes.POINTER(vp)]
    L.s2s_create.restype = ctypes.c_int
    L.s2s_forward.argtypes = [vp, ctypes.c_int, ctypes.c_int, fp, fp, fp]
    L.s2s_forward.restype = ctypes.c_int
    L.s2s_forward_batch.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp, fp, fp]
    L.s2s_forward_batch.restype = ctypes.c_int
    L.s2s_forward_device.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp]
    L.s2s_forward_device.restype = ctypes.c_int
    L.s2s_aux_dims.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_int)]
    L.s2s_aux_dims.restype = ctypes.c_int
    L.s2s_uploaded_bytes.argtypes = [vp]
    L.s2s_uploaded_bytes.restype = ctypes.c_int64
    L.s2s_workspace_bytes.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.s2s_workspace_bytes.restype = ctypes.c_int64
    L.s2s_last_error.argtypes = [vp]
    L.s2s_last_error.restype = ctypes.c_char_p
    L.s2s_profile_enable.argtypes = [vp, ctypes.c_int, ctypes.c_char_p]
    L.s2s_profile_enable.restype = ctypes.c_int
    L.s2s_profile_report.argtypes = [vp, ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
    L.s2s_profile_report.restype = ctypes.c_int
    L.s2s_launch_count.argtypes = [vp]
    L.s2s_launch_count.restype = ctypes.c_int64
    L.s2s_destroy.argtypes = [vp]
    L.s2s_destroy.restype = None
    L.s2s_debug_stop_after.argtypes = [vp, ctypes.c_int64]
    L.s2s_debug_stop_after.restype = ctypes.c_int
    L.s2s_debug_read.argtypes = [vp, ctypes.c_char_p, fp, ctypes.c_int64]
    L.s2s_debug_read.restype = ctypes.c_int64
    L.s2s_debug_halo_loopback.argtypes = [vp, ctypes.c_int, ctypes.c_int]
    L.s2s_debug_halo_loopback.restype = ctypes.c_int
    L.s2s_window_attention_noalloc.argtypes = [vp] + [ctypes.c_int] * 5 + [vp, vp, ctypes.c_int,
                                                                          vp]
    L.s2s_window_attention_noalloc.restype = ctypes.c_int
    ip = ctypes.POINTER(ctypes.c_int)
    L.s2s_band_unique_id.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.s2s_band_unique_id.restype = ctypes.c_int
    L.s2s_band_init.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    L.s2s_band_init.restype = ctypes.c_int
    L.s2s_band_init_local.argtypes = [ctypes.POINTER(vp), ctypes.c_int]
    L.s2s_band_init_local.restype = ctypes.c_int
    L.s2s_band_rows.argtypes = [vp, ctypes.c_int, ip, ip]
    L.s2s_band_rows.restype = ctypes.c_int
    L.s2s_forward_band.argtypes = [vp, ctypes.c_int, ctypes.c_int, vp, vp, vp]
    L.s2s_forward_band.restype = ctypes.c_int
    L.s2s_forward_band_host.argtypes = [vp, ctypes.c_int, ctypes.c_int, fp, fp]
    L.s2s_forward_band_host.restype = ctypes.c_int
    L.s2s_band_partition.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ip, ip]
    L.s2s_band_partition.restype = ctypes.c_int
    L.s2s_band_halo_ops.argtypes = [ctypes.c_int] * 5 + [ip, ctypes.c_int]
    L.s2s_band_halo_ops.restype = ctypes.c_int
    sz = ctypes.c_size_t
    u8p = ctypes.POINTER(ctypes.c_uint8)
    L.s2s_png_header.argtypes = [ctypes.c_char_p, sz, ip, ip, ip, ip]
    L.s2s_png_header.restype = ctypes.c_int
    L.s2s_png_decode.argtypes = [ctypes.c_char_p, sz, vp, sz]
    L.s2s_png_decode.restype = ctypes.c_int
    for f in (L.s2s_png_encode_rgb8, L.s2s_png_encode_rows):
        f.argtypes = [ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, ctypes.c_int,
                      ctypes.POINTER(u8p), ctypes.POINTER(sz)]
        f.restype = ctypes.c_int
    L.s2s_free.argtypes = [vp]
    L.s2s_free.restype = None
    L.s2s_adjust_device.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int,
                                    ctypes.c_int, vp, vp]
    L.s2s_adjust_device.restype = ctypes.c_int
    L.s2s_rgb8_device.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, vp, vp]
    L.s2s_rgb8_device.restype = ctypes.c_int
    L.s2s_forward_image.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, vp, vp]
    L.s2s_forward_image.restype = ctypes.c_int
    L.s2s_selftest.argtypes = [ctypes.POINTER(S2SConfig), ctypes.POINTER(S2STensor), ctypes.c_int,
                               ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    L.s2s_selftest.restype = ctypes.c_int
    L.s2s_version.argtypes = []
    L.s2s_version.restype = ctypes.c_char_p
    _lib = L
    return L


def _fp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def config_of(wt) -> S2SConfig:
    cfg = S2SConfig()
    cfg.upsampler = UPSAMPLER_CODE[wt.upsampler]
    cfg.scale, cfg.window, cfg.embed = wt.scale, wt.window, wt.embed
    cfg.heads, cfg.mlp_ratio, cfg.n_depths = wt.heads, wt.mlp_ratio, len(wt.depths)
    for i, d in enumerate(wt.depths):
        cfg.depths[i] = d
    cfg.img_range = wt.img_range
    for i in range(3):
        cfg.mean[i] = wt.mean[i]
    return cfg


def tensor_array(wt):
    """The s2s_tensor array of every tensor the architecture needs, and the numpy
    buffers it borrows (keep them alive for the call)."""
    names = wt.needed()
    arr = (S2STensor * len(names))()
    keep = []
    for i, n in enumerate(names):
        a = np.ascontiguousarray(wt.t(n), dtype=np.float32)
        keep.append((n.encode(), a))
        arr[i].name = keep[-1][0]
        arr[i].data = _fp(a)
        arr[i].ndim = a.ndim
        for d in range(min(a.ndim, 4)):
            arr[i].shape[d] = a.shape[d]
    return arr, len(names), keep


def selftest(wt, device: int = 0):
    """s2s_selftest: (status, report) of the fast-path consistency checks."""
    L = load()
    arr, n, keep = tensor_array(wt)
    buf = ctypes.create_string_buffer(4096)
    rc = L.s2s_selftest(ctypes.byref(config_of(wt)), arr, n, device, buf, len(buf))
    del keep
    return rc, buf.value.decode()


class Handle:
    """One s2s_handle on one device."""

    def __init__(self, wt, device: int = 0):
        L = load()
        self.L, self.wt, self.device = L, wt, device
        arr, n, keep = tensor_array(wt)
        h = ctypes.c_void_p()
        rc = L.s2s_create(ctypes.byref(config_of(wt)), arr, n, device, ctypes.byref(h))
        if rc != S2S_OK:
            raise S2SError(rc, L.s2s_last_error(None).decode())
        self.h = h

    def _check(self, rc):
        if rc != S2S_OK:
            raise S2SError(rc, self.L.s2s_last_error(self.h).decode())

    def close(self):
        if getattr(self, "h", None):
            self.L.s2s_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def aux_dims(self, h: int, w: int):
        ah, aw = ctypes.c_int(), ctypes.c_int()
        self._check(self.L.s2s_aux_dims(self.h, h, w, ctypes.byref(ah), ctypes.byref(aw)))
        return ah.value, aw.value

    def forward_batch(self, x: np.ndarray, out: np.ndarray | None = None,
                      aux: np.ndarray | None = None):
        """[B][3][h][w] mean-adjusted -> ([B][3][h*s][w*s], aux [B][3][hp][wp] or None).
        `out` / `aux` may be caller buffers (page-locked ones are written directly)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        B, _, h, w = x.shape
        s, win = self.wt.scale, self.wt.window
        if out is None:
            out = np.empty((B, 3, h * s, w * s), np.float32)
        assert out.shape == (B, 3, h * s, w * s) and out.dtype == np.float32
        assert out.flags.c_contiguous
        if self.wt.upsampler == "pixelshuffle_aux":
            if aux is None:
                aux = np.empty((B, 3, (h // win + 1) * win, (w // win + 1) * win), np.float32)
        else:
            aux = None
        self._check(self.L.s2s_forward_batch(self.h, B, h, w, _fp(x), _fp(out),
                                             _fp(aux) if aux is not None else None))
        return out, aux

    def forward_device(self, B, h, w, d_in: int, d_out: int, d_aux: int = 0, stream: int = 0):
        self._check(self.L.s2s_forward_device(self.h, B, h, w, ctypes.c_void_p(d_in),
                                              ctypes.c_void_p(d_out), ctypes.c_void_p(d_aux or None),
                                              ctypes.c_void_p(stream or None)))

    def uploaded_bytes(self) -> int:
        return int(self.L.s2s_uploaded_bytes(self.h))

    def workspace_bytes(self, B, h, w) -> int:
        return int(self.L.s2s_workspace_bytes(self.h, B, h, w))

    def profile(self, on: bool = True, only: str | None = None):
        self._check(self.L.s2s_profile_enable(self.h, 1 if on else 0,
                                              only.encode() if only else None))

    def profile_report(self, reset: bool = True) -> dict:
        n = self.L.s2s_profile_report(self.h, None, 0, 0)
        buf = ctypes.create_string_buffer(max(n, 1))
        self.L.s2s_profile_report(self.h, buf, n, 1 if reset else 0)
        out = {}
        for line in buf.value.decode().splitlines():
            name, cnt, ms = line.split()
            out[name] = (int(cnt), float(ms))
        return out

    def debug_stop_after(self, launches: int):
        self._check(self.L.s2s_debug_stop_after(self.h, int(launches)))

    def debug_halo_loopback(self, rows: int, missing: bool = False) -> None:
        """One-GPU check of the peer-store halo kernel (s2s_debug_halo_loopback)."""
        self._check(self.L.s2s_debug_halo_loopback(self.h, int(rows), int(bool(missing))))

    def debug_read(self, name: str) -> np.ndarray:
        n = self.L.s2s_debug_read(self.h, name.encode(), None, 0)
        if n < 0:
            raise KeyError(name)
        out = np.empty(n, np.float32)
        self.L.s2s_debug_read(self.h, name.encode(), _fp(out), n)
        return out

    def window_attention_noalloc(self, stage: int, block: int, B: int, hp: int, wp: int,
                                 d_qkv: int, d_out: int, ld_out: int, stream: int = 0):
        """s2s_window_attention_noalloc on device pointers (enqueued, not synchronised)."""
        self._check(self.L.s2s_window_attention_noalloc(
            self.h, stage, block, B, hp, wp, ctypes.c_void_p(d_qkv), ctypes.c_void_p(d_out),
            ld_out, ctypes.c_void_p(stream or None)))

    # ---- row-band sharding
    def band_init(self, rank: int, world: int, uid: bytes | None = None):
        self._check(self.L.s2s_band_init(self.h, rank, world, uid, len(uid) if uid else 0))

    def band_rows(self, height: int):
        r0, r1 = ctypes.c_int(), ctypes.c_int()
        self._check(self.L.s2s_band_rows(self.h, height, ctypes.byref(r0), ctypes.byref(r1)))
        return r0.value, r1.value

    def forward_band(self, x_chw: np.ndarray) -> np.ndarray:
        """This rank's output rows of one [3][h][w] image (synchronous, host buffers)."""
        x = np.ascontiguousarray(x_chw, dtype=np.float32)
        _, h, w = x.shape
        r0, r1 = self.band_rows(h)
        s = self.wt.scale
        out = np.empty((3, (r1 - r0) * s, w * s), np.float32)
        self._check(self.L.s2s_forward_band_host(self.h, h, w, _fp(x), _fp(out)))
        return out

    def forward_band_device(self, h: int, w: int, d_in: int, d_out: int, stream: int = 0):
        self._check(self.L.s2s_forward_band(self.h, h, w, ctypes.c_void_p(d_in),
                                            ctypes.c_void_p(d_out), ctypes.c_void_p(stream or None)))

    def launch_count(self) -> int:
        return int(self.L.s2s_launch_count(self.h))

    # ---- the image path (PNG samples in, 8-bit RGB out)
    def forward_image(self, samples: np.ndarray, bit_depth: int = 8, png_rows: bool = False):
        """s2s_forward_image. `samples` [B][h][w][channels] uint8 (8-bit) or
        [B][h][w][channels * 2] uint8 (16-bit, big-endian pairs), as png_decode returns
        them. Returns (out, aux): to_rgb8 bytes [B][h*s][w*s][3] (PNG scanlines
        [B][h*s][1 + 3*w*s] with png_rows) and the aux plane likewise, or None."""
        x = np.ascontiguousarray(samples, dtype=np.uint8)
        B, h, w, cb = x.shape
        ch = cb // (bit_depth // 8)
        s, win = self.wt.scale, self.wt.window
        H, W = h * s, w * s
        out = np.empty((B, H, 1 + 3 * W) if png_rows else (B, H, W, 3), np.uint8)
        aux = None
        if self.wt.upsampler == "pixelshuffle_aux":
            hp, wp = (h // win + 1) * win, (w // win + 1) * win
            aux = np.empty((B, hp, 1 + 3 * wp) if png_rows else (B, hp, wp, 3), np.uint8)
        self._check(self.L.s2s_forward_image(
            self.h, B, h, w, x.ctypes.data, ch, bit_depth, int(png_rows), out.ctypes.data,
            aux.ctypes.data if aux is not None else None))
        return out, aux

    def adjust_device(self, B, h, w, d_samples: int, channels: int, bit_depth: int, d_chw: int,
                      stream: int = 0):
        """s2s_adjust_device on device pointers (enqueued, not synchronised)."""
        self._check(self.L.s2s_adjust_device(self.h, B, h, w, ctypes.c_void_p(d_samples), channels,
                                             bit_depth, ctypes.c_void_p(d_chw),
                                             ctypes.c_void_p(stream or None)))


def band_unique_id() -> bytes:
    """s2s_band_unique_id: the NCCL id one rank makes and hands to the others."""
    L = load()
    buf = ctypes.create_string_buffer(BAND_ID_BYTES)
    rc = L.s2s_band_unique_id(buf, BAND_ID_BYTES)
    if rc != S2S_OK:
        raise S2SError(rc, L.s2s_last_error(None).decode())
    return buf.raw


def band_init_local(handles) -> None:
    """s2s_band_init_local: `handles` become the bands of one in-process group."""
    L = load()
    arr = (ctypes.c_void_p * len(handles))(*[h.h.value for h in handles])
    rc = L.s2s_band_init_local(arr, len(handles))
    if rc != S2S_OK:
        raise S2SError(rc, handles[0].L.s2s_last_error(handles[0].h).decode())


def band_partition(window_rows: int, world: int, rank: int):
    L = load()
    a, b = ctypes.c_int(), ctypes.c_int()
    rc = L.s2s_band_partition(window_rows, world, rank, ctypes.byref(a), ctypes.byref(b))
    if rc != S2S_OK:
        raise S2SError(rc, "bad band partition arguments")
    return a.value, b.value


def band_halo_ops(rank: int, world: int, own_rows: int, rows: int, cyclic: bool):
    """The transfers of one halo exchange: [(kind, peer, first local row, rows)]."""
    L = load()
    buf = (ctypes.c_int * 16)()
    k = L.s2s_band_halo_ops(rank, world, own_rows, rows, int(cyclic), buf, 16)
    if k < 0:
        raise S2SError(S2S_ERR_INVALID, "bad halo arguments")
    return [tuple(buf[4 * i:4 * i + 4]) for i in range(k)]


# ---- PNG codec and device quantisation (handle-less)
def _fail(L, rc):
    if rc != S2S_OK:
        raise S2SError(rc, L.s2s_last_error(None).decode())


def png_header(data: bytes):
    """(width, height, channels, bit_depth) of a PNG image load_rgb accepts."""
    L = load()
    w, h, c, d = (ctypes.c_int() for _ in range(4))
    _fail(L, L.s2s_png_header(data, len(data), ctypes.byref(w), ctypes.byref(h), ctypes.byref(c),
                              ctypes.byref(d)))
    return w.value, h.value, c.value, d.value


def png_decode(data: bytes):
    """Decoded samples [h][w][channels * bit_depth / 8] uint8 and the bit depth."""
    L = load()
    w, h, c, d = png_header(data)
    out = np.empty((h, w, c * (d // 8)), np.uint8)
    _fail(L, L.s2s_png_decode(data, len(data), out.ctypes.data, out.nbytes))
    return out, d


def _encode(fn, w, h, buf, level, threads) -> bytes:
    L = load()
    p = ctypes.POINTER(ctypes.c_uint8)()
    n = ctypes.c_size_t()
    _fail(L, fn(w, h, buf.ctypes.data, level, threads, ctypes.byref(p), ctypes.byref(n)))
    try:
        return ctypes.string_at(p, n.value)
    finally:
        L.s2s_free(p)


def png_encode_rgb8(rgb: np.ndarray, level: int = -1, threads: int = 0) -> bytes:
    """An 8-bit RGB PNG of `rgb` [h][w][3] uint8 (image::save_rgb)."""
    x = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w, c = x.shape
    if c != 3:
        raise ValueError("png_encode_rgb8 takes [h][w][3] bytes")
    return _encode(load().s2s_png_encode_rgb8, w, h, x, level, threads)


def png_encode_rows(rows: np.ndarray, level: int = -1, threads: int = 0) -> bytes:
    """An 8-bit RGB PNG around filtered scanlines [h][1 + 3w] (forward_image png_rows)."""
    x = np.ascontiguousarray(rows, dtype=np.uint8)
    h, L1 = x.shape
    if (L1 - 1) % 3:
        raise ValueError("scanlines must be 1 + 3 * width bytes")
    return _encode(load().s2s_png_encode_rows, (L1 - 1) // 3, h, x, level, threads)


def rgb8_device(B: int, h: int, w: int, d_chw: int, d_out: int, png_rows: bool = False,
                stream: int = 0) -> None:
    """s2s_rgb8_device on device pointers (enqueued, not synchronised)."""
    L = load()
    _fail(L, L.s2s_rgb8_device(B, h, w, ctypes.c_void_p(d_chw), int(png_rows),
                               ctypes.c_void_p(d_out), ctypes.c_void_p(stream or None)))
