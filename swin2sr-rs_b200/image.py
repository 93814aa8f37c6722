"""PNG IO and the planar float image: the host mirror of swin2sr-rs src/image.rs.

``Image`` is the reference's [3][h][w] f32 image (src/image.rs:11-40);
``load_rgb`` / ``save_rgb`` read and write PNG through the library's codec
(``s2s_png_decode`` / ``s2s_png_encode_*``: zlib inflate, unfilter, Adam7 on the
host; deflate split over host threads). The GPU image path does not go through
``Image`` at all: ``Gpu.forward_image`` takes the decoded samples and returns
8-bit RGB (or PNG scanlines), with the sample scaling, ``Pre::adjust`` and
``to_rgb8`` running on the device.
"""
from __future__ import annotations

import numpy as np

from . import capi


class Image:
    """src/image.rs:11-40: a planar RGB image, ``data`` [3][h][w] f32 in [0,1]."""

    def __init__(self, w: int, h: int, data: np.ndarray | None = None):
        self.w, self.h = w, h
        if data is None:
            data = np.zeros((3, h, w), np.float32)
        self.data = np.ascontiguousarray(data, dtype=np.float32).reshape(3, h, w)

    def plane(self, c: int) -> np.ndarray:
        return self.data[c]

    def to_rgb8(self) -> np.ndarray:
        """src/image.rs:28-39: interleaved [h][w][3] bytes; clamp to [0,1], * 255,
        floor(+0.5), min 255 (NaN -> 255), each step one f32 rounding."""
        c = np.clip(self.data, np.float32(0.0), np.float32(1.0))
        v = np.fmin(np.floor(c * np.float32(255.0) + np.float32(0.5)), np.float32(255.0))
        return np.ascontiguousarray(v.astype(np.uint8).transpose(1, 2, 0))


def samples_to_image(samples: np.ndarray, bit_depth: int) -> Image:
    """src/image.rs:57-95: decoded samples [h][w][channels * bit_depth / 8] -> Image."""
    s = np.asarray(samples, np.uint8)
    h, w, cb = s.shape
    channels = cb // (bit_depth // 8)
    if bit_depth == 16:
        v = ((s[..., 0::2].astype(np.uint32) << 8) | s[..., 1::2]).astype(np.float32)
        v *= np.float32(1.0) / np.float32(65535.0)
    else:
        v = s.astype(np.float32) * (np.float32(1.0) / np.float32(255.0))
    v = v.reshape(h, w, channels)
    idx = [0, 0, 0] if channels < 3 else [0, 1, 2]
    return Image(w, h, np.stack([v[..., i] for i in idx]))


def decode(data: bytes):
    """PNG bytes -> (samples [h][w][channels * bit_depth / 8] uint8, bit_depth)."""
    return capi.png_decode(data)


def load_rgb_stream(src) -> Image:
    """src/image.rs:48-96: decode a PNG from a binary stream."""
    samples, depth = decode(src.read())
    return samples_to_image(samples, depth)


def load_rgb(path: str) -> Image:
    """src/image.rs:42-46."""
    with open(path, "rb") as f:
        try:
            return load_rgb_stream(f)
        except capi.S2SError as e:
            raise capi.S2SError(e.code, f"{path}: {e}") from None


def encode_rgb8(rgb: np.ndarray, level: int = -1, threads: int = 0) -> bytes:
    return capi.png_encode_rgb8(rgb, level, threads)


def save_rgb_stream(dst, w: int, h: int, rgb, level: int = -1, threads: int = 0) -> None:
    """src/image.rs:104-114: 8-bit RGB. `rgb` is w*h*3 bytes, interleaved."""
    a = np.frombuffer(bytes(rgb), np.uint8) if not isinstance(rgb, np.ndarray) else rgb
    if a.size != w * h * 3:
        raise ValueError(f"rgb holds {a.size} bytes, a {w}x{h} RGB image needs {w * h * 3}")
    dst.write(encode_rgb8(a.reshape(h, w, 3), level, threads))


def save_rgb(path: str, w: int, h: int, rgb, level: int = -1, threads: int = 0) -> None:
    """src/image.rs:98-102."""
    with open(path, "wb") as f:
        save_rgb_stream(f, w, h, rgb, level, threads)
