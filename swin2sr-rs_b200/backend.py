"""The reference's host interface for the forward pass (src/backend.rs restated).

* ``Backend``   - the trait (src/backend.rs:29-49): ``name``, ``forward(h, w, input)``,
                  ``aux()``.
* ``Pre``       - the window check and the mean adjustment (src/backend.rs:53-87).
* ``run_tiled`` - the tile loop that calls ``forward`` (src/backend.rs:92-164).
* ``Gpu``       - the B200 backend: ``forward`` goes through the C ABI
                  (include/s2s.h) into the sm_100a kernels. There is no CPU fallback.
"""
from __future__ import annotations

import numpy as np

from . import capi
from .plan import Plan, check_size


class Backend:
    def name(self) -> str:  # pragma: no cover - interface
        raise NotImplementedError

    def forward(self, h: int, w: int, inp: np.ndarray) -> np.ndarray:  # pragma: no cover
        raise NotImplementedError

    def aux(self):
        return None


class Pre:
    """Pad/mean bookkeeping of one image (src/backend.rs:53-87)."""

    def __init__(self, wt, h: int, w: int):
        check_size(h, w, wt.window)
        self.plan = Plan.new(h, w, wt.window, wt.embed)
        self.h, self.w = h, w

    def adjust(self, wt, img: np.ndarray) -> np.ndarray:
        """(x - mean) * img_range, the network's single mean subtraction."""
        out = np.array(img, dtype=np.float32, copy=True).reshape(3, self.h, self.w)
        for c in range(3):
            out[c] = (out[c] - np.float32(wt.mean[c])) * np.float32(wt.img_range)
        return out


class Gpu(Backend):
    """The device backend: one s2s handle, weights uploaded once (src/gpu.rs:101-125)."""

    def __init__(self, wt, device: int = 0):
        self.wt = wt
        self.handle = capi.Handle(wt, device)
        self._aux = None

    def name(self) -> str:
        return "gpu"

    def forward(self, h: int, w: int, inp: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(inp, dtype=np.float32).reshape(1, 3, h, w)
        out, aux = self.handle.forward_batch(x)
        self._aux = aux[0] if aux is not None else None
        return out[0]

    def forward_batch(self, x: np.ndarray):
        return self.handle.forward_batch(x)

    def aux(self):
        return self._aux

    def close(self):
        self.handle.close()


def run_tiled(wt, backend: Backend, img: np.ndarray, tile: int, pad: int) -> np.ndarray:
    """src/backend.rs:92-164: whole image when tile == 0, else tiles with context."""
    _, ih, iw = img.shape
    scale = wt.scale
    if tile == 0:
        pre = Pre(wt, ih, iw)
        return backend.forward(ih, iw, pre.adjust(wt, img))
    win = wt.window
    tile = max(tile // win, 1) * win
    pad = max(-(-pad // win), 1) * win
    out = np.zeros((3, ih * scale, iw * scale), np.float32)
    ty = 0
    while ty < ih:
        tx = 0
        while tx < iw:
            y0, x0 = max(ty - pad, 0), max(tx - pad, 0)
            y1, x1 = min(ty + tile + pad, ih), min(tx + tile + pad, iw)
            th, tw = y1 - y0, x1 - x0
            sub = np.ascontiguousarray(img[:, y0:y1, x0:x1])
            pre = Pre(wt, th, tw)
            res = backend.forward(th, tw, pre.adjust(wt, sub))
            oy0, ox0 = ty - y0, tx - x0
            cw, ch = min(tx + tile, iw) - tx, min(ty + tile, ih) - ty
            out[:, ty * scale:(ty + ch) * scale, tx * scale:(tx + cw) * scale] = \
                res[:, oy0 * scale:(oy0 + ch) * scale, ox0 * scale:(ox0 + cw) * scale]
            tx += tile
        ty += tile
    return out
