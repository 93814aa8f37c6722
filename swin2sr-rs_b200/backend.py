"""The reference's host interface for the forward pass (src/backend.rs restated).

* ``Backend``   - the trait (src/backend.rs:29-49): ``name``, ``forward(h, w, input)``,
                  ``aux()``.
* ``Pre``       - the window check and the mean adjustment (src/backend.rs:53-87).
* ``run_tiled`` - the tile loop that calls ``forward`` (src/backend.rs:92-164).
* ``crop_side``, ``auto_tile`` - the tile the memory budget allows
                  (src/backend.rs:168-259), from the library's exact workspace size.
* ``run_with_fallback`` - halve the tile and retry when the device runs out of
                  memory (src/main.rs:579-662).
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

    @classmethod
    def from_handle(cls, handle):
        """A backend over an existing handle (its weights are not uploaded again)."""
        g = cls.__new__(cls)
        g.wt, g.handle, g._aux = handle.wt, handle, None
        return g

    def name(self) -> str:
        return "cuda"  # src/gpu.rs:737-739; --verify prints it (src/main.rs:692)

    def forward(self, h: int, w: int, inp: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(inp, dtype=np.float32).reshape(1, 3, h, w)
        out, aux = self.handle.forward_batch(x)
        self._aux = aux[0] if aux is not None else None
        return out[0]

    def forward_batch(self, x: np.ndarray):
        return self.handle.forward_batch(x)

    def forward_image(self, samples: np.ndarray, bit_depth: int = 8, png_rows: bool = False):
        """The CLI's image path on the device (src/main.rs:205-378 without the file
        IO): decoded PNG samples [B][h][w][c] -> to_rgb8 bytes [B][h*s][w*s][3] (or
        PNG scanlines with png_rows), plus the aux plane for pixelshuffle_aux."""
        out, aux = self.handle.forward_image(samples, bit_depth, png_rows)
        self._aux = None
        return out, aux

    def aux(self):
        return self._aux

    def workspace_bytes(self, h: int, w: int) -> int:
        """Device bytes a forward of one h x w image allocates (s2s_workspace_bytes)."""
        return self.handle.workspace_bytes(1, h, w)

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


def crop_side(h: int, w: int, tile: int, pad: int, win: int) -> int:
    """src/backend.rs:249-259: the padded plane, in pixels a side, that a crop of
    `tile` pixels plus `pad` of context runs on (tile 0 = the whole image)."""
    if tile == 0:
        th, tw = h, w
    else:
        t = max(tile // win, 1) * win
        p = max(-(-pad // win), 1) * win
        th, tw = min(t + 2 * p, h), min(t + 2 * p, w)
    plane = lambda n: (n // win + 1) * win  # noqa: E731
    return max(plane(th), plane(tw))


def auto_tile(wt, backend, budget: int, h: int, w: int, pad: int) -> int:
    """src/backend.rs:168-187: 0 when the whole image fits `budget` bytes of
    activations, else the largest window-multiple tile (from 1024, halving) whose
    crop fits. The size of a crop comes from the backend's own exact workspace
    figure (s2s_workspace_bytes) rather than a per-pixel estimate; the device
    kernels have no launch-size ceiling to check besides it."""
    win = wt.window
    pad = max(-(-pad // win), 1) * win
    whole = crop_side(h, w, 0, pad, win)
    # crop_side reports the padded plane; the workspace is asked for the crop itself
    if backend.workspace_bytes(whole - win, whole - win) <= budget:
        return 0
    t = (max(1024, win) // win) * win
    while True:
        side = crop_side(h, w, t, pad, win)
        if backend.workspace_bytes(side - win, side - win) <= budget or t == win:
            return t
        t = max(t // 2 // win, 1) * win


def is_out_of_memory(err: Exception) -> bool:
    """src/main.rs:660-662: the one failure a smaller tile can fix."""
    msg = str(err)
    return "OUT_OF_MEMORY" in msg or "out of memory" in msg


def run_with_fallback(wt, backend: Backend, img: np.ndarray, tile: int, pad: int,
                      note=None, note_exact=None):
    """src/main.rs:579-657: run_tiled, halving the tile on out-of-memory (a failed
    whole-image pass falls back to half the image), down to one window.
    Returns (image, the tile that ran). `note` receives each retry's message; a retry
    out of the whole-image pass (tile 0, the only exact mode) goes to `note_exact`
    instead when given, since the reference announces that one even under -q
    (src/main.rs:627-640)."""
    for _ in range(64):
        try:
            return run_tiled(wt, backend, img, tile, pad), tile
        except Exception as e:  # noqa: BLE001 - only out-of-memory is retried
            if not (is_out_of_memory(e) and (tile > wt.window or tile == 0)):
                raise
            _, ih, iw = img.shape
            if tile == 0:
                nxt = max(max(ih, iw) // 2 // wt.window, 1) * wt.window
            else:
                nxt = max(tile // 2 // wt.window, 1) * wt.window
            shrinking = nxt != 0 if tile == 0 else nxt < tile
            if not shrinking or nxt == 0:
                raise RuntimeError(f"{e}\n(a {wt.window}-pixel tile is the smallest this engine "
                                   f"will run, and it did not fit either)") from e
            if tile == 0:
                msg = (f"{str(e).rstrip('.')} - retrying with a {nxt}x{nxt} tile (--tile 0 is "
                       f"the only exact mode; this run is now tiled, and tiled results differ "
                       f"slightly from one pass)")
                sink = note_exact or note
            else:
                msg = f"{str(e).rstrip('.')} - retrying with a {nxt}x{nxt} tile"
                sink = note
            if sink:
                sink(msg)
            tile = nxt
    raise RuntimeError(f"gave up after 64 tile reductions at tile {tile}")
