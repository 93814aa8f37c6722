"""Geometry of one forward pass (src/plan.rs restated).

* ``Plan.new`` pads to the NEXT window multiple, ``(n // win + 1) * win`` - an exact
  multiple still gains a whole window (src/plan.rs:39-47).
* ``Plan.index`` is the image coordinate a window token reads on a block shifted by
  ``shift``: ``((wh*win + i + shift) % hp, (ww*win + j + shift) % wp)``
  (src/plan.rs:72-78).
* ``Plan.region`` is the shift-mask region, taken on the ROLLED, unwrapped
  coordinate (src/plan.rs:84-108).
* ``pad_reflect`` mirrors the whole plane, rows first then columns
  (src/plan.rs:116-139).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Plan:
    h: int
    w: int
    hp: int
    wp: int
    win: int
    nwh: int
    nww: int
    nw: int
    n: int
    c: int

    @staticmethod
    def new(h: int, w: int, win: int, c: int) -> "Plan":
        hp = (h // win + 1) * win
        wp = (w // win + 1) * win
        nwh, nww = hp // win, wp // win
        return Plan(h, w, hp, wp, win, nwh, nww, nwh * nww, win * win, c)

    def tokens(self) -> int:
        return self.nw * self.n

    def plane(self) -> int:
        return self.hp * self.wp

    def shift_for(self, b: int) -> int:
        return self.win // 2 if b % 2 == 1 else 0

    def index(self, wi: int, t: int, shift: int):
        wh, ww = divmod(wi, self.nww)
        i, j = divmod(t, self.win)
        return (wh * self.win + i + shift) % self.hp, (ww * self.win + j + shift) % self.wp

    def region(self, wi: int, t: int, shift: int):
        wh, ww = divmod(wi, self.nww)
        i, j = divmod(t, self.win)
        return (region_of(wh * self.win + i, self.hp, self.win, shift),
                region_of(ww * self.win + j, self.wp, self.win, shift))

    def token_pixels(self, shift: int) -> np.ndarray:
        """Flat pixel index ``y*wp + x`` read by every window-major token, vectorised."""
        wi = np.arange(self.nw)[:, None]
        t = np.arange(self.n)[None, :]
        wh, ww = wi // self.nww, wi % self.nww
        i, j = t // self.win, t % self.win
        y = (wh * self.win + i + shift) % self.hp
        x = (ww * self.win + j + shift) % self.wp
        return (y * self.wp + x).reshape(-1)


def region_of(a: int, p: int, win: int, shift: int) -> int:
    """The reference's h_slices: [0, -win), [-win, -shift), [-shift, None)."""
    if a + win < p:
        return 0
    if a + shift < p:
        return 1
    return 2


def pad_reflect(x: np.ndarray, h: int, w: int, hp: int, wp: int) -> np.ndarray:
    """[c][h][w] -> [c][hp][wp] by whole-plane mirroring, rows then columns."""
    sy = np.array([y if y < h else 2 * h - 1 - min(y, 2 * h - 1) for y in range(hp)])
    sx = np.array([v if v < w else 2 * w - 1 - min(v, 2 * w - 1) for v in range(wp)])
    return np.ascontiguousarray(x[:, sy, :][:, :, sx])


def check_size(h: int, w: int, win: int) -> None:
    """The reference refuses images smaller than one window (src/backend.rs:60-71)."""
    if h < win or w < win:
        raise ValueError(
            f"{h}x{w} is smaller than one {win}x{win} window. The reference pads to the NEXT "
            f"window multiple by concatenating the image with its own mirror, which for an image "
            f"shorter than a window truncates the pad and then falls through to a second, "
            f"different padding rule this engine does not implement.")
