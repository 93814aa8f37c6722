"""Shared helpers for the test suite: package loading, SW2F fixtures, comparisons."""
from __future__ import annotations

import importlib.util
import re
import struct
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
TOL = 2e-3  # max-abs on the [0,1] output (north_star; the reference's tests/parity.rs:33)


def pkg():
    """The swin2sr-rs_b200 package (its directory name is not an identifier)."""
    if "swin2sr_b200" in sys.modules:
        return sys.modules["swin2sr_b200"]
    spec = importlib.util.spec_from_file_location(
        "swin2sr_b200", ROOT / "swin2sr-rs_b200" / "__init__.py",
        submodule_search_locations=[str(ROOT / "swin2sr-rs_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["swin2sr_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def oracle():
    if str(ROOT) not in sys.path:
        sys.path.insert(0, str(ROOT))
    from oracle import oracle as O
    return O


def golden_cases():
    lines = (GOLDEN / "MANIFEST.txt").read_text().splitlines()
    out = []
    for line in lines:
        if not line or line.startswith("#"):
            continue
        name = line.split(":")[0]
        out.append(dict(name=name, task=re.search(r"task=(\S+)", line).group(1),
                        wseed=int(re.search(r"wseed=(\d+)", line).group(1)),
                        perturb="perturb=True" in line))
    return out


def load_fixture(name: str):
    """SW2F (src/fixture.rs:52-99): (h, w, scale, win, input, expected, aux|None)."""
    b = (GOLDEN / f"{name}.sw2f").read_bytes()
    assert b[:4] == b"SW2F"
    ver, h, w, c, s, win, flags, _ = struct.unpack("<8I", b[4:36])
    assert ver == 1 and c == 3
    n_in, n_out = 3 * h * w, 3 * h * s * w * s
    x = np.frombuffer(b, "<f4", n_in, 36).reshape(3, h, w).copy()
    y = np.frombuffer(b, "<f4", n_out, 36 + 4 * n_in).reshape(3, h * s, w * s).copy()
    aux = None
    if flags & 1:
        hp, wp = (h // win + 1) * win, (w // win + 1) * win
        aux = np.frombuffer(b, "<f4", 3 * hp * wp, 36 + 4 * (n_in + n_out)).reshape(3, hp, wp).copy()
    return h, w, s, win, x, y, aux


def adjust(wt, x):
    m = np.asarray(wt.mean, np.float32).reshape(3, 1, 1)
    return ((x - m) * np.float32(wt.img_range)).astype(np.float32)


def parity_report(got, want):
    """max-abs raw, max-abs after clamping to [0,1], and the fraction of 8-bit values
    more than one level apart after the reference's to_rgb8 (src/image.rs:28-39)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    raw = float(np.abs(got - want).max())
    gc, wc = np.clip(got, 0, 1), np.clip(want, 0, 1)
    clamped = float(np.abs(gc - wc).max())
    q = np.abs(np.floor(gc * 255 + 0.5) - np.floor(wc * 255 + 0.5))
    return raw, clamped, float((q > 1).mean())


def block_launches(wt) -> int:
    """Kernel launches per Swin block of a forward, by the library's create-time rules:
    the fused QKV + attention kernel for 6 heads of 32 over Cp = 192 only with
    S2S_ATTN=fused (and single-term operands), two-term operands for Cp = 64 (S2S_SPLIT overrides), the
    fused MLP for (Cp, hidden) = (192, 384) / (64, 128) with single-term operands
    (unless S2S_UNFUSED_MLP), with proj inside it at Cp = 192 (unless
    S2S_UNFUSED_PROJ=1)."""
    import os
    cp = -(-wt.embed // 64) * 64
    hid = -(-wt.embed * wt.mlp_ratio // 64) * 64
    dp = -(-(wt.embed // wt.heads) // 16) * 16
    sw = os.environ.get("S2S_SPLIT")
    split = cp == 64 if sw not in ("0", "1") else sw == "1"
    fused_attn = (not split and cp == 192 and wt.heads == 6 and dp == 32
                  and os.environ.get("S2S_ATTN") == "fused")
    fused_mlp = (not split and (cp, hid) in ((192, 384), (64, 128))
                 and os.environ.get("S2S_UNFUSED_MLP", "0") in ("", "0"))
    fused_proj = fused_mlp and cp == 192 and os.environ.get("S2S_UNFUSED_PROJ") != "1"
    return (1 if fused_attn else 2) + (1 if fused_proj else 1 + (1 if fused_mlp else 2))
