#!/usr/bin/env python3
"""Generate the golden fixtures that pin the oracle to the published network.

The reference holds both of its backends to the published PyTorch Swin2SR
(``tools/network_swin2sr.py``, run by ``tools/make_fixture.py``). This script does
the same with seeded weights, because the released checkpoints are not available:

1. build the seeded raw state dict (``weights.seeded_state_dict``), load it into the
   reference's own ``Swin2SR`` module, and run it on a seeded input padded exactly
   as ``tools/make_fixture.py:80-89`` pads;
2. write an ``SW2F`` fixture (``src/fixture.rs:1-99`` format: 36-byte header, input
   [3][h][w], expected [3][h*s][w*s], and for the compressed head the aux plane
   [3][hp][wp]).

Only inputs and outputs are committed; the weights are regenerated from the seed
by ``weights.py`` wherever the fixture is checked. Run in a container that has the
reference checkout (it needs ``network_swin2sr.py`` + ``timm_shim.py``):

    python tests/golden/make_golden.py --ref /path/to/swin2sr-rs
"""
import argparse
import hashlib
import importlib.util
import struct
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
HERE = Path(__file__).resolve().parent


def _load_pkg():
    spec = importlib.util.spec_from_file_location(
        "swin2sr_b200", ROOT / "swin2sr-rs_b200" / "__init__.py",
        submodule_search_locations=[str(ROOT / "swin2sr-rs_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["swin2sr_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


# (name, task, weight seed, perturb, h, w, input seed)
CASES = [
    ("lw_seed0_64x64", "lightweight_sr", 0, False, 64, 64, 1),
    ("lw_perturb_37x29", "lightweight_sr", 0, True, 37, 29, 2),
    ("c2_perturb_20x27", "classical_sr_x2", 0, True, 20, 27, 3),
    ("c4_perturb_21x26", "classical_sr", 0, True, 21, 26, 4),
    ("rw_perturb_18x23", "real_sr", 0, True, 18, 23, 5),
    ("cx_perturb_17x22", "compressed_sr", 0, True, 17, 22, 6),
]

ARCH = {  # tools/make_fixture.py:39-48 plus the classical x2 task
    "classical_sr": dict(depths=[6] * 6, embed_dim=180, num_heads=[6] * 6, upsampler="pixelshuffle"),
    "classical_sr_x2": dict(depths=[6] * 6, embed_dim=180, num_heads=[6] * 6, upsampler="pixelshuffle"),
    "compressed_sr": dict(depths=[6] * 6, embed_dim=180, num_heads=[6] * 6, upsampler="pixelshuffle_aux"),
    "real_sr": dict(depths=[6] * 6, embed_dim=180, num_heads=[6] * 6, upsampler="nearest+conv"),
    "lightweight_sr": dict(depths=[6] * 4, embed_dim=60, num_heads=[6] * 4, upsampler="pixelshuffledirect"),
}


def pad_like_reference(x, ws):
    _, _, h, w = x.size()
    hp = (h // ws + 1) * ws - h
    wp = (w // ws + 1) * ws - w
    x = torch.cat([x, torch.flip(x, [2])], 2)[:, :, :h + hp, :]
    x = torch.cat([x, torch.flip(x, [3])], 3)[:, :, :, :w + wp]
    return x


def write_sw2f(path, h, w, scale, win, x, y, aux):
    flags = 1 if aux is not None else 0
    with open(path, "wb") as f:
        f.write(b"SW2F")
        f.write(struct.pack("<IIIIIIII", 1, h, w, 3, scale, win, flags, 0))
        f.write(np.ascontiguousarray(x, "<f4").tobytes())
        f.write(np.ascontiguousarray(y, "<f4").tobytes())
        if aux is not None:
            f.write(np.ascontiguousarray(aux, "<f4").tobytes())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True,
                    help="checkout of the swin2sr-rs reference (its tools/network_swin2sr.py)")
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref) / "tools"))
    from network_swin2sr import Swin2SR  # noqa: E402  (the reference's published network)

    pkg = _load_pkg()
    W = pkg.weights
    torch.set_num_threads(max(1, torch.get_num_threads()))
    lines = []
    for name, task, wseed, perturb, h, w, iseed in CASES:
        if args.only and args.only != name:
            continue
        cfg = W.CONFIGS[task]
        arch = ARCH[task]
        net = Swin2SR(upscale=cfg["scale"], in_chans=3, img_size=64, window_size=cfg["win"],
                      img_range=1.0, depths=arch["depths"], embed_dim=arch["embed_dim"],
                      num_heads=arch["num_heads"], mlp_ratio=cfg["mlp_ratio"],
                      upsampler=arch["upsampler"], resi_connection="1conv")
        sd = W.seeded_state_dict(task, wseed, perturb)
        ts = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()}
        missing, unexpected = net.load_state_dict(ts, strict=False)
        missing = [k for k in missing if not k.endswith("attn_mask")]
        if missing or unexpected:
            raise SystemExit(f"{name}: state dict mismatch: missing {missing[:4]} "
                             f"unexpected {unexpected[:4]}")
        net.eval()
        g = torch.Generator().manual_seed(iseed)
        x = torch.rand(1, 3, h, w, generator=g)
        xp = pad_like_reference(x, cfg["win"])
        with torch.no_grad():
            y = net(xp)
        aux = None
        if isinstance(y, tuple):
            y, aux = y[0], y[1]
        s = cfg["scale"]
        y = y[0, :, :h * s, :w * s].contiguous().numpy()
        aux = aux[0].contiguous().numpy() if aux is not None else None
        path = HERE / f"{name}.sw2f"
        write_sw2f(path, h, w, s, cfg["win"], x[0].numpy(), y, aux)
        digest = hashlib.sha256(path.read_bytes()).hexdigest()[:16]
        line = (f"{name}: task={task} wseed={wseed} perturb={perturb} {h}x{w} iseed={iseed} "
                f"out range [{y.min():.4f}, {y.max():.4f}] sha256:{digest}")
        print(line)
        lines.append(line)
    if not args.only:
        (HERE / "MANIFEST.txt").write_text(
            "# written by make_golden.py from the reference's tools/network_swin2sr.py\n"
            + "\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
