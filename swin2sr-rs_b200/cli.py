"""Many PNG files through the device image path, batched and on several GPUs.

    python swin2sr-rs_b200/cli.py -m weights.safetensors -i a.png [b.png ...] -o OUT
        [--devices 0,1,...] [--batch N] [--level L] [--threads T] [--aux OUT]
        [--tile N|auto] [--tile-pad P] [-q]

The reference's CLI (src/main.rs:20-419) runs one image: load_rgb -> Pre::adjust
-> forward -> to_rgb8 -> save_rgb. This driver runs that path for many images:
PNG decode on a host thread pool (s2s_png_decode), same-size images batched into
one s2s_forward_image call (sample scaling, mean adjustment, the network and the
PNG row filter on the device; only bytes cross PCIe), one host thread and one
handle per device (data parallel, no communication), deflate of the filtered
scanlines on the pool (s2s_png_encode_rows). Decode, forward and encode of
different batches overlap. `-o` names a file for one input and a directory for
several; `--aux` likewise, for the compressed_sr head (src/main.rs:380-418).

`--tile` (src/main.rs:450-662) runs each image through the tiled driver instead:
tiles of N pixels with `--tile-pad` of context (rounded up to a window multiple),
halving the tile whenever the device runs out of memory. `auto` starts from one
whole-image pass and relies on that retry. A tiled image takes the float path
(backend.run_with_fallback), quantised and encoded on the host; the second image of
`--aux` exists only for a whole-image pass, as in the reference.
"""
from __future__ import annotations

import argparse
import os
import queue
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor

if __name__ == "__main__" and not __package__:  # run as a script: load the package by path
    import importlib.util
    from pathlib import Path
    _here = Path(__file__).resolve().parent
    _spec = importlib.util.spec_from_file_location(
        "swin2sr_b200", _here / "__init__.py", submodule_search_locations=[str(_here)])
    _mod = importlib.util.module_from_spec(_spec)
    sys.modules["swin2sr_b200"] = _mod
    _spec.loader.exec_module(_mod)
    __package__ = "swin2sr_b200"

from . import capi  # noqa: E402


def plan_batches(headers, batch: int):
    """Group image indices by (height, width, channels, bit depth) in input order and
    cut each group into batches of at most `batch`. `headers[i]` is png_header's
    (width, height, channels, bit_depth)."""
    if batch < 1:
        raise ValueError("batch must be >= 1")
    groups: dict = {}
    for i, hd in enumerate(headers):
        groups.setdefault(tuple(hd), []).append(i)
    out = []
    for key, idx in groups.items():
        for k in range(0, len(idx), batch):
            out.append((key, idx[k:k + batch]))
    return out


def upscale_pngs(handles, pngs, batch: int = 8, level: int = -1, threads: int = 0,
                 want_aux: bool = False, stats: dict | None = None, pad: int = 32,
                 note=None, note_exact=None):
    """PNG bytes in -> PNG bytes out (and aux PNGs, or None each), in input order.

    `handles` are capi.Handle objects, one per device; batches are spread over them.
    `threads` sizes the host pool (0 = all cores). A batch whose whole-image pass runs
    out of device memory is redone image by image through the tiled driver from tile 0
    (run_with_fallback: the whole image alone, then halving tiles with `pad` context),
    as the reference's --tile 0 retries (src/main.rs:579-657); its aux is then None."""
    from . import backend, image
    if not handles:
        raise ValueError("at least one handle")
    wt = handles[0].wt
    T = threads or os.cpu_count() or 1
    n = len(pngs)
    out = [None] * n
    aux = [None] * n
    t0 = time.perf_counter()
    headers = [capi.png_header(p) for p in pngs]
    for w, h, _, _ in headers:
        if h < wt.window or w < wt.window:
            raise ValueError(f"{w}x{h} is smaller than one {wt.window}x{wt.window} window")
    batches = plan_batches(headers, batch)
    pool = ThreadPoolExecutor(max_workers=T)
    try:
        dec_f = {i: pool.submit(capi.png_decode, pngs[i]) for i in range(n)}
        work: queue.Queue = queue.Queue()
        for b in batches:
            work.put(b)
        enc_f = []
        lock = threading.Lock()
        errors = []
        enc_threads = max(1, T // max(1, len(handles) * 2))

        def device_loop(H):
            import numpy as np
            while True:
                try:
                    key, idx = work.get_nowait()
                except queue.Empty:
                    return
                try:
                    _, _, _, depth = key
                    samples = np.stack([dec_f[i].result()[0] for i in idx])
                    try:
                        rows, arows = H.forward_image(samples, depth, png_rows=True)
                    except capi.S2SError as e:
                        if not backend.is_out_of_memory(e):
                            raise
                        gpu = backend.Gpu.from_handle(H)
                        for i in idx:
                            img = image.samples_to_image(dec_f[i].result()[0], depth)
                            res, _ = backend.run_with_fallback(wt, gpu, img.data, 0, pad, note,
                                                               note_exact)
                            rgb = image.Image(img.w * wt.scale, img.h * wt.scale, res).to_rgb8()
                            with lock:
                                enc_f.append((i, False, pool.submit(
                                    capi.png_encode_rgb8, rgb, level, enc_threads)))
                        continue
                    with lock:
                        for k, i in enumerate(idx):
                            enc_f.append((i, False, pool.submit(
                                capi.png_encode_rows, rows[k], level, enc_threads)))
                            if want_aux and arows is not None:
                                enc_f.append((i, True, pool.submit(
                                    capi.png_encode_rows, arows[k], level, enc_threads)))
                except Exception as e:  # noqa: BLE001 - reported after the join
                    errors.append(e)
                    return

        ts = [threading.Thread(target=device_loop, args=(H,)) for H in handles]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        if errors:
            raise errors[0]
        for i, is_aux, f in enc_f:
            (aux if is_aux else out)[i] = f.result()
    finally:
        pool.shutdown(wait=True)
    if stats is not None:
        s = wt.scale
        stats["seconds"] = time.perf_counter() - t0
        stats["images"] = n
        stats["output_mpix"] = sum(h * s * w * s for w, h, _, _ in headers) / 1e6
        stats["batches"] = len(batches)
    return out, aux


def upscale_pngs_tiled(handles, pngs, tile: int, pad: int, level: int = -1, threads: int = 0,
                       note=None, stats: dict | None = None, note_exact=None):
    """PNG bytes in -> PNG bytes out through the tiled driver, images spread over the
    handles (one host thread each). Returns (outputs, the tile each image ran with)."""
    from . import backend, image
    if not handles:
        raise ValueError("at least one handle")
    wt = handles[0].wt
    n = len(pngs)
    out, ran = [None] * n, [None] * n
    t0 = time.perf_counter()
    headers = [capi.png_header(p) for p in pngs]
    errors = []

    def work(k):
        gpu = backend.Gpu.from_handle(handles[k])
        for i in range(k, n, len(handles)):
            try:
                samples, depth = capi.png_decode(pngs[i])
                img = image.samples_to_image(samples, depth)
                res, ran[i] = backend.run_with_fallback(wt, gpu, img.data, tile, pad, note,
                                                        note_exact)
                rgb = image.Image(img.w * wt.scale, img.h * wt.scale, res).to_rgb8()
                out[i] = capi.png_encode_rgb8(rgb, level, threads)
            except Exception as e:  # noqa: BLE001 - reported after the join
                errors.append(e)
                return

    ts = [threading.Thread(target=work, args=(k,)) for k in range(len(handles))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    if errors:
        raise errors[0]
    if stats is not None:
        s = wt.scale
        stats["seconds"] = time.perf_counter() - t0
        stats["images"] = n
        stats["output_mpix"] = sum(h * s * w * s for w, h, _, _ in headers) / 1e6
        stats["batches"] = n
    return out, ran


def main(argv=None) -> int:
    from . import weights as W
    ap = argparse.ArgumentParser(prog="swin2sr-b200", description=__doc__.split("\n\n")[0])
    ap.add_argument("-m", "--model", required=True, help="converted .safetensors checkpoint")
    ap.add_argument("-i", "--input", nargs="+", required=True, help="input PNG files")
    ap.add_argument("-o", "--output", required=True,
                    help="output PNG (one input) or directory (several)")
    ap.add_argument("--aux", help="also write the compressed_sr head's second image "
                                  "(file for one input, directory for several)")
    ap.add_argument("--devices", default="0", help="comma-separated CUDA ordinals")
    ap.add_argument("--batch", type=int, default=8, help="images of one size per forward")
    ap.add_argument("--level", type=int, default=-1, help="zlib level -1..9")
    ap.add_argument("--threads", type=int, default=0, help="host threads (0 = all cores)")
    ap.add_argument("--tile", default="0",
                    help="tile side in pixels, 0 for one whole-image pass (the only exact "
                         "mode), or auto: whole image, halved on out-of-memory")
    ap.add_argument("--tile-pad", type=int, default=32,
                    help="context kept around each tile (rounded up to a window multiple)")
    ap.add_argument("-q", "--quiet", action="store_true")
    a = ap.parse_args(argv)
    if a.tile == "auto":
        tile = 0
    else:
        try:
            tile = int(a.tile)
        except ValueError:
            print("error: --tile takes a number or `auto`", file=sys.stderr)
            return 1
    tiled = a.tile != "0"
    wt = W.Weights.load(a.model)
    if a.aux and tiled:
        print(f"error: --aux: the second image exists only for a single pass, and --tile "
              f"{a.tile} would tile it. Re-run with --tile 0.", file=sys.stderr)
        return 1
    if a.aux and wt.upsampler != "pixelshuffle_aux":
        print(f"error: --aux: the {wt.upsampler} head has one output; only the compressed_sr "
              f"head (pixelshuffle_aux) produces a second image", file=sys.stderr)
        return 1
    several = len(a.input) > 1

    def target(base, path):
        if not several:
            return base
        os.makedirs(base, exist_ok=True)
        return os.path.join(base, os.path.basename(path))

    pngs = []
    for p in a.input:
        with open(p, "rb") as f:
            pngs.append(f.read())
    handles = [capi.Handle(wt, int(d)) for d in a.devices.split(",")]
    try:
        stats: dict = {}
        # retry notes take -q, except a whole-image pass falling back to tiles: that run
        # is no longer the exact one asked for, so it is announced regardless
        say = lambda m: print(f"note: {m}", file=sys.stderr)  # noqa: E731
        note = None if a.quiet else say
        if tiled:
            outs, _ = upscale_pngs_tiled(handles, pngs, tile, a.tile_pad, a.level, a.threads,
                                         note, stats, note_exact=say)
            auxs = [None] * len(outs)
        else:
            outs, auxs = upscale_pngs(handles, pngs, a.batch, a.level, a.threads, bool(a.aux),
                                      stats, a.tile_pad, note, say)
    except (capi.S2SError, RuntimeError) as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    finally:
        for H in handles:
            H.close()
    for p, o, x in zip(a.input, outs, auxs):
        with open(target(a.output, p), "wb") as f:
            f.write(o)
        if a.aux and x is not None:
            with open(target(a.aux, p), "wb") as f:
                f.write(x)
    if not a.quiet:
        print(f"  {stats['images']} images, {stats['batches']} batches on {len(handles)} "
              f"device(s): {stats['seconds']:.2f}s "
              f"({stats['output_mpix'] / max(stats['seconds'], 1e-9):.1f} Mpx/s out)",
              file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
