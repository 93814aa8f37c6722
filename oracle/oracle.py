"""ctypes front of the C++ CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference's CPU forward (swin2sr-rs src/cpu.rs, see the
header of s2s_oracle.cpp for the op-by-op citations). It is the parity checker
for the CUDA path and the timed CPU baseline. Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline legs may import this module; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "s2s_oracle.cpp"
LIB = HERE / "libs2s_oracle.so"

UPS_CODE = {"pixelshuffle": 0, "pixelshuffledirect": 1, "nearest+conv": 2, "pixelshuffle_aux": 3}


class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.POINTER(ctypes.c_float)),
                ("numel", ctypes.c_int64)]


class _Config(ctypes.Structure):
    _fields_ = [("upsampler", ctypes.c_int), ("scale", ctypes.c_int), ("window", ctypes.c_int),
                ("embed", ctypes.c_int), ("heads", ctypes.c_int), ("mlp_ratio", ctypes.c_int),
                ("n_depths", ctypes.c_int), ("depths", ctypes.c_int * 16),
                ("img_range", ctypes.c_float), ("mean", ctypes.c_float * 3)]


DUMP_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float), ctypes.c_int64,
                           ctypes.c_void_p)


def build(force: bool = False) -> Path:
    """Compile the oracle (g++, OpenMP, no FMA contraction) into oracle/libs2s_oracle.so."""
    if LIB.exists() and not force and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cmd = ["g++", "-O3", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-march=x86-64-v3",
           "-fPIC", "-shared", "-o", str(LIB), str(SRC)]
    subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = ctypes.CDLL(str(LIB))
        fp = ctypes.POINTER(ctypes.c_float)
        L.oracle_forward.argtypes = [ctypes.POINTER(_Config), ctypes.POINTER(_Tensor), ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, fp, fp, fp, DUMP_FN,
                                     ctypes.c_void_p]
        L.oracle_forward.restype = ctypes.c_int
        L.oracle_bicubic.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, fp]
        L.oracle_conv3x3.argtypes = [fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp,
                                     ctypes.c_int, fp, fp]
        L.oracle_linear.argtypes = [fp, ctypes.c_int, ctypes.c_int, fp, ctypes.c_int, fp, fp]
        L.oracle_layer_norm.argtypes = [fp, fp, fp, fp, ctypes.c_int, ctypes.c_int]
        L.oracle_attention.argtypes = [ctypes.c_int] * 5 + [fp, fp, fp, ctypes.c_int, fp]
        L.oracle_fast_exp.argtypes = [ctypes.c_float]
        L.oracle_fast_exp.restype = ctypes.c_float
        L.oracle_pad_reflect.argtypes = [fp] + [ctypes.c_int] * 5 + [fp]
        L.oracle_set_threads.argtypes = [ctypes.c_int]
        L.oracle_max_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def forward(wt, h: int, w: int, adjusted: np.ndarray, dump=None):
    """Whole forward on a mean-adjusted [3][h][w] plane -> (out [3][h*s][w*s], aux or None)."""
    L = lib()
    names = wt.needed()
    keep, arr = [], (_Tensor * len(names))()
    for i, n in enumerate(names):
        a = np.ascontiguousarray(wt.t(n), dtype=np.float32)
        keep.append((n.encode(), a))
        arr[i].name = keep[-1][0]
        arr[i].data = _fp(a)
        arr[i].numel = a.size
    cfg = _Config()
    cfg.upsampler = UPS_CODE[wt.upsampler]
    cfg.scale, cfg.window, cfg.embed = wt.scale, wt.window, wt.embed
    cfg.heads, cfg.mlp_ratio, cfg.n_depths = wt.heads, wt.mlp_ratio, len(wt.depths)
    for i, d in enumerate(wt.depths):
        cfg.depths[i] = d
    cfg.img_range = wt.img_range
    for i in range(3):
        cfg.mean[i] = wt.mean[i]
    x = np.ascontiguousarray(adjusted, dtype=np.float32).reshape(3, h, w)
    s = wt.scale
    out = np.zeros((3, h * s, w * s), np.float32)
    hp, wp = (h // wt.window + 1) * wt.window, (w // wt.window + 1) * wt.window
    aux = np.zeros((3, hp, wp), np.float32) if wt.upsampler == "pixelshuffle_aux" else None
    store = {}
    if dump:
        def cb(name, data, n, _u):
            store[name.decode()] = np.ctypeslib.as_array(data, shape=(n,)).copy()
        fn = DUMP_FN(cb)
    else:
        fn = DUMP_FN(0)
    rc = L.oracle_forward(ctypes.byref(cfg), arr, len(names), h, w, _fp(x), _fp(out),
                          _fp(aux) if aux is not None else None, fn, None)
    if rc != 0:
        raise RuntimeError("oracle_forward failed (missing tensor?)")
    if dump:
        return out, aux, store
    return out, aux


def bicubic(x: np.ndarray, oh: int, ow: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    c, h, w = x.shape
    out = np.zeros((c, oh, ow), np.float32)
    lib().oracle_bicubic(_fp(x), c, h, w, oh, ow, _fp(out))
    return out


def conv3x3(x: np.ndarray, wgt: np.ndarray, bias: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    wgt = np.ascontiguousarray(wgt, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    ci, h, w = x.shape
    co = wgt.shape[0]
    out = np.zeros((co, h, w), np.float32)
    lib().oracle_conv3x3(_fp(x), ci, h, w, _fp(wgt), co, _fp(bias), _fp(out))
    return out


def linear(x: np.ndarray, wgt: np.ndarray, bias: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    wgt = np.ascontiguousarray(wgt, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    rows, ci = x.shape
    co = wgt.shape[0]
    out = np.zeros((rows, co), np.float32)
    lib().oracle_linear(_fp(x), rows, ci, _fp(wgt), co, _fp(bias), _fp(out))
    return out


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Channel LayerNorm over an NCHW-style [c][hw] plane."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    c, hw = x.shape
    y = np.zeros_like(x)
    lib().oracle_layer_norm(_fp(x), _fp(np.ascontiguousarray(w, np.float32)),
                            _fp(np.ascontiguousarray(b, np.float32)), _fp(y), c, hw)
    return y


def attention(hp, wp, win, heads, logit_scale, cpb, qkv, shift):
    """qkv [3][tokens][c] window-major -> out [tokens][c]."""
    qkv = np.ascontiguousarray(qkv, dtype=np.float32)
    c = qkv.shape[2]
    out = np.zeros((qkv.shape[1], c), np.float32)
    lib().oracle_attention(hp, wp, win, c, heads,
                           _fp(np.ascontiguousarray(logit_scale, np.float32).reshape(-1)),
                           _fp(np.ascontiguousarray(cpb, np.float32)), _fp(qkv), shift, _fp(out))
    return out


def fast_exp(x: float) -> float:
    return float(lib().oracle_fast_exp(float(x)))


def pad_reflect(x: np.ndarray, hp: int, wp: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    c, h, w = x.shape
    out = np.zeros((c, hp, wp), np.float32)
    lib().oracle_pad_reflect(_fp(x), c, h, w, hp, wp, _fp(out))
    return out


# ---- the image path either side of the forward (numpy: byte and scalar float work)

def load_samples(samples: np.ndarray, channels: int, bit_depth: int) -> np.ndarray:
    """swin2sr-rs src/image.rs:57-95: decoded PNG samples -> planar f32 [3][h][w].

    `samples` is [h][w][channels * bit_depth / 8] uint8 as the png crate returns it
    (16-bit samples big-endian). Each sample times the f32 constant 1/255 or 1/65535
    (`sample_scale`, :62-63); grey and grey+alpha repeat channel 0, RGB(A) take 0..2
    (:83-91)."""
    s = np.asarray(samples, np.uint8)
    h, w, _ = s.shape
    if bit_depth == 16:
        v = (s[..., 0::2].astype(np.uint32) << 8) | s[..., 1::2]
        scale = np.float32(1.0) / np.float32(65535.0)
    else:
        v = s.astype(np.uint32)
        scale = np.float32(1.0) / np.float32(255.0)
    v = v.reshape(h, w, channels).astype(np.float32) * scale
    idx = [0, 0, 0] if channels < 3 else [0, 1, 2]
    return np.ascontiguousarray(np.stack([v[..., i] for i in idx]), dtype=np.float32)


def adjust(img: np.ndarray, mean, img_range: float) -> np.ndarray:
    """swin2sr-rs src/backend.rs:76-86 Pre::adjust: (v - mean[c]) * img_range in f32."""
    x = np.asarray(img, np.float32)
    m = np.asarray(mean, np.float32).reshape(3, 1, 1)
    return ((x - m) * np.float32(img_range)).astype(np.float32)


def to_rgb8(img: np.ndarray) -> np.ndarray:
    """swin2sr-rs src/image.rs:28-39 Image::to_rgb8: planar [3][h][w] f32 ->
    interleaved [h][w][3] bytes. Per value: clamp to [0,1] (f32::clamp keeps NaN),
    * 255, + 0.5, floor, min 255 (f32::min returns the non-NaN operand, so NaN ->
    255), `as u8` (saturating)."""
    x = np.asarray(img, np.float32)
    c = np.clip(x, np.float32(0.0), np.float32(1.0))          # NaN stays NaN
    v = np.floor(c * np.float32(255.0) + np.float32(0.5))      # f32 ops, one rounding each
    v = np.fmin(v, np.float32(255.0))                          # NaN -> 255
    return np.ascontiguousarray(v.astype(np.uint8).transpose(1, 2, 0))


if __name__ == "__main__":
    print(build(force=True))
    print("threads", max_threads(), os.cpu_count())
