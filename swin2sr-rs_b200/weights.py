"""The checkpoint the forward pass consumes: seeded generation, conversion, I/O.

Three jobs, each mirroring a piece of the reference:

* ``seeded_state_dict`` builds a raw (torch-named) Swin2SR state dict with the
  initialisation the published network applies (``tools/network_swin2sr.py:886-893``
  and ``tools/timm_shim.py:33-36``): Linear weights normal(0, 0.02) clamped to two
  standard deviations, Linear biases 0, Conv2d kaiming-uniform(a=sqrt 5) weights and
  uniform(+-1/sqrt fan_in) biases, LayerNorm weight 1 / bias 0, ``logit_scale``
  log(10), ``q_bias``/``v_bias`` 0. The random stream is numpy PCG64 from a seed,
  so the GPU box regenerates the same weights without the reference present.
  ``perturb=True`` additionally moves every bias and norm parameter off its
  trivial init, so tests exercise the affine terms.
* ``convert`` restates ``tools/convert.py``: the fused QKV is sliced into
  ``qkv.wq/wk/wv`` + ``qkv.q_bias/v_bias`` (``convert.py:122-138``) and the
  continuous position bias MLP is folded into the ``cpb_pre`` [N*N][heads] table
  (``convert.py:141-167``), with the architecture written to ``__metadata__``
  (``convert.py:224-236``).
* ``Weights`` mirrors ``src/weights.rs``: metadata parse (``:90-137``), shape
  validation (``:142-235``), tensor access ``t``/``shape``/``has`` (``:240-255``)
  and the FLOP counters (``:258-316``).
"""
from __future__ import annotations

import json
import math
import struct
from pathlib import Path

import numpy as np

# The released configurations (tools/convert.py:46-58).
CONFIGS = {
    "classical_sr": dict(upsampler="pixelshuffle", scale=4, win=8, embed=180, heads=6,
                         mlp_ratio=2, depths=[6] * 6),
    "classical_sr_x2": dict(upsampler="pixelshuffle", scale=2, win=8, embed=180, heads=6,
                            mlp_ratio=2, depths=[6] * 6),
    "real_sr": dict(upsampler="nearest+conv", scale=4, win=8, embed=180, heads=6,
                    mlp_ratio=2, depths=[6] * 6),
    "compressed_sr": dict(upsampler="pixelshuffle_aux", scale=4, win=8, embed=180, heads=6,
                          mlp_ratio=2, depths=[6] * 6),
    "lightweight_sr": dict(upsampler="pixelshuffledirect", scale=2, win=8, embed=60, heads=6,
                           mlp_ratio=2, depths=[6] * 4),
}

UPSAMPLERS = ("pixelshuffle", "pixelshuffledirect", "nearest+conv", "pixelshuffle_aux")
RGB_MEAN = (0.4488, 0.4371, 0.4040)        # src/weights.rs:68
NUM_FEAT = 64                              # network_swin2sr.py: num_feat of every head


def octaves(upsampler: str, scale: int) -> int:
    """Reconstruction steps per head (src/weights.rs:58-66)."""
    if upsampler in ("pixelshuffle", "pixelshuffle_aux"):
        return int(round(math.log2(scale)))
    if upsampler == "pixelshuffledirect":
        return 1
    return 2


# ---------------------------------------------------------------------------
# Seeded raw state dict.
# ---------------------------------------------------------------------------

class _Init:
    def __init__(self, seed: int):
        self.rng = np.random.Generator(np.random.PCG64(seed))

    def linear(self, out_f, in_f, bias=True):
        w = self.rng.normal(0.0, 0.02, size=(out_f, in_f)).clip(-0.04, 0.04).astype(np.float32)
        return w, (np.zeros(out_f, np.float32) if bias else None)

    def conv(self, out_c, in_c, k):
        fan_in = in_c * k * k
        bound = 1.0 / math.sqrt(fan_in)
        w = self.rng.uniform(-bound, bound, size=(out_c, in_c, k, k)).astype(np.float32)
        b = self.rng.uniform(-bound, bound, size=(out_c,)).astype(np.float32)
        return w, b


def relative_coords_table(win: int) -> np.ndarray:
    """[1][2w-1][2w-1][2] log-spaced relative coordinates (network_swin2sr.py:103-120)."""
    r = np.arange(-(win - 1), win, dtype=np.float32)
    hh, ww = np.meshgrid(r, r, indexing="ij")
    t = np.stack([hh, ww], axis=-1)[None].astype(np.float32)
    t = t / np.float32(win - 1)
    t = t * np.float32(8)
    t = np.sign(t) * np.log2(np.abs(t) + np.float32(1.0)) / np.float32(np.log2(8))
    return t.astype(np.float32)


def relative_position_index(win: int) -> np.ndarray:
    """[N][N] index into the flattened coords table (network_swin2sr.py:122-131)."""
    ch, cw = np.meshgrid(np.arange(win), np.arange(win), indexing="ij")
    coords = np.stack([ch.reshape(-1), cw.reshape(-1)])            # 2, N
    rel = coords[:, :, None] - coords[:, None, :]                   # 2, N, N
    rel = rel.transpose(1, 2, 0).copy()
    rel[:, :, 0] += win - 1
    rel[:, :, 1] += win - 1
    rel[:, :, 0] *= 2 * win - 1
    return rel.sum(-1).astype(np.int64)


def seeded_state_dict(task: str, seed: int = 0, perturb: bool = False) -> dict:
    """A raw Swin2SR state dict (torch names) for ``task``'s architecture."""
    cfg = CONFIGS[task]
    c, heads, win, mlp = cfg["embed"], cfg["heads"], cfg["win"], cfg["mlp_ratio"]
    ups, scale, feat = cfg["upsampler"], cfg["scale"], NUM_FEAT
    ini = _Init(seed)
    sd: dict[str, np.ndarray] = {}

    def put_conv(name, oc, ic, k=3):
        sd[f"{name}.weight"], sd[f"{name}.bias"] = ini.conv(oc, ic, k)

    def put_ln(name, n):
        sd[f"{name}.weight"] = np.ones(n, np.float32)
        sd[f"{name}.bias"] = np.zeros(n, np.float32)

    put_conv("conv_first", c, 3)
    put_conv("patch_embed.proj", c, c, 1)
    put_ln("patch_embed.norm", c)
    table = relative_coords_table(win)
    index = relative_position_index(win)
    for l, depth in enumerate(cfg["depths"]):
        for b in range(depth):
            p = f"layers.{l}.residual_group.blocks.{b}"
            sd[f"{p}.attn.logit_scale"] = np.full((heads, 1, 1), math.log(10.0), np.float32)
            w0, b0 = ini.linear(512, 2)
            sd[f"{p}.attn.cpb_mlp.0.weight"], sd[f"{p}.attn.cpb_mlp.0.bias"] = w0, b0
            sd[f"{p}.attn.cpb_mlp.2.weight"], _ = ini.linear(heads, 512, bias=False)
            sd[f"{p}.attn.q_bias"] = np.zeros(c, np.float32)
            sd[f"{p}.attn.v_bias"] = np.zeros(c, np.float32)
            sd[f"{p}.attn.relative_coords_table"] = table.copy()
            sd[f"{p}.attn.relative_position_index"] = index.copy()
            sd[f"{p}.attn.qkv.weight"], _ = ini.linear(3 * c, c, bias=False)
            sd[f"{p}.attn.proj.weight"], sd[f"{p}.attn.proj.bias"] = ini.linear(c, c)
            put_ln(f"{p}.norm1", c)
            sd[f"{p}.mlp.fc1.weight"], sd[f"{p}.mlp.fc1.bias"] = ini.linear(mlp * c, c)
            sd[f"{p}.mlp.fc2.weight"], sd[f"{p}.mlp.fc2.bias"] = ini.linear(c, mlp * c)
            put_ln(f"{p}.norm2", c)
        put_conv(f"layers.{l}.conv", c, c)
        put_conv(f"layers.{l}.patch_embed.proj", c, c, 1)
    put_ln("norm", c)
    put_conv("conv_after_body", c, c)
    if ups == "pixelshuffle":
        put_conv("conv_before_upsample.0", feat, c)
        for o in range(octaves(ups, scale)):
            put_conv(f"upsample.{2 * o}", 4 * feat, feat)
        put_conv("conv_last", 3, feat)
    elif ups == "pixelshuffle_aux":
        put_conv("conv_bicubic", feat, 3)
        put_conv("conv_before_upsample.0", feat, c)
        put_conv("conv_aux", 3, feat)
        put_conv("conv_after_aux.0", feat, 3)
        for o in range(octaves(ups, scale)):
            put_conv(f"upsample.{2 * o}", 4 * feat, feat)
        put_conv("conv_last", 3, feat)
    elif ups == "pixelshuffledirect":
        put_conv("upsample.0", 3 * scale * scale, c)
    elif ups == "nearest+conv":
        put_conv("conv_before_upsample.0", feat, c)
        put_conv("conv_up1", feat, feat)
        put_conv("conv_up2", feat, feat)
        put_conv("conv_hr", feat, feat)
        put_conv("conv_last", 3, feat)

    if perturb:
        rng = np.random.Generator(np.random.PCG64(seed + 1000))
        for k in sorted(sd):
            v = sd[k]
            if k.endswith("relative_coords_table") or k.endswith("relative_position_index"):
                continue
            if "norm" in k and k.endswith(".weight"):
                sd[k] = (v + rng.normal(0, 0.1, v.shape)).astype(np.float32)
            elif k.endswith("bias") and ("conv" not in k and "upsample" not in k):
                scale_ = 0.1 if ("norm" in k or "q_bias" in k or "v_bias" in k) else 0.02
                sd[k] = (v + rng.normal(0, scale_, v.shape)).astype(np.float32)
            elif k.endswith("logit_scale"):
                ls = v + rng.normal(0, 0.5, v.shape).astype(np.float32)
                ls.reshape(-1)[0] = 5.0          # above ln(100): exercises the clamp
                sd[k] = ls.astype(np.float32)
    return sd


# ---------------------------------------------------------------------------
# Conversion (tools/convert.py restated).
# ---------------------------------------------------------------------------

def infer(sd: dict):
    """Architecture from tensor names and shapes (tools/convert.py:83-119)."""
    depth = max(int(k.split(".")[1]) for k in sd if k.startswith("layers.")) + 1
    per = [0] * depth
    for k in sd:
        p = k.split(".")
        if len(p) > 4 and p[0] == "layers" and p[2] == "residual_group" and p[3] == "blocks":
            per[int(p[1])] = max(per[int(p[1])], int(p[4]) + 1)
    embed = int(sd["conv_first.weight"].shape[0])
    win = (int(sd["layers.0.residual_group.blocks.0.attn.relative_coords_table"].shape[1]) + 1) // 2
    mlp = int(sd["layers.0.residual_group.blocks.0.mlp.fc1.weight"].shape[0]) // embed
    if "conv_aux.weight" in sd or "conv_bicubic.weight" in sd:
        ups = "pixelshuffle_aux"
    elif "conv_before_upsample.0.weight" in sd:
        ups = "nearest+conv" if "conv_up1.weight" in sd else "pixelshuffle"
    elif "upsample.0.weight" in sd:
        ups = "pixelshuffledirect"
    else:
        ups = "pixelshuffle_aux"
    return per, embed, win, mlp, ups


def precompute_cpb(sd: dict, per, out: dict) -> None:
    """``cpb_pre`` = 16*sigmoid(relu(table W0^T + b0) W2^T)[index] (tools/convert.py:141-167)."""
    base = "layers.0.residual_group.blocks.0.attn"
    t = sd[f"{base}.relative_coords_table"].astype(np.float32).reshape(-1, 2)
    index = sd[f"{base}.relative_position_index"].astype(np.int64)
    for l, depth in enumerate(per):
        for b in range(depth):
            p = f"layers.{l}.residual_group.blocks.{b}.attn"
            w0 = sd[f"{p}.cpb_mlp.0.weight"].astype(np.float32)
            b0 = sd[f"{p}.cpb_mlp.0.bias"].astype(np.float32)
            w2 = sd[f"{p}.cpb_mlp.2.weight"].astype(np.float32)
            h = t @ w0.T + b0
            h = np.maximum(h, 0.0)
            h = h @ w2.T
            bias = h[index.reshape(-1)]
            bias = 16.0 / (1.0 + np.exp(-bias))
            out[f"{p}.cpb_pre"] = np.ascontiguousarray(bias.astype(np.float32))


def convert(sd: dict, task: str, scale: int | None = None):
    """Raw state dict -> (converted tensors, metadata), as tools/convert.py writes them."""
    cfg = CONFIGS[task]
    per, embed, win, mlp, ups = infer(sd)
    heads = int(sd["layers.0.residual_group.blocks.0.attn.logit_scale"].shape[0])
    out = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in sd.items()
           if np.issubdtype(v.dtype, np.floating)}
    for l, depth in enumerate(per):
        for b in range(depth):
            p = f"layers.{l}.residual_group.blocks.{b}.attn"
            w = sd[f"{p}.qkv.weight"]
            c = w.shape[1]
            out[f"{p}.qkv.wq"] = np.ascontiguousarray(w[:c])
            out[f"{p}.qkv.wk"] = np.ascontiguousarray(w[c:2 * c])
            out[f"{p}.qkv.wv"] = np.ascontiguousarray(w[2 * c:])
            out[f"{p}.qkv.q_bias"] = np.ascontiguousarray(sd[f"{p}.q_bias"])
            out[f"{p}.qkv.v_bias"] = np.ascontiguousarray(sd[f"{p}.v_bias"])
    precompute_cpb(sd, per, out)
    meta = {
        "task": task, "upsampler": ups, "scale": str(scale or cfg["scale"]),
        "window_size": str(win), "embed_dim": str(embed), "num_heads": str(heads),
        "mlp_ratio": str(mlp), "depths": ",".join(str(v) for v in per),
        "img_range": "1.0", "rgb_mean": "0.4488,0.4371,0.4040", "format": "pt",
    }
    return out, meta


# ---------------------------------------------------------------------------
# safetensors (F32 only, which is all tools/convert.py writes).
# ---------------------------------------------------------------------------

def save_safetensors(path, tensors: dict, metadata: dict) -> None:
    items = sorted(tensors.items())
    header, offset = {}, 0
    for name, a in items:
        n = a.size * 4
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [offset, offset + n]}
        offset += n
    header["__metadata__"] = metadata
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((-(8 + len(hj))) & 7)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for _, a in items:
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())


def load_safetensors(path):
    raw = Path(path).read_bytes()
    (hl,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hl])
    meta = header.pop("__metadata__", {})
    base = 8 + hl
    out = {}
    for name, info in header.items():
        if info["dtype"] != "F32":
            raise ValueError(f"{path}: {name} is {info['dtype']}, only F32 is supported")
        a, b = info["data_offsets"]
        out[name] = np.frombuffer(raw, dtype="<f4", count=(b - a) // 4, offset=base + a) \
            .reshape(info["shape"]).copy()
    return out, meta


# ---------------------------------------------------------------------------
# Weights (src/weights.rs restated).
# ---------------------------------------------------------------------------

class Weights:
    """A converted checkpoint: tensors plus the architecture its metadata claims."""

    def __init__(self, tensors: dict, meta: dict, source: str = "<memory>"):
        for k in ("task", "upsampler", "scale", "window_size", "embed_dim", "num_heads",
                  "mlp_ratio", "depths", "img_range", "rgb_mean"):
            if k not in meta:
                raise ValueError(f"{source}: no `{k}` in __metadata__ - convert the checkpoint "
                                 f"with tools/convert.py, which records the architecture")
        if meta["upsampler"] not in UPSAMPLERS:
            raise ValueError(f"upsampler `{meta['upsampler']}` is not one this engine implements "
                             f"({', '.join(UPSAMPLERS)})")
        self.tensors = tensors
        self.meta = dict(meta)
        self.task = meta["task"]
        self.upsampler = meta["upsampler"]
        self.scale = int(meta["scale"])
        self.window = int(meta["window_size"])
        self.embed = int(meta["embed_dim"])
        self.heads = int(meta["num_heads"])
        self.head_dim = self.embed // self.heads
        self.mlp_ratio = int(meta["mlp_ratio"])
        self.depths = [int(s) for s in meta["depths"].split(",")]
        self.img_range = float(meta["img_range"])
        mean = [float(s) for s in meta["rgb_mean"].split(",")]
        if len(mean) != 3:
            raise ValueError(f"rgb_mean has {len(mean)} entries, expected 3")
        self.mean = mean
        self.source = source
        self.validate()

    @classmethod
    def load(cls, path):
        t, m = load_safetensors(path)
        return cls(t, m, str(path))

    @classmethod
    def seeded(cls, task: str, seed: int = 0, perturb: bool = False):
        t, m = convert(seeded_state_dict(task, seed, perturb), task)
        return cls(t, m, f"<seeded {task} seed={seed}{' perturbed' if perturb else ''}>")

    def t(self, name: str) -> np.ndarray:
        if name not in self.tensors:
            raise KeyError(f"weight `{name}` is not in {self.source}")
        return self.tensors[name]

    def shape(self, name: str):
        return tuple(self.t(name).shape)

    def has(self, name: str) -> bool:
        return name in self.tensors

    @property
    def feat(self) -> int:
        if self.has("conv_before_upsample.0.weight"):
            return self.shape("conv_before_upsample.0.weight")[0]
        return NUM_FEAT

    def validate(self) -> None:
        """Shape checks of src/weights.rs:142-235."""
        e, src = self.embed, self.source
        want = [("conv_first.weight", (e, 3, 3, 3)), ("conv_after_body.weight", (e, e, 3, 3)),
                ("norm.weight", (e,)), ("patch_embed.proj.weight", (e, e, 1, 1)),
                ("patch_embed.norm.weight", (e,))]
        if self.upsampler != "pixelshuffledirect":
            want.append(("conv_last.bias", (3,)))
        w = self.window
        for l, d in enumerate(self.depths):
            for b in range(d):
                p = f"layers.{l}.residual_group.blocks.{b}"
                want += [(f"{p}.attn.qkv.wq", (e, e)), (f"{p}.attn.qkv.wv", (e, e)),
                         (f"{p}.attn.proj.weight", (e, e)),
                         (f"{p}.mlp.fc1.weight", (self.mlp_ratio * e, e)),
                         (f"{p}.mlp.fc2.weight", (e, self.mlp_ratio * e)),
                         (f"{p}.attn.cpb_pre", (w ** 4, self.heads))]
        if self.upsampler == "pixelshuffle_aux":
            f = self.feat
            want += [("conv_bicubic.weight", (f, 3, 3, 3)), ("conv_bicubic.bias", (f,)),
                     ("conv_aux.weight", (3, f, 3, 3)), ("conv_aux.bias", (3,)),
                     ("conv_after_aux.0.weight", (f, 3, 3, 3)), ("conv_after_aux.0.bias", (f,))]
        if self.upsampler == "pixelshuffledirect":
            want.append(("upsample.0.weight", (self.scale * self.scale * 3, e, 3, 3)))
        for name, shp in want:
            if name not in self.tensors:
                raise ValueError(f"{src}: {name}: tensor not found")
            got = tuple(self.tensors[name].shape)
            if got != shp:
                raise ValueError(f"{src}: {name} is {list(got)}, the {len(self.depths)}-stage/"
                                 f"{e}-wide architecture in the header implies {list(shp)}")

    def needed(self):
        """Every tensor name the forward pass reads (the set src/gpu.rs:801-872 uploads)."""
        names = ["conv_first.weight", "conv_first.bias", "patch_embed.proj.weight",
                 "patch_embed.proj.bias", "patch_embed.norm.weight", "patch_embed.norm.bias",
                 "norm.weight", "norm.bias", "conv_after_body.weight", "conv_after_body.bias"]
        for l, d in enumerate(self.depths):
            for b in range(d):
                p = f"layers.{l}.residual_group.blocks.{b}"
                names += [f"{p}.attn.qkv.{s}" for s in ("wq", "wk", "wv", "q_bias", "v_bias")]
                names += [f"{p}.attn.logit_scale", f"{p}.attn.cpb_pre",
                          f"{p}.attn.proj.weight", f"{p}.attn.proj.bias",
                          f"{p}.norm1.weight", f"{p}.norm1.bias", f"{p}.norm2.weight",
                          f"{p}.norm2.bias", f"{p}.mlp.fc1.weight", f"{p}.mlp.fc1.bias",
                          f"{p}.mlp.fc2.weight", f"{p}.mlp.fc2.bias"]
            names += [f"layers.{l}.conv.weight", f"layers.{l}.conv.bias",
                      f"layers.{l}.patch_embed.proj.weight", f"layers.{l}.patch_embed.proj.bias"]
        u = self.upsampler
        convs = []
        if u == "pixelshuffle":
            convs = ["conv_before_upsample.0"] + [f"upsample.{2 * o}" for o in
                                                  range(octaves(u, self.scale))] + ["conv_last"]
        elif u == "pixelshuffle_aux":
            convs = ["conv_bicubic", "conv_before_upsample.0", "conv_aux", "conv_after_aux.0"] + \
                [f"upsample.{2 * o}" for o in range(octaves(u, self.scale))] + ["conv_last"]
        elif u == "pixelshuffledirect":
            convs = ["upsample.0"]
        elif u == "nearest+conv":
            convs = ["conv_before_upsample.0", "conv_up1", "conv_up2", "conv_hr", "conv_last"]
        for cname in convs:
            names += [f"{cname}.weight", f"{cname}.bias"]
        return names

    # -- FLOP accounting (2*MAC), on the padded plane, as the forward computes it --------
    def flops_forward(self, hp: int, wp: int, batch: int = 1) -> int:
        """Algorithmic FLOPs of one forward over a padded ``hp`` x ``wp`` plane: every conv
        (3x3 and 1x1), every linear (QKV, proj, fc1, fc2) and attention (QK^T + PV)."""
        hw, c, m = hp * wp, self.embed, self.mlp_ratio
        blocks = sum(self.depths)
        mac = hw * 3 * c * 9 + hw * c * c                       # conv_first, patch_embed
        mac += blocks * hw * (4 * c * c + 2 * m * c * c + 2 * self.window ** 2 * c)
        mac += len(self.depths) * hw * (9 * c * c + c * c)      # stage conv + patch_embed
        mac += hw * 9 * c * c                                    # conv_after_body
        f, u, s = self.feat, self.upsampler, self.scale
        if u in ("pixelshuffle", "pixelshuffle_aux"):
            mac += hw * c * f * 9
            cur = hw
            for _ in range(octaves(u, s)):
                mac += cur * f * 4 * f * 9
                cur *= 4
            mac += cur * f * 3 * 9
            if u == "pixelshuffle_aux":
                mac += cur * 3 * f * 9 + hw * f * 3 * 9 + hw * 3 * f * 9
        elif u == "pixelshuffledirect":
            mac += hw * c * 3 * s * s * 9
        else:
            mac += hw * c * f * 9
            mac += 4 * hw * f * f * 9 + 16 * hw * f * f * 9 * 2 + 16 * hw * f * 3 * 9
        return 2 * mac * batch

    def flops_gemm_body(self, hp: int, wp: int, batch: int = 1) -> int:
        """FLOPs of the per-block attention/MLP contractions (QKV, QK^T, PV, proj, fc1, fc2)."""
        hw, c, m = hp * wp, self.embed, self.mlp_ratio
        blocks = sum(self.depths)
        return 2 * batch * blocks * hw * (4 * c * c + 2 * m * c * c + 2 * self.window ** 2 * c)
