"""Seeded random-init ACT checkpoints in the vla.simd converter's directory format.

There is no network here and no trained checkpoint, so the benchmark and the
parity tests run on random-init weights of the ACT architecture, written in
exactly the layout the reference's ``tools/convert_act.py`` produces (and both
the reference's ``vla_act_load`` and this library's read):

    config.txt     img_h / img_w / n_cams / norm_eps / camera names
                   (src/models/act/act_model.cpp:25-44)
    backbone.meta  stem + ``block cin cout stride has_down`` table
    backbone.bin   fp32 arena: stem W [Cout,k,k,Cin] + bias, then per block
                   conv1, conv2, (down) - BatchNorm already folded
                   (src/models/act/resnet_backbone.cpp:50-151)
    act.meta       transformer dims (src/models/act/act_transformer.cpp:29-60)
    act.bin        fp32 arena in ActTransformer::load order (:67-117)
    stats.bin      state mean/std, action mean/std, per-camera image mean/std
                   (src/models/act/act_model.cpp:68-91)

numpy's PCG64 stream makes the files identical on every machine for a seed.
"""
from __future__ import annotations

import dataclasses
import os

import numpy as np


@dataclasses.dataclass(frozen=True)
class ActShape:
    img_h: int = 480
    img_w: int = 640
    n_cams: int = 2
    dim: int = 512
    heads: int = 8
    ff: int = 3200
    n_enc: int = 4
    n_dec: int = 1
    chunk: int = 100
    state_dim: int = 6
    action_dim: int = 6
    stem_out: int = 64
    widths: tuple = (64, 128, 256, 512)   # ResNet-18 stage widths, 2 basic blocks each

    @property
    def head_dim(self) -> int:
        return self.dim // self.heads


# ACT, 2 cameras 480x640, d 512, 8 heads, FFN 3200,
# 4 encoder / 1 decoder layers, chunk 100, 6-dim state and action.
ACT_BASELINE = ActShape()
# a reduced ACT for fast tests (same code paths, every width a multiple of 16)
ACT_SMALL = ActShape(img_h=64, img_w=96, dim=128, heads=2, ff=256, n_enc=2, n_dec=1, chunk=16,
                     stem_out=16, widths=(16, 32, 48, 64))


def _block_table(s: ActShape):
    blocks = []
    cin = s.stem_out
    for si, w in enumerate(s.widths):
        for b in range(2):
            stride = 2 if (si > 0 and b == 0) else 1
            has_down = int(cin != w or stride != 1)
            blocks.append((cin, w, stride, has_down))
            cin = w
    return blocks


def write_act_checkpoint(out_dir: str, shape: ActShape = ACT_BASELINE, seed: int = 0) -> str:
    """Write a random-init ACT checkpoint directory; returns out_dir."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    s = shape

    def normal(shape_, std):
        return (rng.standard_normal(shape_, dtype=np.float32) * np.float32(std)).astype(np.float32)

    # ---- backbone (folded BN: conv weight + bias), He init; the second conv of
    # a block is damped so the residual stream stays O(1) through 8 blocks
    parts = []
    k = 7
    parts += [normal((s.stem_out, k, k, 3), np.sqrt(2.0 / (k * k * 3))), normal((s.stem_out,), 0.05)]
    meta = ["in_ch 3", f"stem_out {s.stem_out}", f"stem_k {k}", "stem_stride 2", f"stem_pad {k // 2}",
            "pool_k 3", "pool_stride 2", "pool_pad 1"]
    for cin, cout, stride, has_down in _block_table(s):
        parts += [normal((cout, 3, 3, cin), np.sqrt(2.0 / (9 * cin))), normal((cout,), 0.05)]
        parts += [normal((cout, 3, 3, cout), 0.5 * np.sqrt(2.0 / (9 * cout))), normal((cout,), 0.05)]
        if has_down:
            parts += [normal((cout, 1, 1, cin), np.sqrt(1.0 / cin)), normal((cout,), 0.05)]
        meta.append(f"block {cin} {cout} {stride} {has_down}")
    with open(os.path.join(out_dir, "backbone.meta"), "w") as f:
        f.write("\n".join(meta) + "\n")
    np.concatenate([p.reshape(-1) for p in parts]).astype(np.float32).tofile(os.path.join(out_dir, "backbone.bin"))

    # ---- transformer, ActTransformer::load order
    d, ff = s.dim, s.ff
    img_ch = s.widths[-1]
    parts = []

    def linear(n, kk):
        parts.extend([normal((n, kk), 0.02), normal((n,), 0.01)])

    def norm():
        parts.extend([(1.0 + normal((d,), 0.05)).astype(np.float32), normal((d,), 0.02)])

    linear(d, img_ch)                # img_proj
    linear(d, s.state_dim)           # state_proj
    parts.append(normal((d,), 0.5))  # latent token
    parts.append(normal((2, d), 0.5))  # pos1d (latent, state)
    for _ in range(s.n_enc):
        for _ in range(4):
            linear(d, d)             # wq wk wv wo
        norm()
        linear(ff, d)
        linear(d, ff)
        norm()
    for _ in range(s.n_dec):
        for _ in range(4):
            linear(d, d)             # self
        norm()
        for _ in range(4):
            linear(d, d)             # cross
        norm()
        linear(ff, d)
        linear(d, ff)
        norm()
    parts.append(normal((s.chunk, d), 0.5))  # decoder query positions
    norm()                                   # final decoder norm
    linear(s.action_dim, d)                  # head
    with open(os.path.join(out_dir, "act.meta"), "w") as f:
        f.write("\n".join([f"dim {d}", f"heads {s.heads}", f"head_dim {s.head_dim}", f"ff {ff}",
                           f"n_enc {s.n_enc}", f"n_dec {s.n_dec}", f"chunk {s.chunk}",
                           f"state_dim {s.state_dim}", f"action_dim {s.action_dim}", "n_1d 2", "n_text 0",
                           "ln_eps 1e-5"]) + "\n")
    np.concatenate([p.reshape(-1) for p in parts]).astype(np.float32).tofile(os.path.join(out_dir, "act.bin"))

    # ---- stats: state / action mean+std, then per camera image mean+std
    stats = [normal((s.state_dim,), 1.0), rng.uniform(0.5, 2.0, s.state_dim).astype(np.float32),
             normal((s.action_dim,), 1.0), rng.uniform(0.5, 2.0, s.action_dim).astype(np.float32)]
    for _ in range(s.n_cams):
        stats.append(np.array([0.485, 0.456, 0.406], np.float32))
        stats.append(np.array([0.229, 0.224, 0.225], np.float32))
    np.concatenate(stats).astype(np.float32).tofile(os.path.join(out_dir, "stats.bin"))

    with open(os.path.join(out_dir, "config.txt"), "w") as f:
        f.write(f"img_h {s.img_h}\nimg_w {s.img_w}\nn_cams {s.n_cams}\nnorm_eps 1e-05\n")
        for c in range(s.n_cams):
            f.write(f"cam{c} observation.images.cam{c}\n")
    return out_dir


def act_inputs(shape: ActShape = ACT_BASELINE, seed: int = 1):
    """Seeded observation: uint8 frames [n_cams, H, W, 3] ~ U{0..255}, state ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    frames = rng.integers(0, 256, size=(shape.n_cams, shape.img_h, shape.img_w, 3), dtype=np.uint8)
    state = rng.standard_normal(shape.state_dim, dtype=np.float32)
    return frames, state
