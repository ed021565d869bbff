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

import collections
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


# ---------------------------------------------------------------------------
# Diffusion Policy (the reference's src/models/diffusion), random-init.
#
#     diffusion.meta                 shapes + sampler settings
#                                    (src/models/diffusion/diffusion_model.cpp:25-88)
#     rgb_encoder{i}_backbone.meta   ResNet-18 table + gn_group_size
#     rgb_encoder{i}_backbone.bin    stem W, GroupNorm scale/shift, then per block
#                                    conv1 W + GN, conv2 W + GN, (down W + GN); no conv
#                                    bias (src/models/act/resnet_backbone.cpp:100-150)
#     rgb_encoder{i}.bin             1x1 keypoint conv [K, C] + bias, output linear
#                                    [2K, 2K] + bias (src/models/diffusion/rgb_encoder.cpp:45-56)
#     unet.bin                       DPUNet1d::load order (src/models/diffusion/unet1d.cpp:18-33)
#     stats.bin                      state min/max, action min/max, per-camera image
#                                    mean/std (diffusion_model.cpp:123-141)

@dataclasses.dataclass(frozen=True)
class DpShape:
    n_obs_steps: int = 2
    n_cams: int = 1
    img_h: int = 96
    img_w: int = 96
    crop_h: int = 84
    crop_w: int = 84
    state_dim: int = 2
    action_dim: int = 2
    horizon: int = 16
    n_action_steps: int = 8
    num_keypoints: int = 32
    kernel_size: int = 5
    n_groups: int = 8
    step_embed_dim: int = 128
    film_scale: bool = True
    separate_encoders: bool = True
    down_dims: tuple = (512, 1024, 2048)
    num_train_timesteps: int = 100
    num_inference_steps: int = 10
    scheduler: str = "DDIM"
    beta_schedule: str = "squaredcos_cap_v2"
    clip_sample: bool = True
    stem_out: int = 64
    widths: tuple = (64, 128, 256, 512)
    gn_group_size: int = 16

    @property
    def cond_dim(self) -> int:
        return self.step_embed_dim + (self.state_dim + self.n_cams * 2 * self.num_keypoints) * self.n_obs_steps


# ResNet-18 + GroupNorm + spatial softmax on a 2-frame
# history of 84x84 crops (96x96 frames, center-cropped as PushT), 2-dim state and
# action, U-Net (512, 1024, 2048), kernel 5, 8 groups, FiLM, horizon 16, DDIM 10.
DP_BASELINE = DpShape()
# reduced DP for fast tests: two cameras with separate encoders, narrow widths
DP_SMALL = DpShape(n_cams=2, img_h=40, img_w=48, crop_h=32, crop_w=40, state_dim=3, action_dim=4, horizon=16,
                   n_action_steps=6, num_keypoints=8, down_dims=(64, 128, 256), step_embed_dim=32,
                   stem_out=16, widths=(16, 32, 48, 64))
# edge cases of the same code paths: one encoder shared by both cameras, no
# crop, a folded-BatchNorm backbone (gn_group_size 0), bias-only FiLM, kernel 3,
# a two-level U-Net on horizon 8 with channel counts that are not multiples of
# 32 per group, scaled_linear betas over 50 training steps (DDIM ladder of 6),
# no sample clipping
DP_EDGE = DpShape(n_cams=2, separate_encoders=False, img_h=32, img_w=40, crop_h=0, crop_w=0, state_dim=5,
                  action_dim=3, horizon=8, n_action_steps=4, num_keypoints=8, kernel_size=3, n_groups=8,
                  step_embed_dim=16, film_scale=False, down_dims=(32, 48), num_train_timesteps=50,
                  num_inference_steps=6, beta_schedule="scaled_linear", clip_sample=False, stem_out=16,
                  widths=(16, 32, 48, 64), gn_group_size=0)
# one camera, one observation step, a four-level U-Net on horizon 32, linear betas
DP_DEEP = DpShape(n_obs_steps=1, n_cams=1, img_h=36, img_w=36, crop_h=28, crop_w=30, state_dim=2, action_dim=2,
                  horizon=32, n_action_steps=12, num_keypoints=16, kernel_size=5, n_groups=4, step_embed_dim=24,
                  down_dims=(16, 32, 64, 96), num_train_timesteps=100, num_inference_steps=8,
                  beta_schedule="linear", stem_out=16, widths=(16, 32, 48, 64), gn_group_size=8)


def write_dp_checkpoint(out_dir: str, shape: DpShape = DP_BASELINE, seed: int = 0) -> str:
    """Write a random-init Diffusion Policy checkpoint directory; returns out_dir."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    s = shape

    def normal(shape_, std):
        return (rng.standard_normal(shape_, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def save(name, parts):
        np.concatenate([p.reshape(-1) for p in parts]).astype(np.float32).tofile(os.path.join(out_dir, name))

    def gn(c):
        return [(1.0 + normal((c,), 0.05)).astype(np.float32), normal((c,), 0.05)]

    def norm(c):   # backbone GroupNorm scale/shift, or a folded BatchNorm's bias (gn_group_size 0)
        return gn(c) if s.gn_group_size else [normal((c,), 0.05)]

    n_enc = s.n_cams if s.separate_encoders else 1
    ashape = ActShape(stem_out=s.stem_out, widths=s.widths)
    for e in range(n_enc):
        parts = []
        k = 7
        parts += [normal((s.stem_out, k, k, 3), np.sqrt(2.0 / (k * k * 3)))] + norm(s.stem_out)
        meta = ["in_ch 3", f"stem_out {s.stem_out}", f"stem_k {k}", "stem_stride 2", f"stem_pad {k // 2}",
                "pool_k 3", "pool_stride 2", "pool_pad 1"]
        for cin, cout, stride, has_down in _block_table(ashape):
            parts += [normal((cout, 3, 3, cin), np.sqrt(2.0 / (9 * cin)))] + norm(cout)
            parts += [normal((cout, 3, 3, cout), np.sqrt(1.0 / (9 * cout)))] + norm(cout)
            if has_down:
                parts += [normal((cout, 1, 1, cin), np.sqrt(1.0 / cin))] + norm(cout)
            meta.append(f"block {cin} {cout} {stride} {has_down}")
        meta.append(f"gn_group_size {s.gn_group_size}")
        with open(os.path.join(out_dir, f"rgb_encoder{e}_backbone.meta"), "w") as f:
            f.write("\n".join(meta) + "\n")
        save(f"rgb_encoder{e}_backbone.bin", parts)
        C, K = s.widths[-1], s.num_keypoints
        save(f"rgb_encoder{e}.bin", [normal((K, C), np.sqrt(1.0 / C)), normal((K,), 0.05),
                                     normal((2 * K, 2 * K), np.sqrt(1.0 / (2 * K))), normal((2 * K,), 0.05)])

    # ---- conditional U-Net, DPUNet1d::load order
    A, D, CD, k = s.action_dim, s.step_embed_dim, s.cond_dim, s.kernel_size
    parts = []

    def lin(n, kk, std=None):
        parts.extend([normal((n, kk), np.sqrt(1.0 / kk) if std is None else std), normal((n,), 0.02)])

    def conv_block(cin, cout):
        lin(cout, k * cin)
        parts.extend(gn(cout))

    def res_block(cin, cout):
        conv_block(cin, cout)
        lin(2 * cout if s.film_scale else cout, CD, 0.5 / np.sqrt(CD))
        conv_block(cout, cout)
        if cin != cout:
            lin(cout, cin)

    lin(4 * D, D)
    lin(D, 4 * D)
    in_out = [(A, s.down_dims[0])] + [(s.down_dims[i], s.down_dims[i + 1]) for i in range(len(s.down_dims) - 1)]
    for i, (ci, co) in enumerate(in_out):
        res_block(ci, co)
        res_block(co, co)
        if i + 1 < len(in_out):
            lin(co, 3 * co)
    mid = s.down_dims[-1]
    res_block(mid, mid)
    res_block(mid, mid)
    for ind in range(len(in_out) - 1):
        dim_out, dim_in = in_out[len(in_out) - 1 - ind]
        res_block(dim_in * 2, dim_out)
        res_block(dim_out, dim_out)
        parts.extend([normal((dim_out, 4, dim_out), np.sqrt(1.0 / (2 * dim_out))), normal((dim_out,), 0.02)])
    conv_block(s.down_dims[0], s.down_dims[0])
    lin(A, s.down_dims[0])
    save("unet.bin", parts)

    # ---- stats: MIN_MAX state / action (non-degenerate), MEAN_STD images
    smin = normal((s.state_dim,), 1.0) - 2.0
    amin = normal((s.action_dim,), 1.0) - 2.0
    stats = [smin, (smin + rng.uniform(1.0, 4.0, s.state_dim)).astype(np.float32),
             amin, (amin + rng.uniform(1.0, 4.0, s.action_dim)).astype(np.float32)]
    for _ in range(s.n_cams):
        stats.append(rng.uniform(0.4, 0.6, 3).astype(np.float32))
        stats.append(rng.uniform(0.2, 0.3, 3).astype(np.float32))
    save("stats.bin", stats)

    meta = [f"n_obs_steps {s.n_obs_steps}", f"n_cams {s.n_cams}", f"img_h {s.img_h}", f"img_w {s.img_w}",
            f"crop_h {s.crop_h}", f"crop_w {s.crop_w}", "resize_h 0", "resize_w 0",
            f"state_dim {s.state_dim}", f"action_dim {s.action_dim}", f"horizon {s.horizon}",
            f"n_action_steps {s.n_action_steps}", f"num_keypoints {s.num_keypoints}",
            f"kernel_size {s.kernel_size}", f"n_groups {s.n_groups}", f"step_embed_dim {s.step_embed_dim}",
            f"film_scale {int(s.film_scale)}", f"separate_encoders {int(s.separate_encoders)}",
            "down_dims " + " ".join(str(d) for d in s.down_dims),
            f"num_train_timesteps {s.num_train_timesteps}", f"num_inference_steps {s.num_inference_steps}",
            "beta_start 0.0001", "beta_end 0.02", f"beta_schedule {s.beta_schedule}", "prediction_type epsilon",
            f"clip_sample {int(s.clip_sample)}", "clip_sample_range 1.0", f"scheduler {s.scheduler}",
            "gn_eps 1e-5"] + [f"cam observation.images.cam{c}" for c in range(s.n_cams)]
    with open(os.path.join(out_dir, "diffusion.meta"), "w") as f:
        f.write("\n".join(meta) + "\n")
    with open(os.path.join(out_dir, "config.txt"), "w") as f:
        f.write("".join(f"cam{c} cam{c}\n" for c in range(s.n_cams)))
    return out_dir


def dp_inputs(shape: DpShape = DP_BASELINE, seed: int = 1, batch: int = 0):
    """Seeded DP query: frames [n_obs_steps * n_cams, H, W, 3] uint8 ~ U{0..255}
    (obs-major, then camera), state [n_obs_steps, state_dim] in the stats' range,
    noise [1 + num_inference_steps, horizon, action_dim] ~ N(0, 1). With batch > 0
    each array gains a leading batch axis."""
    rng = np.random.default_rng(seed)
    s = shape
    lead = (batch,) if batch else ()
    frames = rng.integers(0, 256, size=lead + (s.n_obs_steps * s.n_cams, s.img_h, s.img_w, 3), dtype=np.uint8)
    state = rng.standard_normal(lead + (s.n_obs_steps, s.state_dim), dtype=np.float32)
    noise = rng.standard_normal(lead + (1 + s.num_inference_steps, s.horizon, s.action_dim), dtype=np.float32)
    return frames, state, noise


# ---------------------------------------------------------------------------
# Octo (tools/convert_octo.py's file set; random init)

@dataclasses.dataclass(frozen=True)
class OctoShape:
    d: int = 768
    n_layers: int = 12
    heads: int = 12
    mlp: int = 3072
    max_horizon: int = 10
    n_task: int = 16
    stem_features: tuple = (32, 96, 192, 384)
    stem_dim: int = 512
    gn_groups: int = 32
    t5_dim: int = 768
    t5_layers: int = 12
    t5_heads: int = 12
    t5_ff: int = 3072
    action_dim: int = 7
    horizon: int = 4
    time_dim: int = 32
    num_blocks: int = 3
    hidden: int = 256
    steps: int = 20
    max_action: float = 5.0
    gelu_erf: bool = False
    window: int = 2   # the query window the inputs are drawn for

    def side(self, hw: int) -> int:
        for _ in self.stem_features:
            hw = (hw + 2 - 3) // 2 + 1
        return hw

    @property
    def tok_primary(self) -> int:
        return self.side(256) ** 2

    @property
    def tok_wrist(self) -> int:
        return self.side(128) ** 2

    @property
    def flat(self) -> int:
        return self.action_dim * self.horizon


# Octo-base-shaped (12 layers, d 768, 12 heads, MLP 3072,
# 256 + 64 patch tokens per frame on a 2-frame window, T5-base text tower over
# 16 tokens, 20-step diffusion head, 4 x 7 chunk).
OCTO_BASELINE = OctoShape()
# reduced Octo for fast tests: five stem layers (8 x 8 + 4 x 4 tokens), narrow widths
OCTO_SMALL = OctoShape(d=128, n_layers=3, heads=2, mlp=256, max_horizon=3, stem_features=(16, 16, 32, 32, 32),
                       stem_dim=64, gn_groups=4, t5_dim=64, t5_layers=2, t5_heads=2, t5_ff=128, num_blocks=2,
                       hidden=64)

# the torch-converted form: exact-erf GELU in the MLPs (octo.meta gelu_erf 1)
OCTO_ERF = dataclasses.replace(OCTO_SMALL, gelu_erf=True)

# A synthetic unigram vocabulary: the control pieces, every letter and digit
# alone and after the word marker, and a few hundred made-up words.
_SYLLABLES = ["pi", "ck", "up", "the", "red", "blo", "put", "in", "bo", "wl", "dra", "wer", "op", "en", "clo",
              "se", "gr", "ab", "mu", "g", "sp", "oon", "tow", "el", "left", "righ", "t", "ca", "bi", "net"]


def octo_vocab(seed: int = 7):
    """[(piece, score)] of a synthetic vocab.txt; ids are list positions."""
    rng = np.random.default_rng(seed)
    mark = "▁"
    pieces = [("<pad>", 0.0), ("</s>", 0.0), ("<unk>", 0.0)]
    seen = {p for p, _ in pieces}

    def add(p, sc):
        if p not in seen:
            seen.add(p)
            pieces.append((p, sc))

    add(mark, -3.0)
    for ch in "abcdefghijklmnopqrstuvwxyz0123456789.,!?'-":
        add(ch, -8.0 - float(rng.uniform(0, 2)))
        add(mark + ch, -9.0 - float(rng.uniform(0, 2)))
    for _ in range(400):
        w = "".join(rng.choice(_SYLLABLES, size=int(rng.integers(1, 4))))
        add((mark + w) if rng.uniform() < 0.7 else w, -float(rng.uniform(4.0, 12.0)))
    add("<extra_id_0>", 0.0)
    add("unused_placeholder", 0.0)   # score 0 and not <...>: keeps its id, never matched
    return pieces


def octo_instruction(seed: int, n_words: int = 8) -> str:
    rng = np.random.default_rng(seed)
    words = ["".join(rng.choice(_SYLLABLES, size=int(rng.integers(1, 4)))) for _ in range(n_words)]
    return " ".join(words)


def write_octo_checkpoint(out_dir: str, shape: OctoShape = OCTO_BASELINE, seed: int = 0) -> str:
    """Write a random-init Octo checkpoint directory with its tokenizer in
    out_dir/tok; returns out_dir."""
    os.makedirs(os.path.join(out_dir, "tok"), exist_ok=True)
    rng = np.random.default_rng(seed)
    s = shape

    def normal(shape_, std):
        return (rng.standard_normal(shape_, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def save(name, parts):
        np.concatenate([np.asarray(p, np.float32).reshape(-1) for p in parts]).astype(np.float32).tofile(
            os.path.join(out_dir, name))

    def scale_bias(c):
        return [(1.0 + normal((c,), 0.05)).astype(np.float32), normal((c,), 0.05)]

    vocab = octo_vocab()
    with open(os.path.join(out_dir, "tok", "vocab.txt"), "w", encoding="utf-8") as f:
        for p, sc in vocab:
            f.write(f"{p}\t{sc!r}\n")

    # T5 encoder: embedding, relative bias [32][heads], per layer ln1 q k v o ln2 wi wo, final ln
    D5, hd5 = s.t5_dim, s.t5_dim // s.t5_heads
    parts = [normal((len(vocab), D5), 1.0), normal((32, s.t5_heads), 0.5)]
    for _ in range(s.t5_layers):
        parts += [1.0 + normal((D5,), 0.05)]
        parts += [normal((D5, D5), 1.0 / np.sqrt(D5 * hd5))]          # q (T5 folds 1/sqrt(d_kv) in)
        parts += [normal((D5, D5), 1.0 / np.sqrt(D5)) for _ in range(3)]
        parts += [1.0 + normal((D5,), 0.05), normal((s.t5_ff, D5), 1.0 / np.sqrt(D5)),
                  normal((D5, s.t5_ff), 1.0 / np.sqrt(s.t5_ff))]
    parts += [1.0 + normal((D5,), 0.05)]
    save("t5.bin", parts)
    with open(os.path.join(out_dir, "t5.meta"), "w") as f:
        f.write(f"d_model {D5}\nn_layers {s.t5_layers}\nn_heads {s.t5_heads}\nd_kv {hd5}\nd_ff {s.t5_ff}\n"
                f"vocab {len(vocab)}\nn_buckets 32\nmax_dist 128\neps 1e-6\nn_tokens {s.n_task}\n")

    # SmallStems: per layer conv w [Cout][3][3][Cin], b, GroupNorm scale, bias; embed
    for name in ("stem_primary", "stem_wrist"):
        parts = []
        cin = 6
        for cout in s.stem_features:
            parts += [normal((cout, 3, 3, cin), np.sqrt(2.0 / (9 * cin))), normal((cout,), 0.05)] + scale_bias(cout)
            cin = cout
        parts += [normal((s.stem_dim, cin), np.sqrt(1.0 / cin)), normal((s.stem_dim,), 0.02)]
        save(f"{name}.bin", parts)
        with open(os.path.join(out_dir, f"{name}.meta"), "w") as f:
            f.write(f"in_ch 6\nn_layers {len(s.stem_features)}\nk 3\nstride 2\npad 1\n"
                    "features " + " ".join(str(c) for c in s.stem_features) + "\n"
                    f"embed_dim {s.stem_dim}\ngn_groups {s.gn_groups}\ngn_eps 1e-6\n")

    # transformer: projections, position embeddings, blocks, final LayerNorm
    D = s.d
    parts = []

    def lin(n, k, std=None):
        parts.extend([normal((n, k), np.sqrt(1.0 / k) if std is None else std), normal((n,), 0.02)])

    lin(D, s.t5_dim)
    lin(D, s.stem_dim)
    lin(D, s.stem_dim)
    parts += [normal((s.n_task, D), 0.5), normal((s.max_horizon, s.tok_primary, D), 0.5),
              normal((s.max_horizon, s.tok_wrist, D), 0.5), normal((s.max_horizon, 1, D), 0.5)]
    for _ in range(s.n_layers):
        parts += scale_bias(D)
        for _ in range(4):
            lin(D, D)
        parts += scale_bias(D)
        lin(s.mlp, D)
        lin(D, s.mlp, 0.5 / np.sqrt(s.mlp))
    parts += scale_bias(D)
    save("octo.bin", parts)
    with open(os.path.join(out_dir, "octo.meta"), "w") as f:
        f.write(f"d {D}\nn_layers {s.n_layers}\nheads {s.heads}\nhead_dim {D // s.heads}\nmlp {s.mlp}\n"
                f"max_horizon {s.max_horizon}\nn_task {s.n_task}\ntok_primary {s.tok_primary}\n"
                f"tok_wrist {s.tok_wrist}\nn_readout 1\nt5_dim {s.t5_dim}\nstem_dim {s.stem_dim}\nln_eps 1e-6\n"
                f"window {s.window}\ngelu_erf {int(s.gelu_erf)}\n")

    # diffusion head: Fourier weights, cond MLP, score net, beta schedule
    TD, H, FL = s.time_dim, s.hidden, s.flat
    parts = [normal((TD // 2,), 0.2)]
    lin(2 * TD, TD)
    lin(TD, 2 * TD)
    lin(H, TD + D + FL)
    for _ in range(s.num_blocks):
        parts += scale_bias(H)
        lin(4 * H, H)
        lin(H, 4 * H, 0.5 / np.sqrt(4 * H))
    lin(FL, H)
    # linear betas: a random-init score net would drive a cosine schedule's
    # first steps into the +-max_action clamp and leave nothing to compare
    betas = np.linspace(1e-4, 0.02, s.steps).astype(np.float32)
    alphas = (1.0 - betas).astype(np.float32)
    parts += [betas, alphas, np.cumprod(alphas).astype(np.float32)]
    save("head.bin", parts)
    with open(os.path.join(out_dir, "head.meta"), "w") as f:
        f.write(f"emb {D}\naction_dim {s.action_dim}\nhorizon {s.horizon}\ntime_dim {TD}\n"
                f"num_blocks {s.num_blocks}\nhidden {H}\nsteps {s.steps}\nmax_action {s.max_action!r}\n")

    A = s.action_dim
    normal((A,), 0.1).tofile(os.path.join(out_dir, "stats_action_mean.bin"))
    rng.uniform(0.5, 1.5, A).astype(np.float32).tofile(os.path.join(out_dir, "stats_action_std.bin"))
    np.array([1.0] * (A - 1) + [0.0], np.float32).tofile(os.path.join(out_dir, "stats_action_mask.bin"))
    return out_dir


def octo_inputs(shape: OctoShape = OCTO_BASELINE, seed: int = 1, batch: int = 0, wnd: int = 0):
    """Seeded Octo query: primary [wnd, 256, 256, 3] and wrist [wnd, 128, 128, 3]
    uint8 ~ U{0..255}, timestep mask [wnd] (all real), instruction string,
    noise [flat] and z [steps, flat] ~ N(0, 1). With batch > 0 the arrays gain
    a leading batch axis and the instruction becomes a list."""
    rng = np.random.default_rng(seed)
    s = shape
    w = wnd or s.window
    lead = (batch,) if batch else ()
    primary = rng.integers(0, 256, size=lead + (w, 256, 256, 3), dtype=np.uint8)
    wrist = rng.integers(0, 256, size=lead + (w, 128, 128, 3), dtype=np.uint8)
    tmask = np.ones(lead + (w,), np.uint8)
    noise = rng.standard_normal(lead + (s.flat,), dtype=np.float32)
    z = rng.standard_normal(lead + (s.steps, s.flat), dtype=np.float32)
    instr = [octo_instruction(seed * 131 + b) for b in range(batch)] if batch else octo_instruction(seed * 131)
    return primary, wrist, tmask, instr, noise, z


# ---------------------------------------------------------------------------
# SmolVLA (tools/convert_hf_safetensors.py's file set; random init, bf16 towers)

@dataclasses.dataclass(frozen=True)
class SmolvlaShape:
    vit_hidden: int = 768
    vit_heads: int = 12
    vit_inter: int = 3072
    vit_layers: int = 12
    patch: int = 16
    img: int = 512
    scale_factor: int = 4
    hidden: int = 960          # LM width (= the connector's output)
    n_q: int = 15
    n_kv: int = 5
    ffn: int = 2560
    vlm_layers: int = 16
    expert_h: int = 720
    expert_ffn: int = 1920
    expert_layers: int = 16
    self_attn_every_n: int = 2
    chunk: int = 50
    num_steps: int = 10
    max_action_dim: int = 32
    max_state_dim: int = 32
    state_dim: int = 6
    action_dim: int = 6
    n_views: int = 2
    tok_maxlen: int = 48
    frame_h: int = 480         # the native camera frames the inputs are drawn at
    frame_w: int = 640

    @property
    def n_patches(self) -> int:
        return (self.img // self.patch) ** 2

    @property
    def n_img_tok(self) -> int:
        return self.n_patches // (self.scale_factor ** 2)


# SmolVLA-shaped (SigLIP 12 layers d768 at 512 px -> 64 tokens
# per view after the pixel shuffle, 2 views; SmolLM2 16 layers h960, 15 / 5
# heads of 64, FFN 2560; 48 prompt tokens + state; expert 16 layers h720; 10
# Euler steps; 50 x 6 chunk).
SMOLVLA_BASELINE = SmolvlaShape()
# reduced SmolVLA for fast tests (same code paths; every int8-eligible width a multiple of 16)
SMOLVLA_SMALL = SmolvlaShape(vit_hidden=128, vit_heads=2, vit_inter=256, vit_layers=2, img=128, scale_factor=2,
                             hidden=128, n_q=2, n_kv=1, ffn=256, vlm_layers=3, expert_h=96, expert_ffn=192,
                             expert_layers=3, chunk=10, num_steps=4, max_action_dim=8, max_state_dim=8,
                             state_dim=5, action_dim=4, tok_maxlen=12, frame_h=96, frame_w=120)


# edge cases of the same code paths: one view from small wide frames, a prompt
# shorter than tok_maxlen (padded tokens masked out of the prefix), an expert
# shallower than the text tower with self-attention every third layer, a
# 7-step chunk and 3 flow steps
SMOLVLA_EDGE = SmolvlaShape(vit_hidden=128, vit_heads=2, vit_inter=256, vit_layers=1, img=64, scale_factor=2,
                            hidden=128, n_q=2, n_kv=1, ffn=256, vlm_layers=4, expert_h=64, expert_ffn=128,
                            expert_layers=3, self_attn_every_n=3, chunk=7, num_steps=3, max_action_dim=8,
                            max_state_dim=8, state_dim=3, action_dim=2, n_views=1, tok_maxlen=20, frame_h=50,
                            frame_w=100)


def _gpt2_byte_chars():
    """The byte-level BPE alphabet: printable Latin-1 bytes map to themselves,
    the other 68 bytes to code points 256.. in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    table, extra = {}, 0
    for b in range(256):
        if b in keep:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


def smolvla_tokenizer_files(out_dir: str, n_merges: int = 120, seed: int = 5):
    """A synthetic byte-level BPE tokenizer (vocab.txt "id<TAB>token", merges.txt
    "a b") learned on the synthetic instruction corpus; returns the vocab size."""
    bc = _gpt2_byte_chars()
    corpus = [octo_instruction(seed * 1000 + i) for i in range(200)]
    words = collections.Counter()
    for line in corpus:
        for i, w in enumerate(line.split(" ")):
            words[tuple(bc[b] for b in ((" " if i else "") + w).encode())] += 1
    merges = []
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        best = max(sorted(pairs), key=lambda p: pairs[p])
        merges.append(best)
        new = collections.Counter()
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and (w[i], w[i + 1]) == best:
                    out.append(w[i] + w[i + 1])
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            new[tuple(out)] += c
        words = new
    vocab = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"] + [bc[b] for b in range(256)] + [a + b for a, b in merges]
    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "vocab.txt"), "w", encoding="utf-8") as f:
        for i, t in enumerate(vocab):
            f.write(f"{i}\t{t}\n")
    with open(os.path.join(out_dir, "merges.txt"), "w", encoding="utf-8") as f:
        for a, b in merges:
            f.write(f"{a} {b}\n")
    return len(vocab)


def _bf16(a):
    """Round fp32 to bf16 (nearest even), as uint16."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def write_smolvla_checkpoint(out_dir: str, shape: SmolvlaShape = SMOLVLA_BASELINE, seed: int = 0) -> str:
    """Write a random-init SmolVLA checkpoint directory (tokenizer in out_dir/tok); returns out_dir."""
    os.makedirs(out_dir, exist_ok=True)
    rng = np.random.default_rng(seed)
    s = shape

    def normal(shape_, std):
        return (rng.standard_normal(shape_, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def norm_w(c):
        return (1.0 + normal((c,), 0.05)).astype(np.float32)

    vocab = smolvla_tokenizer_files(os.path.join(out_dir, "tok"))

    # vision: fp32 region, then the bf16 region
    H, I, P = s.vit_hidden, s.vit_inter, 3 * s.patch * s.patch
    SD = H * s.scale_factor ** 2
    f32 = [normal((H,), 0.02), normal((s.n_patches, H), 0.5)]
    for _ in range(s.vit_layers):
        f32 += [norm_w(H), normal((H,), 0.02)] + [normal((H,), 0.02) for _ in range(4)]
        f32 += [norm_w(H), normal((H,), 0.02), normal((I,), 0.02), normal((H,), 0.02)]
    f32 += [norm_w(H), normal((H,), 0.02)]
    w = [normal((H, P), 1.0 / np.sqrt(P))]
    for _ in range(s.vit_layers):
        w += [normal((H, H), 1.0 / np.sqrt(H)) for _ in range(4)]
        w += [normal((I, H), 1.0 / np.sqrt(H)), normal((H, I), 0.5 / np.sqrt(I))]
    w += [normal((s.hidden, SD), 1.0 / np.sqrt(SD))]
    with open(os.path.join(out_dir, "vit.bin"), "wb") as f:
        np.concatenate([a.reshape(-1) for a in f32]).astype(np.float32).tofile(f)
        _bf16(np.concatenate([a.reshape(-1) for a in w])).tofile(f)
    with open(os.path.join(out_dir, "vit.meta"), "w") as f:
        f.write(f"hidden {H}\nn_heads {s.vit_heads}\nhead_dim {H // s.vit_heads}\ninter {I}\n"
                f"n_layers {s.vit_layers}\npatch {s.patch}\nimg {s.img}\nn_patches {s.n_patches}\n"
                f"ln_eps 1e-06\nscale_factor {s.scale_factor}\nmm_out {s.hidden}\nn_img_tok {s.n_img_tok}\n")

    # VLM text tower: per-layer norms + the output norm, then bf16 q k v o gate up down
    D, QF, KV, F = s.hidden, s.n_q * 64, s.n_kv * 64, s.ffn
    f32 = []
    for _ in range(s.vlm_layers):
        f32 += [norm_w(D), norm_w(D)]
    f32 += [norm_w(D)]
    w = []
    for _ in range(s.vlm_layers):
        w += [normal((QF, D), 1.0 / np.sqrt(D)), normal((KV, D), 1.0 / np.sqrt(D)), normal((KV, D), 1.0 / np.sqrt(D)),
              normal((D, QF), 0.5 / np.sqrt(QF)), normal((F, D), 1.0 / np.sqrt(D)), normal((F, D), 1.0 / np.sqrt(D)),
              normal((D, F), 0.5 / np.sqrt(F))]
    with open(os.path.join(out_dir, "vlm.bin"), "wb") as f:
        np.concatenate([a.reshape(-1) for a in f32]).astype(np.float32).tofile(f)
        _bf16(np.concatenate([a.reshape(-1) for a in w])).tofile(f)
    with open(os.path.join(out_dir, "vlm.meta"), "w") as f:
        f.write(f"hidden {D}\nn_q {s.n_q}\nn_kv {s.n_kv}\nhead_dim 64\nffn {F}\neps 1e-05\nrope_base 10000\n"
                f"n_layers {s.vlm_layers}\n")

    # action expert (fp32): per layer ln_in q k v o ln_post gate up down; out norm; flow projections
    EH, EF, MAD = s.expert_h, s.expert_ffn, s.max_action_dim
    parts = []
    for L in range(s.expert_layers):
        self_attn = s.self_attn_every_n > 0 and L % s.self_attn_every_n == 0
        kk = EH if self_attn else KV
        parts += [norm_w(EH), normal((QF, EH), 1.0 / np.sqrt(EH)), normal((KV, kk), 1.0 / np.sqrt(kk)),
                  normal((KV, kk), 1.0 / np.sqrt(kk)), normal((EH, QF), 0.5 / np.sqrt(QF)), norm_w(EH),
                  normal((EF, EH), 1.0 / np.sqrt(EH)), normal((EF, EH), 1.0 / np.sqrt(EH)),
                  normal((EH, EF), 0.5 / np.sqrt(EF))]
    parts += [norm_w(EH), normal((EH, MAD), 1.0 / np.sqrt(MAD)), normal((EH,), 0.02),
              normal((EH, 2 * EH), 1.0 / np.sqrt(2 * EH)), normal((EH,), 0.02), normal((EH, EH), 1.0 / np.sqrt(EH)),
              normal((EH,), 0.02), normal((MAD, EH), 0.3 / np.sqrt(EH)), normal((MAD,), 0.02)]
    np.concatenate([a.reshape(-1) for a in parts]).astype(np.float32).tofile(os.path.join(out_dir, "aex.bin"))
    with open(os.path.join(out_dir, "aex.meta"), "w") as f:
        f.write(f"expert_h {EH}\nexpert_ffn {EF}\nn_q {s.n_q}\nn_kv {s.n_kv}\nhead_dim 64\neps 1e-05\n"
                f"rope_base 10000\nn_layers {s.expert_layers}\nself_attn_every_n {s.self_attn_every_n}\n"
                f"chunk {s.chunk}\nnum_steps {s.num_steps}\nmax_action_dim {MAD}\nmin_period 0.004\n"
                f"max_period 4.0\n")

    # token embeddings (bf16), state projection, stats
    _bf16(normal((vocab, D), 1.0 / np.sqrt(D))).tofile(os.path.join(out_dir, "emb.bin"))
    np.concatenate([normal((D, s.max_state_dim), 1.0 / np.sqrt(s.max_state_dim)).reshape(-1),
                    normal((D,), 0.02)]).tofile(os.path.join(out_dir, "heads.bin"))
    with open(os.path.join(out_dir, "heads.meta"), "w") as f:
        f.write(f"vocab {vocab}\nhidden {D}\nmax_state_dim {s.max_state_dim}\nreal_state_dim {s.state_dim}\n"
                f"real_action_dim {s.action_dim}\nn_views {s.n_views}\n")
    normal((s.state_dim,), 1.0).tofile(os.path.join(out_dir, "stats_state_mean.bin"))
    rng.uniform(0.5, 2.0, s.state_dim).astype(np.float32).tofile(os.path.join(out_dir, "stats_state_std.bin"))
    normal((s.action_dim,), 1.0).tofile(os.path.join(out_dir, "stats_action_mean.bin"))
    rng.uniform(0.5, 2.0, s.action_dim).astype(np.float32).tofile(os.path.join(out_dir, "stats_action_std.bin"))
    with open(os.path.join(out_dir, "config.txt"), "w") as f:
        f.write(f"instruction {octo_instruction(1)}\ntokenizer_max_length {s.tok_maxlen}\npad_token_id 2\n"
                f"chunk {s.chunk}\nnum_steps {s.num_steps}\nn_views {s.n_views}\n")
    return out_dir


def smolvla_inputs(shape: SmolvlaShape = SMOLVLA_BASELINE, seed: int = 1, batch: int = 0):
    """Seeded SmolVLA query: frames [n_views, frame_h, frame_w, 3] uint8, an
    instruction string, raw state [state_dim] ~ N(0, 1), noise [chunk,
    max_action_dim] ~ N(0, 1). With batch > 0 the arrays gain a leading batch
    axis and the instruction becomes a list."""
    rng = np.random.default_rng(seed)
    s = shape
    lead = (batch,) if batch else ()
    frames = rng.integers(0, 256, size=lead + (s.n_views, s.frame_h, s.frame_w, 3), dtype=np.uint8)
    state = rng.standard_normal(lead + (s.state_dim,), dtype=np.float32)
    noise = rng.standard_normal(lead + (s.chunk, s.max_action_dim), dtype=np.float32)
    instr = [octo_instruction(seed * 17 + b) for b in range(batch)] if batch else octo_instruction(seed * 17)
    return frames, instr, state, noise


# ---------------------------------------------------------------------------
# vla.simd GGUF packing of a converted directory (the container the reference's
# converters write by default; read back by src/io/gguf_vla_simd.cpp): GGUF v3,
# key/value "general.architecture" = "vla-simd", "vla_simd.format" = 1, every
# text file as the string "vla_simd.file.<name>", every .bin as one F32 tensor
# named by the file, data aligned to 32 bytes.

def _gguf_str(s: bytes) -> bytes:
    import struct
    return struct.pack("<Q", len(s)) + s


def pack_gguf(model_dir: str, out_path: str, model: str) -> str:
    """Pack the files of a converted directory into one vla.simd GGUF at out_path."""
    import struct
    align = 32
    names = sorted(os.listdir(model_dir))
    kv = [("general.architecture", 8, b"vla-simd"), ("general.name", 8, os.path.basename(out_path).encode()),
          ("vla_simd.model", 8, model.encode()), ("vla_simd.format", 4, 1), ("vla_simd.source", 8, b"")]
    bins = []
    for n in names:
        path = os.path.join(model_dir, n)
        if not os.path.isfile(path):
            continue
        size = os.path.getsize(path)
        if n.endswith(".bin") and size:
            if size % 4:
                raise ValueError(f"{n}: not a whole number of floats")
            bins.append((n, path, size))
        else:
            kv.append((f"vla_simd.file.{n}", 8, open(path, "rb").read()))
    head = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(bins), len(kv)))
    for key, ty, val in kv:
        head += _gguf_str(key.encode()) + struct.pack("<I", ty)
        head += _gguf_str(val) if ty == 8 else struct.pack("<I", val)
    offsets, off = [], 0
    for n, _, size in bins:
        off = (off + align - 1) // align * align
        offsets.append(off)
        head += _gguf_str(n.encode()) + struct.pack("<IQIQ", 1, size // 4, 0, off)   # 1-D F32
        off += size
    with open(out_path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (-len(head) % align))
        base = f.tell()
        for (_, path, _), o in zip(bins, offsets):
            f.write(b"\0" * (base + o - f.tell()))
            with open(path, "rb") as src:
                f.write(src.read())
    return out_path
