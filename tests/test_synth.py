"""The synthetic checkpoint writer: deterministic, and in exactly the format
the reference's own loader accepts (src/models/act/act_model.cpp:22-104)."""
import hashlib
import os

import numpy as np

from vla_simd_b200 import synth


def _digest(d):
    h = hashlib.sha256()
    for name in sorted(os.listdir(d)):
        h.update(name.encode())
        h.update(open(os.path.join(d, name), "rb").read())
    return h.hexdigest()


def test_writer_is_deterministic(tmp_path):
    a = synth.write_act_checkpoint(str(tmp_path / "a"), synth.ACT_SMALL, seed=5)
    b = synth.write_act_checkpoint(str(tmp_path / "b"), synth.ACT_SMALL, seed=5)
    assert _digest(a) == _digest(b)
    c = synth.write_act_checkpoint(str(tmp_path / "c"), synth.ACT_SMALL, seed=6)
    assert _digest(a) != _digest(c)


def test_baseline_shape_sizes(tmp_path):
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_BASELINE, seed=0)
    # ResNet-18: 11.2M conv params (+ biases); DETR part: img_proj, 4 enc, 1 dec, head
    n_bb = os.path.getsize(os.path.join(d, "backbone.bin")) // 4
    assert 11_000_000 < n_bb < 11_300_000
    meta = open(os.path.join(d, "backbone.meta")).read().split("\n")
    assert sum(1 for l in meta if l.startswith("block")) == 8
    frames, state = synth.act_inputs(synth.ACT_BASELINE)
    assert frames.shape == (2, 480, 640, 3) and frames.dtype == np.uint8 and state.shape == (6,)


def test_reference_loads_and_runs_synthetic_checkpoint(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("ACT_INT8", "63")
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    frames, state = synth.act_inputs(synth.ACT_SMALL, seed=1)
    a = reference.act_predict(d, frames, state)
    assert a.shape == (synth.ACT_SMALL.chunk, synth.ACT_SMALL.action_dim) and np.isfinite(a).all()


def test_dp_writer_is_deterministic(tmp_path):
    a = synth.write_dp_checkpoint(str(tmp_path / "a"), synth.DP_SMALL, seed=5)
    b = synth.write_dp_checkpoint(str(tmp_path / "b"), synth.DP_SMALL, seed=5)
    assert _digest(a) == _digest(b)


def test_dp_baseline_shape_sizes(tmp_path):
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_BASELINE, seed=0)
    # conditional U-Net (512, 1024, 2048), kernel 5: ~256M parameters
    n_unet = os.path.getsize(os.path.join(d, "unet.bin")) // 4
    assert 240_000_000 < n_unet < 270_000_000
    assert synth.DP_BASELINE.cond_dim == 128 + (2 + 64) * 2
    frames, state, noise = synth.dp_inputs(synth.DP_BASELINE)
    assert frames.shape == (2, 96, 96, 3) and state.shape == (2, 2) and noise.shape == (11, 16, 2)
    fb, sb, nb = synth.dp_inputs(synth.DP_SMALL, batch=3)
    assert fb.shape[0] == sb.shape[0] == nb.shape[0] == 3


def test_reference_runs_synthetic_dp_checkpoint(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("DIFFUSION_INT8", "3")
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_SMALL, seed=0)
    frames, state, noise = synth.dp_inputs(synth.DP_SMALL, seed=1)
    a = reference.dp_predict(d, frames, state, noise)
    assert a.shape == (synth.DP_SMALL.n_action_steps, synth.DP_SMALL.action_dim) and np.isfinite(a).all()
