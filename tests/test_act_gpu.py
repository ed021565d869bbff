"""The whole ACT policy step on the B200 (one CUDA graph) against the
reference's own vla_act_predict on the same synthetic checkpoint and inputs
(committed fixtures from tests/golden/make_golden.py). Tolerance: the north
star's action-chunk max-abs 1e-3."""
import os

import numpy as np
import pytest

from vla_simd_b200 import synth

from _parity import check_actions

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3


def _policy(tmp_path, shape, mask, monkeypatch, graph=True):
    from vla_simd_b200 import ActPolicy
    monkeypatch.setenv("ACT_INT8", str(mask))
    monkeypatch.setenv("VLA_CUDA_GRAPH", "1" if graph else "0")
    d = synth.write_act_checkpoint(str(tmp_path / f"ck{mask}"), shape, seed=0)
    return ActPolicy(d)


@pytest.mark.parametrize("mask", [63, 0, 31, 40])
def test_small_act_matches_reference(tmp_path, monkeypatch, mask):
    pol = _policy(tmp_path, synth.ACT_SMALL, mask, monkeypatch)
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    got = pol.predict(f, s)
    want = np.load(os.path.join(GOLDEN, f"act_small_m{mask}.npy"))
    check_actions(f"act-small-m{mask}", got, want, TOL)
    pol.close()


def test_baseline_act_matches_reference(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.ACT_BASELINE, 63, monkeypatch)
    assert pol.int8_layers == 30 + 20   # transformer GEMMs (wq;wk stacked) + backbone convs
    f, s = synth.act_inputs(synth.ACT_BASELINE, seed=1)
    got = pol.predict(f, s)
    want = np.load(os.path.join(GOLDEN, "act_base_m63.npy"))
    check_actions("act-base-m63", got, want, TOL)
    again = pol.predict(f, s)
    assert np.array_equal(got, again), "step is not deterministic"
    assert pol.kernels_per_step > 50
    pol.close()


def test_graph_equals_eager(tmp_path, monkeypatch):
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    a = _policy(tmp_path, synth.ACT_SMALL, 63, monkeypatch, graph=True)
    ga = a.predict(f, s)
    a.close()
    b = _policy(tmp_path, synth.ACT_SMALL, 63, monkeypatch, graph=False)
    gb = b.predict(f, s)
    b.close()
    assert np.array_equal(ga, gb)


@pytest.mark.parametrize("shape", ["small", "baseline"])
def test_conv_forms_are_bit_identical(tmp_path, monkeypatch, shape):
    """Implicit-GEMM convs and the space-to-depth stem (stride-2 7x7 over 3
    channels as 4x1 taps over 64 channels) give the explicit im2col + GEMM
    path's bits for the whole step."""
    sh = synth.ACT_SMALL if shape == "small" else synth.ACT_BASELINE
    f, s = synth.act_inputs(sh, seed=1)
    monkeypatch.setenv("VLA_CONV_IM2COL", "1")
    a = _policy(tmp_path, sh, 63, monkeypatch)
    want = a.predict(f, s)
    a.close()
    monkeypatch.delenv("VLA_CONV_IM2COL")
    b = _policy(tmp_path, sh, 63, monkeypatch)
    got = b.predict(f, s)
    b.close()
    assert np.array_equal(got, want)


def test_unnormalize_flag(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.ACT_SMALL, 63, monkeypatch)
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    raw = pol.predict(f, s, unnormalize=False)
    real = pol.predict(f, s, unnormalize=True)
    st = np.fromfile(os.path.join(str(tmp_path / "ck63"), "stats.bin"), np.float32)
    sd, ad = synth.ACT_SMALL.state_dim, synth.ACT_SMALL.action_dim
    mean, std = st[2 * sd:2 * sd + ad], st[2 * sd + ad:2 * sd + 2 * ad]
    assert np.abs(real - (raw * std + mean)).max() <= 1e-5
    pol.close()


def test_bad_inputs_rejected(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.ACT_SMALL, 63, monkeypatch)
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    with pytest.raises(ValueError):
        pol.predict(f[:1], s)
    with pytest.raises(ValueError):
        pol.predict(f, s[:3])
    pol.close()
