"""Octo on the B200 (the T5 language tower once per instruction, then one CUDA
graph: both SmallStems, the block-causal ViT with a readout-only last layer,
20 DDPM steps of the diffusion head) against the reference's own
vla_octo_predict_ex on the same synthetic checkpoint, frames, instruction and
noise (committed fixtures from tests/golden/make_golden.py). Tolerance: the
north star's action-chunk max-abs 1e-3; the readout embedding (the head's
input) to 1e-5 (LayerNorm's rare double -> float ties)."""
import os

import numpy as np
import pytest

from vla_simd_b200 import synth

from _parity import check_actions

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3

import sys
sys.path.insert(0, GOLDEN)
from make_golden import octo_query  # noqa: E402  (the fixture cases' inputs)


def _policy(tmp_path, shape, mask, monkeypatch, max_batch=1, graph=True, name=None):
    from vla_simd_b200 import OctoPolicy
    monkeypatch.setenv("OCTO_INT8", str(mask))
    monkeypatch.setenv("VLA_CUDA_GRAPH", "1" if graph else "0")
    d = synth.write_octo_checkpoint(str(tmp_path / (name or f"octo{mask}")), shape, seed=0)
    return OctoPolicy(d, max_batch=max_batch)


def _want(cfg, mask, variant=""):
    return np.load(os.path.join(GOLDEN, f"octo_{cfg}_m{mask}" + (f"_{variant}" if variant else "") + ".npy"))


@pytest.mark.parametrize("mask,n_int8", [(63, 38), (0, 0), (31, 33)])
def test_small_octo_matches_reference(tmp_path, monkeypatch, mask, n_int8):
    pol = _policy(tmp_path, synth.OCTO_SMALL, mask, monkeypatch)
    assert pol.int8_layers == n_int8   # the reference's count on this checkpoint
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_SMALL, "")
    got = pol.predict(p, w, tm, ins, n, z)
    check_actions(f"octo-small-m{mask}", got, _want("small", mask), TOL)
    pol.close()


def test_erf_gelu_octo_matches_reference(tmp_path, monkeypatch):
    """The torch-converted form (octo.meta gelu_erf 1: exact-erf GELU in every MLP)."""
    pol = _policy(tmp_path, synth.OCTO_ERF, 63, monkeypatch)
    assert pol.int8_layers == 38
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_ERF, "")
    check_actions("octo-erf-m63", pol.predict(p, w, tm, ins, n, z), _want("erf", 63), TOL)
    pol.close()


def test_small_octo_readout_matches_reference(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch)
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_SMALL, "")
    pol.predict(p, w, tm, ins, n, z)
    check_actions("octo-small-m63-readout", pol.readout()[0], _want("small", 63, "readout"), 1e-5)
    pol.close()


@pytest.mark.parametrize("variant", ["nowrist", "pad", "w1", "seed"])
def test_small_octo_variants_match_reference(tmp_path, monkeypatch, variant):
    pol = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch)
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_SMALL, variant)
    got = pol.predict(p, w, tm, ins, n, z, seed=seed)
    check_actions(f"octo-small-m63-{variant}", got, _want("small", 63, variant), TOL)
    pol.close()


def test_baseline_octo_matches_reference(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.OCTO_BASELINE, 63, monkeypatch)
    assert pol.int8_layers == 92
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_BASELINE, "")
    got = pol.predict(p, w, tm, ins, n, z)
    check_actions("octo-base-m63", got, _want("base", 63), TOL)
    assert np.array_equal(got, pol.predict(p, w, tm, ins, n, z)), "query is not deterministic"
    assert pol.t5_runs == 2   # the warm-up's empty instruction, then this one once
    assert pol.kernels_per_step > 100
    pol.close()


def test_octo_batch_equals_single_queries(tmp_path, monkeypatch):
    B = 3
    pol = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch, max_batch=4)
    p, w, tm, ins, n, z = synth.octo_inputs(synth.OCTO_SMALL, seed=5, batch=B, wnd=2)
    tm[1] = [0, 1]
    got = pol.predict_batch(p, w, tm, ins, n, z)
    for b in range(B):
        assert np.array_equal(got[b], pol.predict(p[b], w[b], tm[b], ins[b], n[b], z[b])), b
    pol.close()


def test_octo_graph_equals_eager(tmp_path, monkeypatch):
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_SMALL, "")
    a = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch, graph=True, name="g")
    ga = a.predict(p, w, tm, ins, n, z)
    a.close()
    b = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch, graph=False, name="e")
    gb = b.predict(p, w, tm, ins, n, z)
    b.close()
    assert np.array_equal(ga, gb)


def test_octo_refuses_bad_shapes(tmp_path, monkeypatch):
    from vla_simd_b200 import VlaError
    pol = _policy(tmp_path, synth.OCTO_SMALL, 63, monkeypatch, max_batch=2)
    p, w, tm, ins, n, z = synth.octo_inputs(synth.OCTO_SMALL, seed=5, wnd=4)   # max_window is 3
    with pytest.raises(VlaError) as e:
        pol.predict(p, w, tm, ins, n, z)
    assert e.value.code == -2
    p, w, tm, ins, n, z = synth.octo_inputs(synth.OCTO_SMALL, seed=5, batch=3)
    with pytest.raises(VlaError) as e:
        pol.predict_batch(p, w, tm, ins, n, z)
    assert e.value.code == -2
    pol.close()
