"""SmolVLA on the B200 (one CUDA graph: resize-with-pad, the SigLIP tower and
connector, the SmolLM2 prefix pass, the action expert's flow-matching loop)
against the reference's own vla_smolvla_predict_rtc on the same synthetic
checkpoint, frames, instruction, state and noise (committed fixtures from
tests/golden/make_golden.py). Tolerance: the north star's action-chunk
max-abs 1e-3."""
import os
import sys

import numpy as np
import pytest

from vla_simd_b200 import synth

from _parity import check_actions

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
TOL = 1e-3
sys.path.insert(0, GOLDEN)
from make_golden import smolvla_query  # noqa: E402  (the fixture cases' inputs)


def _policy(tmp_path, shape, mask, monkeypatch, max_batch=1, graph=True, name=None):
    from vla_simd_b200 import SmolvlaPolicy
    monkeypatch.setenv("SMOLVLA_INT8", str(mask))
    monkeypatch.setenv("VLA_CUDA_GRAPH", "1" if graph else "0")
    d = synth.write_smolvla_checkpoint(str(tmp_path / (name or f"smol{mask}")), shape, seed=0)
    return SmolvlaPolicy(d, max_batch=max_batch)


def _want(cfg, mask, variant=""):
    return np.load(os.path.join(GOLDEN, f"smolvla_{cfg}_m{mask}" + (f"_{variant}" if variant else "") + ".npy"))


@pytest.mark.parametrize("mask,n_int8,variant", [(63, 56, ""), (0, 0, ""), (59, 54, ""), (63, 56, "rtc"),
                                                 (63, 56, "seed")])
def test_small_smolvla_matches_reference(tmp_path, monkeypatch, mask, n_int8, variant):
    pol = _policy(tmp_path, synth.SMOLVLA_SMALL, mask, monkeypatch)
    assert pol.int8_layers == n_int8   # the reference's count on this checkpoint
    f, ins, st, nz, seed, pv, wt, g = smolvla_query(synth.SMOLVLA_SMALL, variant)
    got = pol.predict(f, ins, st, nz, seed, pv, wt, g)
    check_actions(f"smolvla-small-m{mask}-{variant or 'plain'}", got, _want("small", mask, variant), TOL)
    pol.close()


@pytest.mark.parametrize("mask,n_int8", [(63, 57), (0, 0)])
def test_edge_smolvla_matches_reference(tmp_path, monkeypatch, mask, n_int8):
    """One view from 50x100 frames, a two-token prompt padded to 20 (masked
    prefix rows and keys), an expert shallower than the text tower with
    self-attention every third layer, a 7-step chunk and 3 flow steps."""
    pol = _policy(tmp_path, synth.SMOLVLA_EDGE, mask, monkeypatch)
    assert pol.int8_layers == n_int8
    f, ins, st, nz, seed, pv, wt, g = smolvla_query(synth.SMOLVLA_EDGE, "short")
    got = pol.predict(f, ins, st, nz, seed, pv, wt, g)
    check_actions(f"smolvla-edge-m{mask}", got, _want("edge", mask, "short"), TOL)
    pol.close()


def test_baseline_smolvla_matches_reference(tmp_path, monkeypatch):
    pol = _policy(tmp_path, synth.SMOLVLA_BASELINE, 63, monkeypatch)
    assert pol.int8_layers == 298
    f, ins, st, nz, seed, pv, wt, g = smolvla_query(synth.SMOLVLA_BASELINE, "")
    got = pol.predict(f, ins, st, nz, seed)
    check_actions("smolvla-base-m63", got, _want("base", 63), TOL)
    assert np.array_equal(got, pol.predict(f, ins, st, nz, seed)), "query is not deterministic"
    pol.close()


def test_smolvla_batch_equals_single_queries(tmp_path, monkeypatch):
    B = 3
    pol = _policy(tmp_path, synth.SMOLVLA_SMALL, 63, monkeypatch, max_batch=4)
    f, ins, st, nz = synth.smolvla_inputs(synth.SMOLVLA_SMALL, seed=5, batch=B)
    got = pol.predict_batch(f, ins, st, nz)
    for b in range(B):
        assert np.array_equal(got[b], pol.predict(f[b], ins[b], st[b], nz[b])), b
    pol.close()


def test_smolvla_graph_equals_eager(tmp_path, monkeypatch):
    f, ins, st, nz, seed, pv, wt, g = smolvla_query(synth.SMOLVLA_SMALL, "")
    a = _policy(tmp_path, synth.SMOLVLA_SMALL, 63, monkeypatch, graph=True, name="g")
    ga = a.predict(f, ins, st, nz)
    a.close()
    b = _policy(tmp_path, synth.SMOLVLA_SMALL, 63, monkeypatch, graph=False, name="e")
    gb = b.predict(f, ins, st, nz)
    b.close()
    assert np.array_equal(ga, gb)
