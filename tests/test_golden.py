"""The committed fixtures (made by tests/golden/make_golden.py from the
reference's own code) pin the C restatement on machines without the reference,
and the synthetic checkpoint writer still reproduces the bytes they came from."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, HERE)
from make_golden import GEMM_SHAPES, dir_digest, gemm_inputs, sha  # noqa: E402

from vla_simd_b200 import synth  # noqa: E402

GEMM = json.load(open(os.path.join(HERE, "gemm.json")))


@pytest.mark.parametrize("seq,N,K", GEMM_SHAPES)
def test_restated_oracle_reproduces_reference_fixtures(restated, seq, N, K):
    x, W, b = gemm_inputs(seq, N, K)
    xq, xs = restated.quantize_rows(x)
    wq, ws = restated.quantize_rows(W)
    acc = restated.gemm_acc(xq, wq, K)
    out = restated.dense_linear_i8_ref(xq, xs, wq, ws, b, K)
    g = GEMM[f"{seq}x{N}x{K}"]
    assert sha(xq) == g["xq"] and sha(xs) == g["ascale"]
    assert sha(wq) == g["wq"] and sha(ws) == g["wscale"]
    assert sha(acc) == g["acc"] and sha(out) == g["out"]


def test_small_fixture_arrays_are_consistent():
    z = np.load(os.path.join(HERE, "gemm.npz"))
    for key in [k[:-4] for k in z.files if k.endswith("_out")]:
        assert sha(z[f"{key}_out"]) == GEMM[key]["out"]
        assert sha(z[f"{key}_acc"]) == GEMM[key]["acc"]


@pytest.mark.parametrize("cfg,shape", [("small", synth.ACT_SMALL), ("base", synth.ACT_BASELINE),
                                       ("dp_small", synth.DP_SMALL), ("dp_base", synth.DP_BASELINE),
                                       ("dp_edge", synth.DP_EDGE), ("dp_deep", synth.DP_DEEP)])
def test_checkpoint_writer_matches_fixture_source(tmp_path, cfg, shape):
    if cfg.startswith("dp_"):
        d = synth.write_dp_checkpoint(str(tmp_path / cfg), shape, seed=0)
    else:
        d = synth.write_act_checkpoint(str(tmp_path / cfg), shape, seed=0)
    assert dir_digest(d) == json.load(open(os.path.join(HERE, "checkpoints.json")))[cfg]


@pytest.mark.parametrize("cfg,shape", [("octo_small", synth.OCTO_SMALL), ("octo_base", synth.OCTO_BASELINE),
                                       ("smolvla_small", synth.SMOLVLA_SMALL), ("smolvla_base", synth.SMOLVLA_BASELINE),
                                       ("smolvla_edge", synth.SMOLVLA_EDGE), ("octo_erf", synth.OCTO_ERF)])
def test_octo_checkpoint_writer_matches_fixture_source(tmp_path, cfg, shape):
    writer = synth.write_smolvla_checkpoint if cfg.startswith("smolvla") else synth.write_octo_checkpoint
    d = writer(str(tmp_path / cfg), shape, seed=0)
    want = json.load(open(os.path.join(HERE, "checkpoints.json")))[cfg]
    assert dir_digest(d) + dir_digest(os.path.join(d, "tok"))[:16] == want


def test_reference_octo_fixture_is_current(tmp_path, reference, monkeypatch):
    from make_golden import octo_query
    monkeypatch.setenv("OCTO_INT8", "0")   # read once per process by the reference; 0 is its default
    d = synth.write_octo_checkpoint(str(tmp_path / "octo"), synth.OCTO_SMALL, seed=0)
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_SMALL, "")
    got = reference.octo_predict(d, d + "/tok", p, w, tm, ins, n, z)
    if os.environ.get("OCTO_INT8", "0") == "0":
        assert np.array_equal(got, np.load(os.path.join(HERE, "octo_small_m0.npy")))


def test_reference_policy_fixture_is_current(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("ACT_INT8", "63")
    d = synth.write_act_checkpoint(str(tmp_path / "small"), synth.ACT_SMALL, seed=0)
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    got = reference.act_predict(d, f, s)
    assert np.array_equal(got, np.load(os.path.join(HERE, "act_small_m63.npy")))


def test_reference_dp_fixture_is_current(tmp_path, reference, monkeypatch):
    monkeypatch.setenv("DIFFUSION_INT8", "3")
    monkeypatch.setenv("OMP_NUM_THREADS", "1")
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_SMALL, seed=0)
    f, s, n = synth.dp_inputs(synth.DP_SMALL, seed=1)
    got = reference.dp_predict(d, f, s, n)
    assert np.array_equal(got, np.load(os.path.join(HERE, "dp_small_m3.npy")))
