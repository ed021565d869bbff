"""The drop-in boundary exercised from the reference's side.

1. Op level (a TCPU_HAL_CUDA backend): oracle/_ref/libvla_ref_cuda.so is the
   reference's own sources with their int8 op API (src/ops/quant_ops.h:40-92)
   defined over this library's vla_tcpu_* C ABI (oracle/ref_cuda_backend.cpp).
   The reference's nn::Linear (src/nn/linear.cpp:66-134), its int8 convolution
   and its whole ACT model then run their int8 layers on the B200 and must give
   the CPU build's bits.
2. Model level: the reference's policy server (vla_simd/policy_server.py,
   copied unmodified into oracle/_ref by oracle/Makefile) drives
   libvla_simd_b200.so through its own ActEngine / DiffusionEngine /
   SmolvlaEngine classes (:276-307, :544-591, :347-451) and must get the
   actions it gets from the reference's library on the same inputs.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from vla_simd_b200 import LIB_PATH, synth

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def ref_cuda():
    from oracle import oracle
    r = oracle.reference_cuda()
    if r is None:
        pytest.skip("oracle/_ref/libvla_ref_cuda.so (the reference over this backend) not built")
    return r


@pytest.mark.parametrize("seq,N,K", [(1, 16, 3), (7, 64, 100), (100, 512, 512), (33, 48, 1027), (602, 3200, 512)])
def test_reference_linear_runs_int8_on_the_gpu_with_the_cpu_bits(ref_cuda, reference, seq, N, K):
    rng = np.random.default_rng(seq * 7 + N + K)
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.01).astype(np.float32)
    x = rng.standard_normal((seq, K), dtype=np.float32)
    got, on_gpu = ref_cuda.nn_linear_forward(W, b, x, int8=True)
    want, on_cpu = reference.nn_linear_forward(W, b, x, int8=True)
    assert on_gpu and on_cpu, "init_int8 declined the layer"
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_reference_int8_ops_over_the_backend(ref_cuda, reference):
    """pack / quantize / pre-quantized GEMM / the backend's own reference GEMM and
    the per-tensor conv (quantize_span_i8 inside) through the reference's op API."""
    rng = np.random.default_rng(5)
    N, K, seq = 96, 147, 41
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float32)
    x = rng.standard_normal((seq, K), dtype=np.float32)
    pg, sg = ref_cuda.pack_weights_i8(W)
    pc, sc = reference.pack_weights_i8(W)
    assert np.array_equal(pg, pc) and np.array_equal(sg.view(np.uint32), sc.view(np.uint32))
    qg, ag = ref_cuda.quantize_act_i8(x)
    qc, ac = reference.quantize_act_i8(x)
    assert np.array_equal(qg, qc) and np.array_equal(ag.view(np.uint32), ac.view(np.uint32))
    b = (rng.standard_normal(N, dtype=np.float32) * 0.01).astype(np.float32)
    ref_out = reference.dense_linear_i8_ref(qc, ac, pc, sc, b, N, K)
    assert np.array_equal(ref_cuda.dense_linear_i8_ref(qg, ag, pg, sg, b, N, K).view(np.uint32),
                          ref_out.view(np.uint32))
    xc = rng.standard_normal((20, 24, 16), dtype=np.float32)
    Wc = (rng.standard_normal((32, 3 * 3 * 16), dtype=np.float32) * 0.05).astype(np.float32)
    pwg, swg = ref_cuda.pack_weights_i8(Wc)
    pwc, swc = reference.pack_weights_i8(Wc)
    bc = (rng.standard_normal(32, dtype=np.float32) * 0.01).astype(np.float32)
    cg = ref_cuda.conv2d_i8(xc, pwg, swg, bc, 32, 3, 2, 1)
    cc = reference.conv2d_i8(xc, pwc, swc, bc, 32, 3, 2, 1)
    assert np.array_equal(cg.view(np.uint32), cc.view(np.uint32))


def _run(code: str, env: dict, timeout=600):
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env}, capture_output=True, text=True,
                       timeout=timeout, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]


def test_reference_act_model_over_the_backend_matches_its_cpu_actions(tmp_path, ref_cuda):
    """The reference's own vla_act_predict with ACT_INT8=63 (int8 transformer and
    backbone) on this backend gives the actions its CPU build gave (fixture)."""
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    out = str(tmp_path / "a.npy")
    code = ("import sys, numpy as np; sys.path.insert(0, %r); from oracle import oracle; "
            "from vla_simd_b200 import synth; r = oracle.reference_cuda(); "
            "f, s = synth.act_inputs(synth.ACT_SMALL, seed=1); np.save(%r, r.act_predict(%r, f, s))") % (ROOT, out, d)
    _run(code, {"ACT_INT8": "63"})
    want = np.load(os.path.join(GOLDEN, "act_small_m63.npy"))
    assert np.array_equal(np.load(out), want)


# The server's engines, run in their own processes: the reference reads its
# int8 masks at load, and its GroupNorm sums are order-defined with one thread.
_ENGINE = r"""
import argparse, importlib.util, json, sys
import numpy as np
sys.path.insert(0, %(root)r)
from oracle import oracle
spec = importlib.util.spec_from_file_location("policy_server", oracle.SERVER_PY)
ps = importlib.util.module_from_spec(spec)
spec.loader.exec_module(ps)
job = json.load(open(%(job)r))
args = argparse.Namespace(lib=job["lib"], model_dir=job["model_dir"], tok_dir=None, rtc_horizon=0,
                          rtc_max_guidance=5.0, rtc_delay=None, fps=30)
eng = getattr(ps, job["engine"])(args)
inputs = [np.load(p) for p in job["inputs"]]
if job["engine"] == "SmolvlaEngine":
    inputs.append(job["task"])
out = eng.predict(tuple(inputs), job["seed"])
np.save(job["out"], out)
eng.close()
"""


def _engine_actions(tmp_path, tag, engine, lib, model_dir, inputs, env, task=None):
    paths = []
    for i, a in enumerate(inputs):
        p = str(tmp_path / f"{tag}_in{i}.npy")
        np.save(p, a)
        paths.append(p)
    job = {"engine": engine, "lib": lib, "model_dir": model_dir, "inputs": paths, "seed": 7, "task": task,
           "out": str(tmp_path / f"{tag}_out.npy")}
    jp = str(tmp_path / f"{tag}.json")
    json.dump(job, open(jp, "w"))
    _run(_ENGINE % {"root": ROOT, "job": jp}, env)
    return np.load(job["out"])


def _server_or_skip():
    from oracle import oracle
    if not os.path.exists(oracle.SERVER_PY) or oracle.reference() is None:
        pytest.skip("the reference build / its copied policy server are not present")
    return oracle.REFERENCE_SO


def test_reference_server_act_engine_unchanged(tmp_path):
    ref_lib = _server_or_skip()
    d = synth.write_act_checkpoint(str(tmp_path / "act"), synth.ACT_SMALL, seed=0)
    f, s = synth.act_inputs(synth.ACT_SMALL, seed=1)
    env = {"ACT_INT8": "63"}
    ours = _engine_actions(tmp_path, "ours", "ActEngine", LIB_PATH, d, [f, s], env)
    theirs = _engine_actions(tmp_path, "ref", "ActEngine", ref_lib, d, [f, s], env)
    assert np.array_equal(ours, theirs)
    assert np.array_equal(ours, np.load(os.path.join(GOLDEN, "act_small_m63.npy")))


def test_reference_server_diffusion_engine_unchanged(tmp_path):
    ref_lib = _server_or_skip()
    d = synth.write_dp_checkpoint(str(tmp_path / "dp"), synth.DP_SMALL, seed=0)
    f, s, _ = synth.dp_inputs(synth.DP_SMALL, seed=1)
    cfg = synth.DP_SMALL
    f = f.reshape(cfg.n_obs_steps, cfg.n_cams, *f.shape[1:])   # the server's [n_obs, n_cams, H, W, 3]
    env = {"DIFFUSION_INT8": "3", "OMP_NUM_THREADS": "1"}
    ours = _engine_actions(tmp_path, "ours", "DiffusionEngine", LIB_PATH, d, [f, s], env)
    theirs = _engine_actions(tmp_path, "ref", "DiffusionEngine", ref_lib, d, [f, s], env)
    assert np.array_equal(ours, theirs)


def test_reference_server_smolvla_engine_unchanged(tmp_path):
    ref_lib = _server_or_skip()
    d = synth.write_smolvla_checkpoint(str(tmp_path / "smol"), synth.SMOLVLA_SMALL, seed=0)
    rng = np.random.default_rng(3)
    cfg = synth.SMOLVLA_SMALL
    frames = rng.integers(0, 256, (cfg.n_views, 48, 64, 3), dtype=np.uint8)
    state = rng.standard_normal(cfg.state_dim, dtype=np.float32)
    env = {"SMOLVLA_INT8": "63"}
    ours = _engine_actions(tmp_path, "ours", "SmolvlaEngine", LIB_PATH, d, [frames, state], env,
                           task="pick up the red cube")
    theirs = _engine_actions(tmp_path, "ref", "SmolvlaEngine", ref_lib, d, [frames, state], env,
                             task="pick up the red cube")
    assert np.array_equal(ours, theirs)
