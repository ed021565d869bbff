"""The tensor-core attention (tcgen05 kind::tf32, 3xTF32 split precision,
vla_cuda_gqa_attention_tc) against the exact kernel and against float64, and
what it does to the policies' actions when they run on it (VLA_ATT_TC=1).

The exact kernel is the reference's arithmetic (bit-identical to its AVX2
attention, src/hal/avx2/attn.cpp:134-251); the tensor-core one sums in another
order, so the test bounds its error instead: within 1e-5 of the largest output
magnitude of the float64 result (measured: 1-4e-6, about five times the exact
kernel's own 2-7e-7; the tf32 truncation of each split's low part is the rest).
The policy drift is measured against the reference's action fixtures and
recorded (VLA_PARITY_LOG), and bounded loosely: its size is the finding.
"""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="module")
def dev():
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _f64_attention(Q, K, V, n_q, n_kv, scale, mask):
    sq, sk = Q.shape[0], K.shape[0]
    out = np.zeros((sq, n_q * 64))
    for h in range(n_q):
        g = h // (n_q // n_kv)
        q = Q[:, h * 64:(h + 1) * 64].astype(np.float64)
        k = K[:, g * 64:(g + 1) * 64].astype(np.float64)
        v = V[:, g * 64:(g + 1) * 64].astype(np.float64)
        s = q @ k.T * scale
        if mask is not None:
            s = s + mask.astype(np.float64)
        blocked = ~(s.max(axis=1) > -np.finfo(np.float32).max)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=1, keepdims=True)
        p[blocked] = 1.0 / sk
        out[:, h * 64:(h + 1) * 64] = p @ v
    return out


CASES = [(602, 602, 8, 8, None), (100, 602, 8, 8, None), (100, 100, 8, 8, "causal"), (77, 130, 15, 5, "causal"),
         (200, 65, 12, 12, "blocked"), (1, 1, 1, 1, None), (300, 690, 12, 12, "blocked")]


@pytest.mark.parametrize("sq,sk,nq,nkv,mask_kind", CASES)
def test_tc_attention_within_fp32_error(dev, sq, sk, nq, nkv, mask_kind):
    import torch
    from vla_simd_b200 import ops
    rng = np.random.default_rng(sq * 31 + sk)
    Q = rng.standard_normal((sq, nq * 64), dtype=np.float32)
    K = rng.standard_normal((sk, nkv * 64), dtype=np.float32)
    V = rng.standard_normal((sk, nkv * 64), dtype=np.float32)
    mask = None
    if mask_kind == "causal":
        mask = np.where(np.arange(sk)[None, :] <= np.arange(sq)[:, None] + (sk - sq), 0.0,
                        -np.finfo(np.float32).max).astype(np.float32)
    elif mask_kind == "blocked":   # block-causal rows plus some rows with every key blocked
        mask = np.where((np.arange(sk)[None, :] // 16) <= (np.arange(sq)[:, None] // 16), 0.0,
                        -np.finfo(np.float32).max).astype(np.float32)
        mask[::7] = -np.finfo(np.float32).max
    scale = np.float32(0.125)
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    tc = ops.gqa_attention_tc(t(Q), t(K), t(V), nq, nkv, float(scale), t(mask)).cpu().numpy()
    ex = ops.gqa_attention(t(Q), t(K), t(V), nq, nkv, float(scale), t(mask)).cpu().numpy()
    torch.cuda.synchronize()
    want = _f64_attention(Q, K, V, nq, nkv, scale, mask)
    big = max(1.0, float(np.abs(want).max()))
    err_tc = float(np.abs(tc - want).max()) / big
    err_ex = float(np.abs(ex - want).max()) / big
    print(f"{sq}x{sk}x{nq}/{nkv} {mask_kind}: tensor-core {err_tc:.3g}, exact kernel {err_ex:.3g} (relative to f64)")
    assert np.isfinite(tc).all()
    assert err_tc <= 1e-5, (err_tc, err_ex)
    assert ops.device_status() == 0


_POLICY = r"""
import json, sys
import numpy as np
sys.path.insert(0, %(root)r)
sys.path.insert(0, %(golden)r)
from vla_simd_b200 import synth
kind = %(kind)r
import tempfile
d = tempfile.mkdtemp()
if kind == "act":
    from vla_simd_b200 import ActPolicy
    path = synth.write_act_checkpoint(d + "/m", synth.ACT_BASELINE, seed=0)
    pol = ActPolicy(path)
    f, s = synth.act_inputs(synth.ACT_BASELINE, seed=1)
    got = pol.predict(f, s)
elif kind == "octo":
    from vla_simd_b200 import OctoPolicy
    from make_golden import octo_query
    path = synth.write_octo_checkpoint(d + "/m", synth.OCTO_BASELINE, seed=0)
    pol = OctoPolicy(path, max_batch=1)
    p, w, tm, ins, n, z, seed = octo_query(synth.OCTO_BASELINE, "")
    got = pol.predict(p, w, tm, ins, n, z)
else:
    from vla_simd_b200 import SmolvlaPolicy
    from make_golden import smolvla_query
    path = synth.write_smolvla_checkpoint(d + "/m", synth.SMOLVLA_BASELINE, seed=0)
    pol = SmolvlaPolicy(path, max_batch=1)
    f, ins, st, nz, seed, pv, wt, g = smolvla_query(synth.SMOLVLA_BASELINE, "")
    got = pol.predict(f, ins, st, nz, seed)
np.save(%(out)r, got)
"""

POLICIES = [("act", "act_base_m63.npy", {"ACT_INT8": "63"}), ("octo", "octo_base_m63.npy", {"OCTO_INT8": "63"}),
            ("smolvla", "smolvla_base_m63.npy", {"SMOLVLA_INT8": "63"})]


@pytest.mark.parametrize("kind,fixture,env", POLICIES, ids=[p[0] for p in POLICIES])
def test_tc_attention_policy_drift(tmp_path, kind, fixture, env):
    """The BASELINE-config policies with every attention on the tensor cores:
    the max-abs difference of their actions from the reference's."""
    out = str(tmp_path / "a.npy")
    code = _POLICY % {"root": ROOT, "golden": GOLDEN, "kind": kind, "out": out}
    r = subprocess.run([sys.executable, "-c", code], env={**os.environ, **env, "VLA_ATT_TC": "1"},
                       capture_output=True, text=True, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    got = np.load(out)
    want = np.load(os.path.join(GOLDEN, fixture))
    err = float(np.abs(got - want).max())
    scale = float(np.abs(want).max())
    print(f"{kind} baseline with tensor-core attention: actions max-abs {err:.3g} vs reference "
          f"(action magnitude {scale:.3g})")
    log = os.environ.get("VLA_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps({"label": f"{kind}-base-m63-attention-tc", "max_abs": err,
                                "bit_identical": bool(np.array_equal(got, want))}) + "\n")
    assert np.isfinite(got).all()
    assert err <= 0.1 * max(1.0, scale)
