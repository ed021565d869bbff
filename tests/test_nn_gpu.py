"""The non-GEMM kernels of the policy step against the reference's semantics:
LayerNorm (double accumulation), attention (dense / masked / GQA / fully-masked
rows), max-pool + ReLU, and the per-tensor int8 convolution."""
import numpy as np
import pytest

from oracle.oracle import XorShift

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.parametrize("seq,H", [(1, 768), (50, 960), (7, 6), (602, 512), (100, 512), (3, 2048)])
def test_layernorm(dev, seq, H):
    """tests/test_ops.cpp:296-320: |err| <= 1e-5 against a double LayerNorm."""
    from vla_simd_b200 import ops
    g = XorShift()
    x = g.uniform(seq * H, -3.0, 5.0).reshape(seq, H)
    w, b = g.uniform(H), g.uniform(H)
    y = ops.layernorm(_t(x, dev), _t(w, dev), _t(b, dev), 1e-5).cpu().numpy()
    xd = x.astype(np.float64)
    mu = xd.mean(axis=1, keepdims=True)
    var = ((xd - mu) ** 2).mean(axis=1, keepdims=True)
    want = (xd - mu) / np.sqrt(var + 1e-5) * w + b
    assert np.abs(y - want).max() <= 1e-5


def test_layernorm_matches_reference(dev, reference):
    from vla_simd_b200 import ops
    g = XorShift(99)
    x = g.uniform(602 * 512, -3.0, 5.0).reshape(602, 512)
    w, b = g.uniform(512), g.uniform(512)
    y = ops.layernorm(_t(x, dev), _t(w, dev), _t(b, dev), 1e-5).cpu().numpy()
    assert np.abs(y - reference.layernorm(x, w, b, 1e-5)).max() <= 1e-6


def naive_attention(Q, K, V, mask, sq, sk, nq, nkv, hd, scale):
    out = np.zeros((sq, nq * hd))
    Qd, Kd, Vd = (a.astype(np.float64) for a in (Q, K, V))
    for h in range(nq):
        g = h // (nq // nkv)
        q = Qd[:, h * hd:(h + 1) * hd]
        k = Kd[:, g * hd:(g + 1) * hd]
        v = Vd[:, g * hd:(g + 1) * hd]
        s = q @ k.T * scale
        if mask is not None:
            s = s + mask
        mx = s.max(axis=1, keepdims=True)
        e = np.where(np.isinf(s), 0.0, np.exp(s - mx))
        out[:, h * hd:(h + 1) * hd] = (e @ v) / e.sum(axis=1, keepdims=True)
    return out


CFGS = [(1, 50, 8, 2), (50, 50, 8, 2), (50, 113, 15, 5), (256, 256, 12, 12), (12, 512, 4, 2), (602, 602, 8, 8),
        (100, 602, 8, 8)]


@pytest.mark.parametrize("sq,sk,nq,nkv", CFGS)
def test_attention_dense_and_causal(dev, sq, sk, nq, nkv):
    """tests/test_ops.cpp:221-255: <= 2e-6 against a double oracle."""
    from vla_simd_b200 import ops
    hd = 64
    g = XorShift()
    Q = g.uniform(sq * nq * hd).reshape(sq, nq * hd)
    K = g.uniform(sk * nkv * hd).reshape(sk, nkv * hd)
    V = g.uniform(sk * nkv * hd).reshape(sk, nkv * hd)
    scale = np.float32(1.0) / np.sqrt(np.float32(hd))
    dense = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, float(scale)).cpu().numpy()
    assert np.abs(dense - naive_attention(Q, K, V, None, sq, sk, nq, nkv, hd, scale)).max() <= 2e-6
    zero = np.zeros((sq, sk), np.float32)
    masked0 = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, float(scale),
                                mask=_t(zero, dev)).cpu().numpy()
    assert np.array_equal(masked0, dense)
    i = np.arange(sq)[:, None]
    j = np.arange(sk)[None, :]
    causal = np.where(j > i + (sk - sq), -np.inf, 0.0).astype(np.float32)
    got = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, float(scale), mask=_t(causal, dev))
    want = naive_attention(Q, K, V, causal, sq, sk, nq, nkv, hd, scale)
    assert np.abs(got.cpu().numpy() - want).max() <= 2e-6


@pytest.mark.parametrize("block", [-np.inf, np.finfo(np.float32).min])
def test_attention_fully_masked_rows_are_mean_v(dev, block):
    from vla_simd_b200 import ops
    sq, sk, nq, nkv, hd = 17, 33, 4, 2, 64
    g = XorShift(5)
    Q = g.uniform(sq * nq * hd).reshape(sq, nq * hd)
    K = g.uniform(sk * nkv * hd).reshape(sk, nkv * hd)
    V = g.uniform(sk * nkv * hd).reshape(sk, nkv * hd)
    mask = np.full((sq, sk), block, np.float32)
    out = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, 0.125, mask=_t(mask, dev)).cpu().numpy()
    for h in range(nq):
        gk = h // (nq // nkv)
        mean = V[:, gk * hd:(gk + 1) * hd].astype(np.float64).mean(axis=0)
        assert np.isfinite(out).all()
        assert np.abs(out[:, h * hd:(h + 1) * hd] - mean).max() < 2e-6


def test_attention_matches_reference(dev, reference):
    from vla_simd_b200 import ops
    g = XorShift(7)
    sq, sk, n = 602, 602, 8
    Q = g.uniform(sq * n * 64).reshape(sq, n * 64)
    K = g.uniform(sk * n * 64).reshape(sk, n * 64)
    V = g.uniform(sk * n * 64).reshape(sk, n * 64)
    got = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), n, n, 0.125).cpu().numpy()
    assert np.abs(got - reference.attention(Q, K, V, n, n, 64, np.float32(0.125))).max() <= 2e-6


@pytest.mark.parametrize("sq,sk,nq,nkv", [(1024, 1024, 12, 12), (690, 690, 12, 12), (50, 227, 15, 5)])
def test_attention_tile_heights_vs_reference(dev, reference, sq, sk, nq, nkv):
    """Shapes whose default query tile is 32 rows (SigLIP's 1024 keys, Octo's
    690) or 8 rows (the SmolVLA expert's GQA): the reference's bits."""
    from vla_simd_b200 import ops
    g = XorShift(sq + sk)
    Q = g.uniform(sq * nq * 64).reshape(sq, nq * 64)
    K = g.uniform(sk * nkv * 64).reshape(sk, nkv * 64)
    V = g.uniform(sk * nkv * 64).reshape(sk, nkv * 64)
    got = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, 0.125).cpu().numpy()
    assert np.array_equal(got, reference.attention(Q, K, V, nq, nkv, 64, np.float32(0.125)))


@pytest.mark.parametrize("seq,N,K", [(128, 720, 1440), (96, 720, 1037), (400, 720, 520), (50, 720, 1440),
                                      (50, 32, 720), (33, 4, 1000)])
def test_dense_linear_f32_long_k_vs_reference(dev, reference, seq, N, K):
    """K > 512 (the SmolVLA expert's time MLP and projections): the tiled
    kernel streaming K through shared memory in chunks (rows x outputs >=
    65536) and the warp-per-output kernel below that: the reference's bits."""
    from vla_simd_b200 import ops
    rng = np.random.default_rng(seq * N + K)
    x = rng.standard_normal((seq, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    got = ops.dense_linear_f32(_t(x, dev), _t(W, dev), _t(b, dev)).cpu().numpy()
    assert np.array_equal(got, reference.dense_linear(x, W, b))


@pytest.mark.parametrize("H,W,C", [(240, 320, 64), (7, 9, 16), (1, 1, 64)])
def test_maxpool_relu_exact(dev, H, W, C):
    from vla_simd_b200 import ops
    rng = np.random.default_rng(H * W)
    x = rng.standard_normal((2, H, W, C), dtype=np.float32)
    got = ops.maxpool2d_relu(_t(x, dev)).cpu().numpy()
    Ho, Wo = (H + 2 - 3) // 2 + 1, (W + 2 - 3) // 2 + 1
    xp = np.full((2, H + 2, W + 2, C), -np.inf, np.float32)
    xp[:, 1:-1, 1:-1] = x
    want = np.full((2, Ho, Wo, C), -np.inf, np.float32)
    for ky in range(3):
        for kx in range(3):
            want = np.maximum(want, xp[:, ky:ky + 2 * Ho:2, kx:kx + 2 * Wo:2][:, :Ho, :Wo])
    want = np.where(want > 0, want, np.float32(0))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("H,W,Cin,Cout,k,st,pd", [(30, 30, 3, 64, 7, 2, 3), (28, 28, 64, 64, 3, 1, 1),
                                                  (15, 15, 64, 128, 3, 2, 1), (9, 11, 32, 16, 1, 2, 0),
                                                  (60, 80, 128, 128, 3, 1, 1)])
def test_conv2d_i8_bit_exact(dev, restated, H, W, Cin, Cout, k, st, pd):
    """Two frames at once, each with its own per-tensor scale, against the oracle per frame."""
    import torch
    from vla_simd_b200 import ops
    g = XorShift(0x1234567)
    x = np.stack([g.uniform(H * W * Cin).reshape(H, W, Cin), 3.0 * g.uniform(H * W * Cin).reshape(H, W, Cin)])
    Wt = g.uniform(Cout * k * k * Cin, -0.1, 0.1).reshape(Cout, k * k * Cin)
    b = g.uniform(Cout)
    wq, ws = ops.pack_weights_i8(_t(Wt, dev))
    got = ops.conv2d_i8(_t(x, dev), wq, ws, _t(b, dev), Cout, k, st, pd)
    torch.cuda.synchronize()
    wqh, wsh = restated.quantize_rows(Wt)
    for f in range(2):
        want = restated.conv2d_i8(x[f], wqh, wsh, b, Cout, k, st, pd)
        assert np.array_equal(got[f].cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert ops.device_status() == 0


# ---- bit-exactness of the fp32 ops that feed int8 quantizers, against the
# reference's own outputs (tests/golden/gemm.json, made by make_golden.py)

def _golden():
    import json
    import os
    import sys
    here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, here)
    import make_golden
    return make_golden, json.load(open(os.path.join(here, "gemm.json")))["fp32_ops"], here


def test_attention_bit_exact_vs_reference(dev):
    from vla_simd_b200 import ops
    mg, fp, _ = _golden()
    for sq, sk, nq, nkv in mg.ATTN_CASES:
        Q, K, V = mg.attn_inputs(sq, sk, nq, nkv)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(64.0)))
        got = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, scale).cpu().numpy()
        assert mg.sha(got) == fp[f"attn_{sq}x{sk}x{nq}x{nkv}"], (sq, sk, nq, nkv)
        m = _t(mg.causal_mask(sq, sk), dev)
        got = ops.gqa_attention(_t(Q, dev), _t(K, dev), _t(V, dev), nq, nkv, scale, mask=m).cpu().numpy()
        assert mg.sha(got) == fp[f"attn_causal_{sq}x{sk}x{nq}x{nkv}"], ("causal", sq, sk, nq, nkv)


def test_dense_linear_f32_bit_exact_vs_reference(dev):
    from vla_simd_b200 import ops
    mg, fp, _ = _golden()
    for seq, N, K in mg.F32_LINEAR_CASES:
        x, W, b = mg.f32_linear_inputs(seq, N, K)
        got = ops.dense_linear_f32(_t(x, dev), _t(W, dev), _t(b, dev)).cpu().numpy()
        assert mg.sha(got) == fp[f"f32lin_{seq}x{N}x{K}"], (seq, N, K)


def test_layernorm_vs_reference_bits(dev):
    """Double accumulation in a different order: identical bits except on
    rare double->float rounding ties."""
    import os
    from vla_simd_b200 import ops
    mg, fp, here = _golden()
    z = np.load(os.path.join(here, "gemm.npz"))
    for seq, H in mg.LN_CASES:
        x, w, b = mg.ln_inputs(seq, H)
        got = ops.layernorm(_t(x, dev), _t(w, dev), _t(b, dev), 1e-5).cpu().numpy()
        want = z[f"ln_{seq}x{H}"]
        diff = got.view(np.uint32) != want.view(np.uint32)
        assert diff.mean() <= 1e-4 and np.abs(got - want).max() <= 1e-6
