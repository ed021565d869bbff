"""lm / conv ops of the other policy families against the reference's own CPU functions.

RMSNorm, ReLU, im2col1d, conv_transpose1d and the SIMD bodies of the
activations (every element but the n % 8 scalar tail, which the reference
runs through libm) must be the reference's bits. RoPE (double sin/cos),
silu and spatial softmax (libm exp) and GroupNorm (OpenMP-partitioned sums
in the reference) are held to the reference tests' tolerances
(tests/test_ops.cpp: activations <= 2e-6, norms <= 1e-5).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("seq,hidden", [(177, 960), (3, 768), (5, 37), (1, 6144)])
def test_rmsnorm_bit_exact(dev, reference, seq, hidden):
    from vla_simd_b200 import ops
    rng = np.random.default_rng(seq * hidden)
    x = (rng.standard_normal((seq, hidden)) * 3).astype(np.float32)
    w = rng.standard_normal(hidden).astype(np.float32)
    got = ops.rmsnorm(_t(x, dev), _t(w, dev), 1e-6).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(reference.rmsnorm(x, w, 1e-6)))


@pytest.mark.parametrize("seq,heads,hd,base", [(17, 15, 64, 10000.0), (5, 5, 64, 100000.0), (3, 2, 128, 10000.0)])
def test_rope_neox(dev, reference, seq, heads, hd, base):
    import torch
    from vla_simd_b200 import ops
    rng = np.random.default_rng(seq + heads)
    x = rng.standard_normal((seq, heads * hd)).astype(np.float32)
    pos = rng.integers(0, 512, seq).astype(np.int32)
    got = ops.rope_neox(_t(x, dev), torch.from_numpy(pos).to(dev), heads, hd, base).cpu().numpy()
    want = reference.rope_neox(x, pos, heads, hd, base)
    assert np.abs(got - want).max() <= 1e-6 * max(1.0, np.abs(want).max())
    # the double trig differs from the C library's by at most an ulp or two:
    # almost every output rounds to the same float
    assert np.mean(_bits(got) == _bits(want)) > 0.999


@pytest.mark.parametrize("name", ["relu", "silu_gate", "gelu_tanh", "gelu_erf", "mish", "silu"])
@pytest.mark.parametrize("n", [1003, 4096, 7])
def test_activations(dev, reference, name, n):
    """Bit-identical to the reference: its 8-lane bodies (Cephes exp) and, past
    them, its scalar forms with the C library's float functions (restated);
    silu is that scalar form everywhere. gelu_erf's tail stays within tolerance."""
    from vla_simd_b200 import ops
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 4).astype(np.float32)
    specials = np.array([0.0, -0.0, 25.0, -25.0, 90.0, -90.0, 1e-30, -1e-30, 21.0, 19.9, -0.3, 1e-8],
                        np.float32)
    x[:min(n, 8)] = specials[:min(n, 8)]           # saturation, exp clamps, denormal range
    x[-min(n, 4):] = specials[8:8 + min(n, 4)]     # and the scalar tail's branches
    u = rng.standard_normal(n).astype(np.float32)
    got = ops.activation(name, _t(x, dev), _t(u, dev) if name == "silu_gate" else None).cpu().numpy()
    want = reference.activation(name, x, u if name == "silu_gate" else None)
    if name == "gelu_erf":
        body = n - n % 8
        assert np.array_equal(_bits(got[:body]), _bits(want[:body])), name
        assert np.allclose(got[body:], want[body:], rtol=2e-6, atol=2e-6)
        return
    assert np.array_equal(_bits(got), _bits(want)), name


def test_silu_libm_exp_on_many_inputs(dev, reference):
    """silu = x / (1 + expf(-x)) over 2^22 inputs spread across the float range
    (the restated expf on the device against the host library's)."""
    from vla_simd_b200 import ops
    rng = np.random.default_rng(11)
    bits = rng.integers(0, 2**32, 1 << 22, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32).copy()
    x[~np.isfinite(x)] = 1.0
    x = np.concatenate([x, np.linspace(-100, 100, 1 << 20, dtype=np.float32)])
    got = ops.activation("silu", _t(x, dev)).cpu().numpy()
    want = reference.activation("silu", x)
    same = (_bits(got) == _bits(want)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), x[~same][:5]


def test_mish_tail_libm_on_many_inputs(dev, reference):
    """The scalar Mish tail (expf, log1pf, tanhf restated) on 7-element calls,
    where every element is past the 8-lane loop."""
    from vla_simd_b200 import ops
    rng = np.random.default_rng(12)
    vals = np.concatenate([rng.standard_normal(700) * 8, np.linspace(-30, 30, 700)]).astype(np.float32)
    for i in range(0, len(vals), 7):
        x = vals[i:i + 7]
        got = ops.activation("mish", _t(x, dev)).cpu().numpy()
        want = reference.activation("mish", x)
        assert np.array_equal(_bits(got), _bits(want)), x


@pytest.mark.parametrize("P,C,groups,relu", [(100, 512, 8, False), (1764, 64, 8, True), (16, 2048, 32, False)])
def test_groupnorm(dev, reference, P, C, groups, relu):
    from vla_simd_b200 import ops
    rng = np.random.default_rng(P + C)
    x = (rng.standard_normal((P, C)) * 2 + 0.5).astype(np.float32)
    sc = rng.standard_normal(C).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    got = ops.groupnorm(_t(x, dev), _t(sc, dev), _t(b, dev), groups, 1e-5, relu).cpu().numpy()
    want = reference.groupnorm(x, sc, b, groups, 1e-5, relu)
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("P,C", [(49, 64), (441, 512), (1, 3)])
def test_spatial_softmax(dev, reference, P, C):
    from vla_simd_b200 import ops
    rng = np.random.default_rng(P * C)
    x = (rng.standard_normal((P, C)) * 3).astype(np.float32)
    grid = rng.uniform(-1, 1, (P, 2)).astype(np.float32)
    got = ops.spatial_softmax(_t(x, dev), _t(grid, dev)).cpu().numpy()
    assert np.allclose(got, reference.spatial_softmax(x, grid), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("T,Cin,k,stride,pad", [(16, 64, 5, 1, 2), (33, 7, 3, 2, 1), (4, 512, 5, 1, 2)])
def test_im2col1d_exact(dev, reference, T, Cin, k, stride, pad):
    from vla_simd_b200 import ops
    x = np.random.default_rng(T).standard_normal((T, Cin)).astype(np.float32)
    got = ops.im2col1d(_t(x, dev), k, stride, pad).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(reference.im2col1d(x, k, stride, pad)))


# the U-Net's two upsampling shapes (1024 and 512 channels: 16 and 8 weight
# chunks resident in shared memory), a ragged last weight chunk and input
# block (Cin 100) with four chains per thread (Tout 40), and Cin 3, which only
# the general kernel takes
@pytest.mark.parametrize("T,Cin,Cout,k,stride,pad,bias", [(16, 64, 32, 4, 2, 1, True), (8, 256, 128, 3, 1, 1, False),
                                                          (5, 3, 70, 4, 2, 1, True), (4, 1024, 1024, 4, 2, 1, True),
                                                          (8, 512, 512, 4, 2, 1, False), (20, 100, 64, 4, 2, 1, False)])
def test_conv_transpose1d_exact(dev, reference, T, Cin, Cout, k, stride, pad, bias):
    from vla_simd_b200 import ops
    rng = np.random.default_rng(T * Cin)
    x = rng.standard_normal((T, Cin)).astype(np.float32)
    x[x < -0.8] = 0.0                      # the reference skips zero inputs
    W = (rng.standard_normal((Cin, k, Cout)) * 0.1).astype(np.float32)
    b = rng.standard_normal(Cout).astype(np.float32) if bias else None
    got = ops.conv_transpose1d(_t(x, dev), _t(W, dev), _t(b, dev) if bias else None, k, stride, pad).cpu().numpy()
    assert np.array_equal(_bits(got), _bits(reference.conv_transpose1d(x, W, b, k, stride, pad)))


def test_bad_arguments_are_refused(dev):
    import ctypes
    from vla_simd_b200 import lib
    L = lib()
    fake = ctypes.c_void_p(256)
    assert L.vla_cuda_rmsnorm(fake, fake, fake, 4, 7000, 1e-6, None) != 0          # hidden > 6144
    assert L.vla_cuda_rope_neox(fake, fake, 4, 2, 63, 1e4, None) != 0               # odd head_dim
    assert L.vla_cuda_groupnorm(fake, fake, fake, fake, 4, 30, 8, 1e-5, 0, fake, None) != 0   # C % groups
    assert L.vla_cuda_silu_gate(fake, fake, None, 8, None) != 0                      # no gate operand
