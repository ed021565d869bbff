"""Implicit-GEMM convolution (stride 1, C % 64 == 0) against the im2col path and the oracle.

The implicit path quantizes the NHWC input once and lets the tensor-core GEMM
gather each filter tap with a 4D TMA tile load; output tiles are patches of
output pixels. It must give exactly the bits of the explicit im2col + GEMM
path (VLA_CONV_IM2COL=1) and of the reference conv, for ragged patches, every
tap count, padding, both k-block widths (64-channel and 128-channel blocks)
and every GEMM launch plan.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [  # H, W, C, Cout, k, pad
    (28, 28, 64, 64, 3, 1),      # 64-byte k-blocks
    (15, 20, 128, 96, 3, 1),     # 128-byte k-blocks, partial patches
    (7, 9, 192, 64, 3, 1),       # C % 128 != 0 -> 64-byte blocks, 3 per tap
    (30, 40, 256, 256, 3, 1),
    (9, 11, 64, 32, 1, 0),       # 1x1
    (12, 10, 128, 64, 5, 2),     # 5x5
    (6, 6, 64, 48, 3, 0),        # no padding
    (1, 1, 128, 128, 3, 1),      # single pixel
]


@pytest.fixture(scope="module")
def dev():
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _inputs(H, W, C, Cout, k, seed):
    rng = np.random.default_rng(seed)
    x = np.stack([rng.standard_normal((H, W, C), dtype=np.float32),
                  3.0 * rng.standard_normal((H, W, C), dtype=np.float32)])
    Wt = (rng.standard_normal((Cout, k * k * C), dtype=np.float32) * 0.05).astype(np.float32)
    b = (rng.standard_normal(Cout, dtype=np.float32) * 0.1).astype(np.float32)
    return x, Wt, b


def _run(dev, monkeypatch, x, Wt, b, Cout, k, pad, im2col, mode=0, res=None):
    import torch
    from vla_simd_b200 import ops
    if im2col:
        monkeypatch.setenv("VLA_CONV_IM2COL", "1")
    else:
        monkeypatch.delenv("VLA_CONV_IM2COL", raising=False)
    wq, ws = ops.pack_weights_i8(_t(Wt, dev))
    out = ops.conv2d_i8(_t(x, dev), wq, ws, _t(b, dev), Cout, k, 1, pad, mode=mode,
                        res=_t(res, dev) if res is not None else None)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    return out.cpu().numpy()


@pytest.mark.parametrize("H,W,C,Cout,k,pad", SHAPES)
def test_implicit_equals_im2col_and_reference(dev, restated, monkeypatch, H, W, C, Cout, k, pad):
    x, Wt, b = _inputs(H, W, C, Cout, k, H * W + C)
    got = _run(dev, monkeypatch, x, Wt, b, Cout, k, pad, im2col=False)
    ref = _run(dev, monkeypatch, x, Wt, b, Cout, k, pad, im2col=True)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    wqh, wsh = restated.quantize_rows(Wt)
    for f in range(2):
        want = restated.conv2d_i8(x[f], wqh, wsh, b, Cout, k, 1, pad)
        assert np.array_equal(got[f].view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("plan", ["32:1", "64:1", "128:1", "64:3", "128:4", "256:2"])
def test_implicit_every_plan(dev, monkeypatch, plan):
    """128-channel blocks: persistent and cluster split-K plans, residual epilogue."""
    from vla_simd_b200 import EPI_ADD_RELU
    H, W, C, Cout, k, pad = 15, 20, 256, 128, 3, 1
    x, Wt, b = _inputs(H, W, C, Cout, k, 7)
    res = np.random.default_rng(8).standard_normal((2, H, W, Cout), dtype=np.float32)
    ref = _run(dev, monkeypatch, x, Wt, b, Cout, k, pad, im2col=True, mode=EPI_ADD_RELU, res=res)
    monkeypatch.setenv("VLA_GEMM_PLAN", plan)
    got = _run(dev, monkeypatch, x, Wt, b, Cout, k, pad, im2col=False, mode=EPI_ADD_RELU, res=res)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))

