"""Every launch plan of the W8A8 GEMM gives the same bits.

The tensor-core GEMM runs either as a persistent kernel (one CTA per SM
looping over 128 x BN tiles) or split over K across the CTAs of a
thread-block cluster, whose int32 partial tiles are summed through
distributed shared memory. VLA_GEMM_PLAN=<bn>:<splits> forces a plan; each
one must reproduce the reference's int32 accumulators and fp32 epilogue
outputs exactly, including the in-place residual and the absmax tap.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# <bn>:<splits>[:<ring stages>]
PLANS = ["32:1", "64:1", "128:1", "256:1", "32:2", "64:3", "128:2", "128:4", "128:7", "256:2", "128:8",
         "64:1:2", "32:1:8", "128:1:6", "128:4:3", "256:3:3", "64:5:8"]


@pytest.fixture(scope="module")
def dev():
    import torch
    torch.cuda.set_device(0)
    return torch.device("cuda:0")


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _bits_equal(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))


@pytest.mark.parametrize("plan", PLANS)
@pytest.mark.parametrize("M,N,K", [(1, 48, 129), (129, 272, 1152), (600, 512, 4608), (602, 512, 3200),
                                   (2400, 256, 2304), (77, 96, 2000)])
def test_plan_int32_exact(dev, restated, monkeypatch, plan, M, N, K):
    import torch
    from vla_simd_b200 import EPI_ACC, ops
    monkeypatch.setenv("VLA_GEMM_PLAN", plan)
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ld = ops.i8_ld(K)
    xpad = np.zeros((M, ld), np.int8)
    xpad[:, :K] = xq
    wpad = np.full((N, ld), -5, np.int8)     # bytes past K must be ignored
    wpad[:, :K] = wq
    one = torch.ones(max(M, N), device=dev)
    acc = ops.gemm_i8(_t(xpad, dev), one, _t(wpad, dev), one, K, mode=EPI_ACC)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), restated.gemm_acc(xq, wq, K))
    assert ops.device_status() == 0


@pytest.mark.parametrize("plan", PLANS)
@pytest.mark.parametrize("mode", ["none", "relu", "add", "add_relu"])
def test_plan_epilogues_bit_exact(dev, restated, monkeypatch, plan, mode):
    import torch
    from vla_simd_b200 import EPI_ADD, EPI_ADD_RELU, EPI_RELU, ops
    monkeypatch.setenv("VLA_GEMM_PLAN", plan)
    M, N, K = 333, 320, 1408
    rng = np.random.default_rng(11)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float32)
    res = rng.standard_normal((M, N), dtype=np.float32)
    xq, xs = restated.quantize_rows(x)
    wqh, wsh = restated.quantize_rows(W)
    y = restated.dense_linear_i8_ref(xq, xs, wqh, wsh, b, K)
    flag = {"none": 0, "relu": EPI_RELU, "add": EPI_ADD, "add_relu": EPI_ADD_RELU}[mode]
    if mode == "relu":
        want = np.where(y < 0, np.float32(0), y)
    elif mode == "add":
        want = (res + y).astype(np.float32)
    elif mode == "add_relu":
        v = (y + res).astype(np.float32)
        want = np.where(v > 0, v, np.float32(0))
    else:
        want = y
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    # in place (out aliases the residual) with an absmax tap whose slots are
    # 30 rows: five slots per 128-row tile, so both the shared-memory and the
    # direct atomic paths of the split-K reduction run
    r = _t(res, dev)
    rows = 30
    am = torch.zeros((M + rows - 1) // rows, dtype=torch.int32, device=dev)
    ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=flag, res=r if flag & (EPI_ADD | EPI_ADD_RELU) else None,
                out=r, amax=am, amax_rows=rows)
    torch.cuda.synchronize()
    got = r.cpu().numpy()
    assert _bits_equal(got, want)
    rowmax = np.concatenate([np.abs(got).max(axis=1), np.zeros(am.numel() * rows - M, np.float32)])
    assert np.array_equal(am.cpu().numpy().view(np.float32), rowmax.reshape(-1, rows).max(axis=1))
    assert ops.device_status() == 0
