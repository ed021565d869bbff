"""The slab W8A8 GEMM (one 128-row x bn-column output slab per CTA, the A tile
resident, B streamed in slices, TMA-store epilogue) gives the reference's bits.

VLA_GEMM_SLAB=<bn>:<sl>[:<stages>] forces a slab shape (columns per CTA, B
slice rows = MMA N, B slices in flight); every shape must reproduce
dense_linear_i8_ref (src/hal/common/gemm_i8.cpp:262-281) bit for bit, with
every epilogue, the residual aliasing the output, the absmax tap, ragged M / N
/ K and a strided output. The default plan routes the policies' one-wave
linears here, so the policy tests cover it as well.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# <bn>:<sl>[:<stages>]
SLABS = ["32:32", "64:32", "96:32", "128:32", "256:32", "64:64", "128:64", "256:128", "128:32:1", "256:32:2",
         "192:64:1"]


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


def _inputs(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float32)
    res = rng.standard_normal((M, N), dtype=np.float32)
    return x, W, b, res


def _want(restated, x, W, b, res, mode):
    K = x.shape[1]
    xq, xs = restated.quantize_rows(x)
    wqh, wsh = restated.quantize_rows(W)
    y = restated.dense_linear_i8_ref(xq, xs, wqh, wsh, b, K)
    if mode == "relu":
        return np.where(y < 0, np.float32(0), y)
    if mode == "add":
        return (res + y).astype(np.float32)
    if mode == "add_relu":
        v = (y + res).astype(np.float32)
        return np.where(v > 0, v, np.float32(0))
    return y


@pytest.mark.parametrize("slab", SLABS)
@pytest.mark.parametrize("M,N,K", [(602, 3200, 512), (1, 48, 129), (100, 512, 512), (333, 272, 1000),
                                   (130, 96, 1024), (77, 33, 40)])
def test_slab_shapes_bit_exact(dev, restated, monkeypatch, slab, M, N, K):
    from vla_simd_b200 import ops
    monkeypatch.setenv("VLA_GEMM_SLAB", slab)
    x, W, b, _ = _inputs(M, N, K, seed=M + 5 * N + 11 * K)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    out = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev))
    import torch
    torch.cuda.synchronize()
    assert _bits_equal(out.cpu().numpy(), _want(restated, x, W, b, None, "none"))
    assert ops.device_status() == 0


@pytest.mark.parametrize("slab", ["128:32", "64:64", "256:32:2", "default"])
@pytest.mark.parametrize("mode", ["none", "relu", "add", "add_relu"])
def test_slab_epilogues_in_place_with_absmax(dev, restated, monkeypatch, slab, mode):
    import torch
    from vla_simd_b200 import EPI_ADD, EPI_ADD_RELU, EPI_RELU, ops
    if slab != "default":
        monkeypatch.setenv("VLA_GEMM_SLAB", slab)
    M, N, K = 333, 320, 768
    x, W, b, res = _inputs(M, N, K, seed=21)
    want = _want(restated, x, W, b, res, mode)
    flag = {"none": 0, "relu": EPI_RELU, "add": EPI_ADD, "add_relu": EPI_ADD_RELU}[mode]
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    r = _t(res, dev)
    for rows in (1, 30, 1000):     # per row (ACT's FFN tap), a few slots per tile, one slot
        r.copy_(_t(res, dev))
        am = torch.zeros((M + rows - 1) // rows, dtype=torch.int32, device=dev)
        ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=flag,
                    res=r if flag & (EPI_ADD | EPI_ADD_RELU) else None, out=r, amax=am, amax_rows=rows)
        torch.cuda.synchronize()
        got = r.cpu().numpy()
        assert _bits_equal(got, want)
        rowmax = np.concatenate([np.abs(got).max(axis=1), np.zeros(am.numel() * rows - M, np.float32)])
        assert np.array_equal(am.cpu().numpy().view(np.float32), rowmax.reshape(-1, rows).max(axis=1))
    assert ops.device_status() == 0


def test_slab_strided_output_leaves_the_gaps(dev, restated, monkeypatch):
    """ldo > N: the TMA stores write the N columns of each row and nothing past them."""
    import torch
    from vla_simd_b200 import ops
    monkeypatch.setenv("VLA_GEMM_SLAB", "64:32")
    M, N, K, ldo = 150, 100, 256, 132
    x, W, b, _ = _inputs(M, N, K, seed=3)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    big = torch.full((M, ldo), -7.0, device=dev)
    ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), out=big)
    torch.cuda.synchronize()
    got = big.cpu().numpy()
    assert (got[:, N:] == -7.0).all()
    assert _bits_equal(got[:, :N], _want(restated, x, W, b, None, "none"))


def test_default_plan_takes_the_slab_and_matches_forced_persistent(dev, monkeypatch):
    """The ACT FFN shape under the default plan (slab) and a forced persistent plan give the same bits."""
    import torch
    from vla_simd_b200 import EPI_RELU, ops
    M, N, K = 602, 3200, 512
    x, W, b, _ = _inputs(M, N, K, seed=9)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    a = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=EPI_RELU)
    monkeypatch.setenv("VLA_GEMM_PLAN", "128:1")
    c = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=EPI_RELU)
    torch.cuda.synchronize()
    assert _bits_equal(a.cpu().numpy(), c.cpu().numpy())


@pytest.mark.parametrize("M,N,K", [(602, 3200, 512), (100, 3200, 512), (1, 64, 129), (130, 96, 1024),
                                   (333, 256, 1000)])
@pytest.mark.parametrize("relu", [False, True])
def test_rowq_output_equals_gemm_then_row_quantizer(dev, M, N, K, relu):
    """The GEMM writing its output already quantized per row (the FFN
    up-projection's int8 hidden for the down-projection) gives exactly the
    int8 rows and scales that the fp32 GEMM followed by the row quantizer give;
    twice in a row (its counters and absmax slots are left zero for the next
    call)."""
    import torch
    from vla_simd_b200 import ops, EPI_RELU
    if not ops.gemm_i8_rowq_supported(M, N, K):
        pytest.skip("not one wave of slab CTAs on this device")
    x, W, b, _ = _inputs(M, N, K, seed=3 * M + N + K)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    y = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=EPI_RELU if relu else 0)
    q_ref, s_ref = ops.quantize_act_i8(y, ld=N)
    qamax = torch.zeros(M, dtype=torch.int32, device=dev)
    qsync = torch.zeros(2 * ((M + 127) // 128), dtype=torch.int32, device=dev)
    for _ in range(2):
        q, s = ops.gemm_i8_rowq(dq, ds, wq, ws, K, qamax, qsync, bias=_t(b, dev), relu=relu)
        torch.cuda.synchronize()
        assert np.array_equal(q.cpu().numpy(), q_ref.cpu().numpy())
        assert _bits_equal(s.cpu().numpy(), s_ref.cpu().numpy())
        assert int(qamax.abs().sum()) == 0 and int(qsync.abs().sum()) == 0
    assert ops.device_status() == 0
