"""W8A8 GEMM on the B200 against the CPU oracle: int32 accumulators and fp32
outputs bit-identical, every epilogue, ragged shapes, both GPU kernels."""
import json
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, HERE)
from make_golden import GEMM_SHAPES, gemm_inputs, sha  # noqa: E402

GEMM = json.load(open(os.path.join(HERE, "gemm.json")))


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


@pytest.mark.parametrize("seq,N,K", GEMM_SHAPES)
@pytest.mark.parametrize("simt", [False, True])
def test_linear_matches_reference_fixtures(dev, seq, N, K, simt):
    import torch
    from vla_simd_b200 import EPI_ACC, ops
    x, W, b = gemm_inputs(seq, N, K)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    xq, xs = ops.quantize_act_i8(_t(x, dev))
    acc = ops.gemm_i8(xq, xs, wq, ws, K, mode=EPI_ACC, force_simt=simt)
    out = ops.gemm_i8(xq, xs, wq, ws, K, bias=_t(b, dev), force_simt=simt)
    torch.cuda.synchronize()
    g = GEMM[f"{seq}x{N}x{K}"]
    assert sha(xq.cpu().numpy()[:, :K]) == g["xq"]
    assert sha(xs.cpu().numpy()) == g["ascale"]
    assert sha(wq.cpu().numpy()[:, :K]) == g["wq"] and sha(ws.cpu().numpy()) == g["wscale"]
    assert sha(acc.cpu().numpy()) == g["acc"], "int32 accumulators differ from the reference"
    assert sha(out.cpu().numpy()) == g["out"], "fp32 outputs differ from the reference"
    assert ops.device_status() == 0


def test_dense_linear_i8_entry_point(dev, restated):
    """tcpu::dense_linear_i8 semantics: fp32 in, quantize per token, W8A8, fp32 out."""
    import torch
    from vla_simd_b200 import ops
    x, W, b = gemm_inputs(602, 3200, 512)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    out = ops.dense_linear_i8(_t(x, dev), wq, ws, _t(b, dev)).cpu().numpy()
    xq, xs = restated.quantize_rows(x)
    wqh, wsh = restated.quantize_rows(W)
    assert _bits_equal(out, restated.dense_linear_i8_ref(xq, xs, wqh, wsh, b, 512))


RAGGED = [(1, 16, 1), (1, 16, 16), (127, 48, 17), (128, 64, 128), (129, 272, 129), (1000, 96, 15),
          (3, 32, 12288), (640, 1024, 640), (2, 512, 3200), (4800, 128, 1152)]


@pytest.mark.parametrize("M,N,K", RAGGED)
def test_ragged_shapes_int32_exact(dev, restated, M, N, K):
    import torch
    from vla_simd_b200 import EPI_ACC, ops
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ld = ops.i8_ld(K)
    xpad = np.zeros((M, ld), np.int8)
    xpad[:, :K] = xq
    wpad = np.full((N, ld), 77, np.int8)     # bytes past K must be ignored
    wpad[:, :K] = wq
    one = torch.ones(max(M, N), device=dev)
    acc = ops.gemm_i8(_t(xpad, dev), one, _t(wpad, dev), one, K, mode=EPI_ACC)
    torch.cuda.synchronize()
    assert np.array_equal(acc.cpu().numpy(), restated.gemm_acc(xq, wq, K))


@pytest.mark.parametrize("mode", ["relu", "add", "add_relu"])
def test_epilogues_bit_exact(dev, restated, mode):
    import torch
    from vla_simd_b200 import EPI_ADD, EPI_ADD_RELU, EPI_RELU, ops
    M, N, K = 300, 512, 512
    x, W, b = gemm_inputs(M, N, K, seed=3)
    res = np.random.default_rng(4).standard_normal((M, N), dtype=np.float32)
    xq, xs = restated.quantize_rows(x)
    wqh, wsh = restated.quantize_rows(W)
    y = restated.dense_linear_i8_ref(xq, xs, wqh, wsh, b, K)
    if mode == "relu":
        want, flag = np.where(y < 0, np.float32(0), y), EPI_RELU
    elif mode == "add":
        want, flag = (res + y).astype(np.float32), EPI_ADD
    else:
        v = (y + res).astype(np.float32)
        want, flag = np.where(v > 0, v, np.float32(0)), EPI_ADD_RELU
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    r = _t(res, dev)
    out = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=flag, res=r)
    # in place (out aliases the residual), as the encoder's x += W x does
    r2 = _t(res, dev)
    ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=flag, res=r2, out=r2)
    torch.cuda.synchronize()
    assert _bits_equal(out.cpu().numpy(), want)
    assert _bits_equal(r2.cpu().numpy(), want)


def test_strided_output_and_per_tensor_scale(dev, restated):
    """Writing rows into a wider buffer at an offset (token assembly), one
    activation scale for every row (conv per-tensor quantization)."""
    import torch
    from vla_simd_b200 import ops
    M, N, K, ldo, off = 300, 512, 512, 512, 2
    x, W, b = gemm_inputs(M, N, K, seed=5)
    xq, _ = restated.quantize_rows(x)
    s = np.float32(0.0123)
    wqh, wsh = restated.quantize_rows(W)
    want = restated.dense_linear_i8_ref(xq, np.full(M, s, np.float32), wqh, wsh, b, K)
    big = torch.full((M + off, ldo), -7.0, device=dev)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    ops.gemm_i8(_t(xq, dev), torch.tensor([s], device=dev), wq, ws, K, bias=_t(b, dev), out=big[off:],
                ascale_per_row=False)
    torch.cuda.synchronize()
    got = big.cpu().numpy()
    assert (got[:off] == -7.0).all()
    assert _bits_equal(got[off:], want)


def test_absmax_tap(dev, restated):
    import torch
    from vla_simd_b200 import EPI_RELU, ops
    M, N, K, rows = 600, 256, 512, 300
    x, W, b = gemm_inputs(M, N, K, seed=6)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    dq, ds = ops.quantize_act_i8(_t(x, dev))
    am = torch.zeros(M // rows, dtype=torch.int32, device=dev)
    out = ops.gemm_i8(dq, ds, wq, ws, K, bias=_t(b, dev), mode=EPI_RELU, amax=am, amax_rows=rows)
    torch.cuda.synchronize()
    o = np.abs(out.cpu().numpy()).reshape(M // rows, -1).max(axis=1)
    assert np.array_equal(am.cpu().numpy().view(np.float32), o)


def test_host_pointer_shims_take_the_reference_panel_layout(restated):
    """vla_tcpu_* take the reference's own CPU layouts and give its results."""
    import ctypes
    from vla_simd_b200 import lib
    L = lib()
    seq, N, K = 50, 768, 1027
    x, W, b = gemm_inputs(seq, N, K)
    panels, ws = restated.pack_weights_panels(W)
    mine_p = np.zeros_like(panels)
    mine_s = np.zeros_like(ws)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    assert L.vla_tcpu_pack_weights_i8(P(W), P(mine_p), P(mine_s), N, K) == 0
    assert np.array_equal(mine_p, panels) and np.array_equal(mine_s, ws)
    Kp = (K + 3) & ~3
    out = np.zeros((seq, N), np.float32)
    xq = np.zeros((seq, Kp), np.int8)
    xs = np.zeros(seq, np.float32)
    assert L.vla_tcpu_dense_linear_i8(P(out), P(x), P(panels), P(ws), P(b), seq, N, K, P(xq), P(xs)) == 0
    q_ref, s_ref = restated.quantize_rows(x, ld=Kp)
    assert np.array_equal(xq, q_ref) and np.array_equal(xs, s_ref)
    wq, wsr = restated.quantize_rows(W)
    assert _bits_equal(out, restated.dense_linear_i8_ref(q_ref[:, :K], s_ref, wq, wsr, b, K))


SPLITK_SHAPES = [(16, 2048, 10240), (16, 512, 2560), (8, 1024, 5120), (4, 1024, 20480), (128, 384, 4096),
                 (1, 64, 1000), (77, 4096, 4096), (16, 16, 130)]


@pytest.mark.parametrize("reducer", ["every_cta", "last_cta"])
@pytest.mark.parametrize("M,N,K", SPLITK_SHAPES)
def test_splitk_workspace_gemm_matches_oracle(dev, restated, M, N, K, reducer):
    """K split over independent CTAs (workspace reduction): the same int32 sums
    and fp32 outputs as the oracle and the ordinary kernels, every epilogue; the
    counters are left zero, so a second call gives the same bits. With two
    counters per output tile the CTAs (all resident, a cooperative launch) each
    reduce rows after all have written; with one, the last to arrive reduces."""
    import torch
    from vla_simd_b200 import EPI_ACC, EPI_ADD, EPI_RELU, ops
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    x = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    b = (rng.standard_normal(N, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    r = rng.standard_normal((M, N), dtype=np.float32)
    wq, ws = ops.pack_weights_i8(_t(W, dev))
    xq, xs = ops.quantize_act_i8(_t(x, dev))
    work = torch.empty(148 * 128 * 128, dtype=torch.int32, device=dev)
    n_tiles = -(-N // (128 if N >= 1024 else 64 if N >= 256 else 32))
    counters = torch.zeros(4096 if reducer == "every_cta" else n_tiles, dtype=torch.int32, device=dev)
    acc = ops.gemm_i8_splitk(xq, xs, wq, ws, K, work, counters, mode=EPI_ACC)
    out = ops.gemm_i8_splitk(xq, xs, wq, ws, K, work, counters, bias=_t(b, dev))
    relu = ops.gemm_i8_splitk(xq, xs, wq, ws, K, work, counters, bias=_t(b, dev), mode=EPI_RELU)
    add = ops.gemm_i8_splitk(xq, xs, wq, ws, K, work, counters, bias=_t(b, dev), mode=EPI_ADD, res=_t(r, dev))
    again = ops.gemm_i8_splitk(xq, xs, wq, ws, K, work, counters, bias=_t(b, dev))
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert int(counters.abs().sum().item()) == 0, "arrival counters not reset"
    xqh, xsh = restated.quantize_rows(x)
    wqh, wsh = restated.quantize_rows(W)
    assert np.array_equal(acc.cpu().numpy(), restated.gemm_acc(xqh, wqh, K))
    want = restated.dense_linear_i8_ref(xqh, xsh, wqh, wsh, b, K)
    assert _bits_equal(out.cpu().numpy(), want)
    assert _bits_equal(again.cpu().numpy(), want)
    assert _bits_equal(relu.cpu().numpy(), ops.gemm_i8(xq, xs, wq, ws, K, bias=_t(b, dev), mode=EPI_RELU).cpu().numpy())
    assert _bits_equal(add.cpu().numpy(),
                       ops.gemm_i8(xq, xs, wq, ws, K, bias=_t(b, dev), mode=EPI_ADD, res=_t(r, dev)).cpu().numpy())
