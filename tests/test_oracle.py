"""The C restatement (oracle/i8_oracle.c) against the reference's own compiled
int8 code (oracle/_ref), bit for bit - this pins the oracle the GPU parity
tests use. Cases follow the reference's op tests (tests/test_ops.cpp:93-157):
quantizer edge magnitudes and widths, and the five GEMM shapes."""
import numpy as np
import pytest

from oracle.oracle import XorShift

SHAPES = [(1, 16, 3), (7, 48, 64), (50, 768, 1027), (13, 64, 17), (257, 96, 48)]


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint8)


@pytest.mark.parametrize("mag", [0.0, np.float32(1e-45), np.float32(1e-37), 1.0])
@pytest.mark.parametrize("width", [3, 16, 33])
def test_quantizer_edges(restated, mag, width):
    x = np.array([(-1 if i % 2 else 1) * mag for i in range(width)], np.float32)[None, :]
    q, s = restated.quantize_rows(x, ld=(width + 3) & ~3)
    assert np.isfinite(s[0]) and s[0] > 0
    assert (q[0, :width] >= -127).all()
    assert (np.abs(q[0, :width].astype(np.float64) * s[0] - x[0]) <= s[0] * 0.51).all()
    assert (q[0, width:] == 0).all()


@pytest.mark.parametrize("mag", [0.0, np.float32(1e-45), np.float32(1e-37), 1.0])
@pytest.mark.parametrize("width", [3, 16, 33])
def test_quantizer_edges_match_reference(restated, reference, mag, width):
    x = np.array([(-1 if i % 2 else 1) * mag for i in range(width)], np.float32)[None, :]
    q_ref, s_ref = reference.quantize_act_i8(x)
    q, s = restated.quantize_rows(x, ld=q_ref.shape[1])
    assert np.array_equal(q, q_ref) and np.array_equal(_bits(s), _bits(s_ref))
    W = np.full((16, width), mag, np.float32)
    p_ref, ws_ref = reference.pack_weights_i8(W)
    p, ws = restated.pack_weights_panels(W)
    assert np.array_equal(p, p_ref) and np.array_equal(_bits(ws), _bits(ws_ref))


@pytest.mark.parametrize("seq,N,K", SHAPES)
def test_int8_path_matches_reference(restated, reference, seq, N, K):
    g = XorShift()
    x = g.uniform(seq * K).reshape(seq, K)
    W = g.uniform(N * K, -0.2, 0.2).reshape(N, K)
    b = g.uniform(N)
    # activation quantizer
    q_ref, s_ref = reference.quantize_act_i8(x)
    q, s = restated.quantize_rows(x, ld=q_ref.shape[1])
    assert np.array_equal(q, q_ref) and np.array_equal(_bits(s), _bits(s_ref))
    if N % 16:
        return
    # weight packer: panel layout, scales and int32 row sums
    p_ref, ws_ref = reference.pack_weights_i8(W)
    p, ws = restated.pack_weights_panels(W)
    assert np.array_equal(p, p_ref) and np.array_equal(_bits(ws), _bits(ws_ref))
    # scalar oracle, and the AVX-VNNI kernel the reference dispatches to here
    y_ref = reference.dense_linear_i8_ref(q_ref, s_ref, p_ref, ws_ref, b, N, K)
    wq, wsr = restated.quantize_rows(W)
    y = restated.dense_linear_i8_ref(q[:, :K], s, wq, wsr, b, K)
    assert np.array_equal(_bits(y), _bits(y_ref))
    y_full = reference.dense_linear_i8(x, p_ref, ws_ref, b, N)
    assert np.array_equal(_bits(y_full), _bits(y_ref))


@pytest.mark.parametrize("seq,N,K", SHAPES)
def test_int8_accuracy_vs_double(restated, seq, N, K):
    """tests/test_ops.cpp:153: scaled error of the int8 linear <= 2e-2."""
    if N % 16:
        pytest.skip("int8 linears need N % 16 == 0")
    g = XorShift()
    x = g.uniform(seq * K).reshape(seq, K)
    W = g.uniform(N * K, -0.2, 0.2).reshape(N, K)
    b = g.uniform(N)
    q, s = restated.quantize_rows(x)
    wq, ws = restated.quantize_rows(W)
    y = restated.dense_linear_i8_ref(q, s, wq, ws, b, K).astype(np.float64)
    ref = x.astype(np.float64) @ W.astype(np.float64).T + b
    mag = np.abs(x.astype(np.float64)) @ np.abs(W.astype(np.float64)).T + np.abs(b)
    assert (np.abs(y - ref) / (mag + 1e-30)).max() <= 2e-2


def test_int32_accumulators_exact(restated):
    """acc = sum_k xq*wq at the ACT FFN shape, against a numpy int64 product."""
    rng = np.random.default_rng(3)
    M, N, K = 64, 96, 3200
    xq = rng.integers(-127, 128, (M, K), dtype=np.int8)
    wq = rng.integers(-127, 128, (N, K), dtype=np.int8)
    acc = restated.gemm_acc(xq, wq, K)
    assert np.array_equal(acc, (xq.astype(np.int64) @ wq.astype(np.int64).T).astype(np.int32))


@pytest.mark.parametrize("H,W,Cin,Cout,k,st,pd", [(30, 30, 3, 64, 7, 2, 3), (28, 28, 64, 64, 3, 1, 1),
                                                  (15, 15, 64, 128, 3, 2, 1), (9, 11, 32, 16, 1, 2, 0)])
def test_conv2d_i8_matches_reference(restated, reference, H, W, Cin, Cout, k, st, pd):
    g = XorShift(0x1234567)
    x = g.uniform(H * W * Cin).reshape(H, W, Cin)
    Wt = g.uniform(Cout * k * k * Cin, -0.1, 0.1).reshape(Cout, k * k * Cin)
    b = g.uniform(Cout)
    p_ref, ws_ref = reference.pack_weights_i8(Wt)
    y_ref = reference.conv2d_i8(x, p_ref, ws_ref, b, Cout, k, st, pd)
    wq, ws = restated.quantize_rows(Wt)
    y = restated.conv2d_i8(x, wq, ws, b, Cout, k, st, pd)
    assert np.array_equal(_bits(y), _bits(y_ref))
