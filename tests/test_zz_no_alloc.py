"""vla_cuda_dense_linear_i8_noalloc against the allocating entry point.

The no-alloc variant exists for callers that may not allocate device memory
(a real-time control loop that cannot afford cudaMalloc's device-wide
synchronization, or a host framework that owns all GPU memory). It must give
exactly the result of vla_cuda_dense_linear_i8, whose scratch the caller
passes, and keep doing so on back-to-back calls that reuse its one static
scratch array. This file is collected last so a failure here cannot hide any
other test's result; it passes alone in a fresh process as well.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

VLA_OK, VLA_ERR_ARG, VLA_ERR_SHAPE = 0, -1, -2


def _case(torch, dev, seq, N, K, seed):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((seq, K), dtype=np.float32)).to(dev)
    W = torch.from_numpy((rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)).to(dev)
    b = torch.from_numpy((rng.standard_normal(N, dtype=np.float32) * 0.01).astype(np.float32)).to(dev)
    return x, W, b


def test_noalloc_linear_equals_allocating_entry_point():
    import torch
    from vla_simd_b200 import lib, ops
    L = lib()
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    # ACT's FFN input (602 x 512 -> 3200) and its widest one (602 x 3200 -> 512)
    for seq, N, K, seed in [(602, 3200, 512, 1), (602, 512, 3200, 2), (7, 48, 1027, 3)]:
        x, W, b = _case(torch, dev, seq, N, K, seed)
        wq, ws = ops.pack_weights_i8(W)
        want = ops.dense_linear_i8(x, wq, ws, b)   # caller-owned scratch
        for _ in range(2):                         # two calls in a row share the static scratch
            out = torch.full((seq, N), float("nan"), device=dev)
            rc = L.vla_cuda_dense_linear_i8_noalloc(out.data_ptr(), x.data_ptr(), wq.data_ptr(), ws.data_ptr(),
                                                    b.data_ptr(), seq, N, K, wq.stride(0), stream)
            assert rc == VLA_OK
            torch.cuda.synchronize()
            # bit-identical: the tolerance these W8A8 tests use
            assert torch.equal(out.view(torch.int32), want.view(torch.int32))
    assert ops.device_status() == 0


def test_noalloc_at_the_scratch_limit():
    """The largest call that fits the 2 MiB array runs and matches; one more row is refused.

    Scratch need = seq * ceil16(K) rounded up to 256 bytes, plus 4 * seq. At
    K = 512 that is 516 * seq: 4064 rows need 2,097,024 bytes (128 under the
    limit), 4065 rows 2,097,540 (388 over). No (seq, K) needs exactly 2 MiB:
    it would take 64 * a * (ceil16(K) + 4) == 2**21 with ceil16(K) + 4 four
    times an odd number."""
    import torch
    from vla_simd_b200 import lib, ops
    L = lib()
    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    stream = torch.cuda.current_stream().cuda_stream
    seq, N, K = 4064, 64, 512
    x, W, b = _case(torch, dev, seq + 1, N, K, 4)
    wq, ws = ops.pack_weights_i8(W)
    want = ops.dense_linear_i8(x[:seq], wq, ws, b)
    out = torch.full((seq + 1, N), float("nan"), device=dev)
    rc = L.vla_cuda_dense_linear_i8_noalloc(out.data_ptr(), x.data_ptr(), wq.data_ptr(), ws.data_ptr(),
                                            b.data_ptr(), seq, N, K, wq.stride(0), stream)
    assert rc == VLA_OK
    torch.cuda.synchronize()
    assert torch.equal(out[:seq].view(torch.int32), want.view(torch.int32))
    assert torch.isnan(out[seq]).all()
    rc = L.vla_cuda_dense_linear_i8_noalloc(out.data_ptr(), x.data_ptr(), wq.data_ptr(), ws.data_ptr(),
                                            b.data_ptr(), seq + 1, N, K, wq.stride(0), stream)
    assert rc == VLA_ERR_SHAPE


def test_noalloc_on_a_second_device():
    """Each device has its own copy of the array: a call on device 1 after device 0 matches too."""
    import torch
    from vla_simd_b200 import lib, ops
    if torch.cuda.device_count() < 2:
        pytest.skip("one visible GPU")
    L = lib()
    for d in (0, 1, 0):
        torch.cuda.set_device(d)
        dev = torch.device("cuda", d)
        stream = torch.cuda.current_stream().cuda_stream
        x, W, b = _case(torch, dev, 100, 512, 512, 5 + d)
        wq, ws = ops.pack_weights_i8(W)
        want = ops.dense_linear_i8(x, wq, ws, b)
        out = torch.empty((100, 512), device=dev)
        rc = L.vla_cuda_dense_linear_i8_noalloc(out.data_ptr(), x.data_ptr(), wq.data_ptr(), ws.data_ptr(),
                                                b.data_ptr(), 100, 512, 512, wq.stride(0), stream)
        assert rc == VLA_OK
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), want.view(torch.int32))
    torch.cuda.set_device(0)


def test_noalloc_rejects_calls_beyond_its_scratch():
    import ctypes
    from vla_simd_b200 import lib
    L = lib()
    fake = ctypes.c_void_p(256)   # never dereferenced: the size check comes first
    # 4096 x 4096 int8 activations = 16 MiB, far past the 2 MiB array
    assert L.vla_cuda_dense_linear_i8_noalloc(fake, fake, fake, fake, None, 4096, 64, 4096, 4096, None) \
        == VLA_ERR_SHAPE
    assert L.vla_cuda_dense_linear_i8_noalloc(None, fake, fake, fake, None, 4, 64, 64, 64, None) == VLA_ERR_ARG
