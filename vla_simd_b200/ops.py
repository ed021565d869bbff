"""Op-level wrappers over include/vla_simd_cuda.h for torch CUDA tensors.

Each function mirrors one reference op (src/ops/quant_ops.h, lm_ops.h,
conv_ops.h) - same argument meaning, the outputs allocated here for
convenience - and launches on torch's current stream. torch supplies device
memory and the stream handle only; the compute is the library's kernels.
"""
from __future__ import annotations

import torch

from . import EPI_ACC, check, lib


def _p(t):
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def i8_ld(K: int) -> int:
    return int(lib().vla_cuda_i8_ld(K))


def quantize_act_i8(x: torch.Tensor, ld: int | None = None):
    """x [seq, K] fp32 -> (xq [seq, ld] int8, ascale [seq] fp32)."""
    seq, K = x.shape
    ld = ld or i8_ld(K)
    xq = torch.empty((seq, ld), dtype=torch.int8, device=x.device)
    s = torch.empty(seq, dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_quantize_act_i8(_p(x.contiguous()), _p(xq), _p(s), seq, K, ld, _stream()),
          "vla_cuda_quantize_act_i8")
    return xq, s


def pack_weights_i8(W: torch.Tensor, ld: int | None = None):
    """W [N, K] fp32 -> (Wq [N, ld] int8, wscale [N])."""
    N, K = W.shape
    ld = ld or i8_ld(K)
    q = torch.empty((N, ld), dtype=torch.int8, device=W.device)
    s = torch.empty(N, dtype=torch.float32, device=W.device)
    check(lib().vla_cuda_pack_weights_i8(_p(W.contiguous()), _p(q), _p(s), N, K, ld, _stream()),
          "vla_cuda_pack_weights_i8")
    return q, s


def gemm_i8(xq, ascale, Wq, wscale, K, bias=None, mode=0, res=None, out=None, amax=None, amax_rows=1,
            force_simt=False, ascale_per_row=True):
    """The W8A8 GEMM with its fused epilogue (vla_cuda_gemm_i8)."""
    M, N = xq.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32 if mode & EPI_ACC else torch.float32, device=xq.device)
    ldr = res.stride(0) if res is not None else 0
    check(lib().vla_cuda_gemm_i8(_p(out), out.stride(0), _p(xq), xq.stride(0), _p(ascale), 1 if ascale_per_row else 0,
                                 _p(Wq), Wq.stride(0), _p(wscale), _p(bias), _p(res), ldr, M, N, K, mode, _p(amax),
                                 amax_rows, 1 if force_simt else 0, _stream()), "vla_cuda_gemm_i8")
    return out


def gemm_i8_rowq_supported(M, N, K):
    return bool(lib().vla_cuda_gemm_i8_rowq_supported(int(M), int(N), int(K)))


def gemm_i8_rowq(xq, ascale, Wq, wscale, K, qamax, qsync, bias=None, relu=False):
    """The W8A8 GEMM (+ ReLU) with its output quantized per row for the next
    W8A8 GEMM (vla_cuda_gemm_i8_rowq): returns (q int8 [M, N], scale [M]).
    qamax [M] and qsync [2 * ceil(M / 128)] int32 (zeroed) are the caller's."""
    M, N = xq.shape[0], Wq.shape[0]
    q = torch.empty((M, N), dtype=torch.int8, device=xq.device)
    s = torch.empty(M, dtype=torch.float32, device=xq.device)
    check(lib().vla_cuda_gemm_i8_rowq(_p(q), N, _p(s), _p(xq), xq.stride(0), _p(ascale), _p(Wq), Wq.stride(0),
                                      _p(wscale), _p(bias), M, N, K, 1 if relu else 0, _p(qamax), _p(qsync),
                                      _stream()), "vla_cuda_gemm_i8_rowq")
    return q, s


def gemm_i8_splitk(xq, ascale, Wq, wscale, K, ws, counters, bias=None, mode=0, res=None, out=None):
    """The W8A8 GEMM with K split over independent CTAs (vla_cuda_gemm_i8_splitk):
    M <= 128 rows; ws int32 and counters int32 (zeroed) are the caller's workspace."""
    M, N = xq.shape[0], Wq.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.int32 if mode & EPI_ACC else torch.float32, device=xq.device)
    ldr = res.stride(0) if res is not None else 0
    check(lib().vla_cuda_gemm_i8_splitk(_p(out), out.stride(0), _p(xq), xq.stride(0), _p(ascale), _p(Wq), Wq.stride(0),
                                        _p(wscale), _p(bias), _p(res), ldr, M, N, K, mode, _p(ws), ws.numel(),
                                        _p(counters), counters.numel(), _stream()), "vla_cuda_gemm_i8_splitk")
    return out


def dense_linear_i8(x, Wq, wscale, bias=None):
    """tcpu::dense_linear_i8: fp32 x [seq, K] -> fp32 [seq, N], x quantized per token."""
    seq, K = x.shape
    N = Wq.shape[0]
    out = torch.empty((seq, N), dtype=torch.float32, device=x.device)
    xq = torch.empty((seq, i8_ld(K)), dtype=torch.int8, device=x.device)
    s = torch.empty(seq, dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_dense_linear_i8(_p(out), _p(x.contiguous()), _p(Wq), _p(wscale), _p(bias), seq, N, K,
                                         Wq.stride(0), _p(xq), _p(s), _stream()), "vla_cuda_dense_linear_i8")
    return out


def conv2d_i8(x, Wq, wscale, bias, Cout, k, stride, pad, clip=1.0, mode=0, res=None):
    """tcpu::conv2d_i8 over F NHWC frames: x [F, H, W, Cin] -> [F, Ho, Wo, Cout]."""
    F, H, W, Cin = x.shape
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    ldw = Wq.stride(0)
    out = torch.empty((F, Ho, Wo, Cout), dtype=torch.float32, device=x.device)
    col = torch.empty((F * Ho * Wo, ldw), dtype=torch.int8, device=x.device)
    rs = torch.empty(F * Ho * Wo, dtype=torch.float32, device=x.device)
    am = torch.zeros(F, dtype=torch.int32, device=x.device)
    check(lib().vla_cuda_conv2d_i8(_p(out), _p(x.contiguous()), F, H, W, Cin, _p(Wq), ldw, _p(wscale), _p(bias), Cout,
                                   k, stride, pad, clip, mode, _p(res), _p(col), _p(rs), _p(am), _stream()),
          "vla_cuda_conv2d_i8")
    return out


def layernorm(x, w, b, eps=1e-5):
    seq, H = x.shape
    out = torch.empty_like(x)
    check(lib().vla_cuda_layernorm(_p(out), _p(x.contiguous()), _p(w), _p(b), seq, H, eps, _stream()),
          "vla_cuda_layernorm")
    return out


def gqa_attention(Q, K, V, n_q, n_kv, scale, mask=None, head_dim=64):
    seq_q, seq_k = Q.shape[0], K.shape[0]
    out = torch.empty((seq_q, n_q * head_dim), dtype=torch.float32, device=Q.device)
    check(lib().vla_cuda_gqa_attention(_p(out), _p(Q.contiguous()), _p(K.contiguous()), _p(V.contiguous()), seq_q,
                                       seq_k, n_q, n_kv, head_dim, scale, _p(mask), _stream()),
          "vla_cuda_gqa_attention")
    return out


def gqa_attention_tc(Q, K, V, n_q, n_kv, scale, mask=None, head_dim=64):
    """The tensor-core (3xTF32 tcgen05) attention: same contract, not bit-identical."""
    seq_q, seq_k = Q.shape[0], K.shape[0]
    out = torch.empty((seq_q, n_q * head_dim), dtype=torch.float32, device=Q.device)
    check(lib().vla_cuda_gqa_attention_tc(_p(out), _p(Q.contiguous()), _p(K.contiguous()), _p(V.contiguous()),
                                          seq_q, seq_k, n_q, n_kv, head_dim, scale, _p(mask), _stream()),
          "vla_cuda_gqa_attention_tc")
    return out


def maxpool2d_relu(x, k=3, stride=2, pad=1):
    F, H, W, C = x.shape
    Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    out = torch.empty((F, Ho, Wo, C), dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_maxpool2d_relu(_p(out), _p(x.contiguous()), F, H, W, C, k, stride, pad, _stream()),
          "vla_cuda_maxpool2d_relu")
    return out


def dense_linear_f32(x, W, bias=None):
    """tcpu::dense_linear (fp32), the reference's summation order."""
    seq, K = x.shape
    N = W.shape[0]
    out = torch.empty((seq, N), dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_dense_linear_f32(_p(out), _p(x.contiguous()), _p(W.contiguous()), _p(bias), seq, N, K,
                                          _stream()), "vla_cuda_dense_linear_f32")
    return out


# ---- lm / conv ops of the other policy families (src/ops/lm_ops.h, conv_ops.h)

def rmsnorm(x, w, eps=1e-6):
    """tcpu::rmsnorm: sequential double sum of squares per row."""
    seq, hidden = x.shape
    out = torch.empty_like(x)
    check(lib().vla_cuda_rmsnorm(_p(out), _p(x.contiguous()), _p(w.contiguous()), seq, hidden, eps, _stream()),
          "vla_cuda_rmsnorm")
    return out


def rope_neox(x, pos, n_heads, head_dim, base=10000.0):
    """tcpu::rope_neox on a copy of x [seq, n_heads*head_dim]; pos int32 [seq]."""
    y = x.contiguous().clone()
    check(lib().vla_cuda_rope_neox(_p(y), _p(pos.to(torch.int32).contiguous()), y.shape[0], n_heads, head_dim, base,
                                   _stream()), "vla_cuda_rope_neox")
    return y


def activation(name, x, u=None):
    """tcpu::{silu_gate, silu, gelu_tanh, gelu_erf, relu, mish}; returns a new tensor."""
    x = x.contiguous()
    out = torch.empty_like(x)
    fn = getattr(lib(), f"vla_cuda_{name}")
    if name == "silu_gate":
        rc = fn(_p(out), _p(x), _p(u.contiguous()), x.numel(), _stream())
    else:
        rc = fn(_p(out), _p(x), x.numel(), _stream())
    check(rc, f"vla_cuda_{name}")
    return out


def groupnorm(x, scale, bias, groups, eps=1e-5, fuse_relu=False):
    """tcpu::groupnorm over x [n_pixels, C] (channels last)."""
    P, C = x.shape
    out = torch.empty_like(x)
    scratch = torch.empty(int(lib().vla_cuda_groupnorm_scratch_bytes(C)), dtype=torch.uint8, device=x.device)
    check(lib().vla_cuda_groupnorm(_p(out), _p(x.contiguous()), _p(scale.contiguous()), _p(bias.contiguous()), P, C,
                                   groups, eps, 1 if fuse_relu else 0, _p(scratch), _stream()), "vla_cuda_groupnorm")
    return out


def spatial_softmax(x, grid):
    """tcpu::spatial_softmax: x [n_pixels, C], grid [n_pixels, 2] -> [C, 2]."""
    P, C = x.shape
    out = torch.empty((C, 2), dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_spatial_softmax(_p(out), _p(x.contiguous()), _p(grid.contiguous()), P, C, _stream()),
          "vla_cuda_spatial_softmax")
    return out


def im2col1d(x, k, stride, pad):
    """tcpu::im2col1d: x [T, Cin] -> [Tout, k*Cin]."""
    T, Cin = x.shape
    Tout = (T + 2 * pad - k) // stride + 1
    col = torch.empty((Tout, k * Cin), dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_im2col1d(_p(col), _p(x.contiguous()), T, Cin, k, stride, pad, Tout, _stream()),
          "vla_cuda_im2col1d")
    return col


def conv_transpose1d(x, W, bias, k, stride, pad):
    """tcpu::conv_transpose1d: x [T, Cin], W [Cin, k, Cout] -> [(T-1)*stride-2*pad+k, Cout]."""
    T, Cin = x.shape
    Cout = W.shape[-1]
    Tout = (T - 1) * stride - 2 * pad + k
    out = torch.empty((Tout, Cout), dtype=torch.float32, device=x.device)
    check(lib().vla_cuda_conv_transpose1d(_p(out), _p(x.contiguous()), _p(W.contiguous()), _p(bias), T, Cin, Cout, k,
                                          stride, pad, _stream()), "vla_cuda_conv_transpose1d")
    return out


def device_status() -> int:
    return int(lib().vla_cuda_device_status())
