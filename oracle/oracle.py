"""TEST INFRASTRUCTURE ONLY: ctypes loaders for the two CPU oracles.

* ``restated()`` - this repository's C restatement of the reference's int8
  algorithm (oracle/i8_oracle.c -> oracle/_build/libi8_oracle.so).
* ``reference()`` - the reference's own sources compiled by oracle/Makefile
  (oracle/_ref/libvla_ref.so): its tcpu:: int8 / attention / norm / conv ops
  through ref_shim.cpp, and its full vla_act_* C ABI.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the library never does. The xorshift generator below restates the
reference test's RNG (tests/test_ops.cpp:31-40) so parity cases use the same
inputs as the reference's own op tests.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
RESTATED_SO = os.path.join(HERE, "_build", "libi8_oracle.so")
REFERENCE_SO = os.path.join(HERE, "_ref", "libvla_ref.so")
# the reference's own sources with their int8 op API defined over this
# repository's library (ref_cuda_backend.cpp): its models run their int8
# layers on the GPU
REFERENCE_CUDA_SO = os.path.join(HERE, "_ref", "libvla_ref_cuda.so")
SERVER_PY = os.path.join(HERE, "_ref", "vla_simd", "policy_server.py")

VP, I32, I64, F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def reference_dir() -> str | None:
    """The reference checkout: $VLA_REF_DIR, else a checkout named ``reference``
    beside this repository; None when neither holds the reference's sources."""
    cand = os.environ.get("VLA_REF_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isfile(os.path.join(cand, "include", "vla_simd.h")) else None


def build(reference: bool | None = None) -> None:
    """make the restatement (always) and the reference build (when its sources exist)."""
    targets = ["oracle"]
    ref = reference_dir()
    if reference is None:
        reference = ref is not None
    env = dict(os.environ)
    if reference:
        if ref is None:
            raise RuntimeError("the reference build needs its sources: set VLA_REF_DIR")
        targets.append("ref")
        # the reference over this repository's CUDA backend needs the product library
        if os.path.exists(os.path.join(os.path.dirname(HERE), "vla_simd_b200", "libvla_simd_b200.so")):
            targets.append("refcuda")
        env["REF"] = ref
    subprocess.run(["make", "-s", "-j8", "-C", HERE, *targets], check=True, env=env)


class Restated:
    def __init__(self):
        if not os.path.exists(RESTATED_SO):
            build(reference=False)
        l = ctypes.CDLL(RESTATED_SO)
        l.or_i8_kpad.restype = I32
        l.or_i8_kpad.argtypes = [I32]
        l.or_row_scale.restype = F32
        l.or_row_scale.argtypes = [F32]
        l.or_quantize_rows.argtypes = [VP, I32, I32, VP, I64, VP]
        l.or_pack_weights_i8.argtypes = [VP, VP, VP, I32, I32]
        l.or_gemm_i8_acc.argtypes = [VP, VP, I64, VP, I64, I32, I32, I32]
        l.or_dense_linear_i8_ref.argtypes = [VP, VP, I64, VP, VP, I64, VP, VP, I32, I32, I32]
        l.or_quantize_span_i8.argtypes = [VP, VP, ctypes.c_size_t, F32]
        l.or_tensor_scale.restype = F32
        l.or_tensor_scale.argtypes = [VP, ctypes.c_size_t, F32]
        l.or_conv2d_i8.argtypes = [VP, VP, VP, I64, VP, VP, I32, I32, I32, I32, I32, I32, I32, F32, VP, VP]
        self.l = l

    def quantize_rows(self, x, ld=None):
        x = np.ascontiguousarray(x, np.float32)
        rows, K = x.shape
        ld = ld or K
        q = np.zeros((rows, ld), np.int8)
        s = np.zeros(rows, np.float32)
        self.l.or_quantize_rows(_ptr(x), rows, K, _ptr(q), ld, _ptr(s))
        return q, s

    def pack_weights_panels(self, W):
        W = np.ascontiguousarray(W, np.float32)
        N, K = W.shape
        Kp = self.l.or_i8_kpad(K)
        buf = np.zeros(N * Kp + 4 * N, np.int8)
        s = np.zeros(N, np.float32)
        self.l.or_pack_weights_i8(_ptr(W), _ptr(buf), _ptr(s), N, K)
        return buf, s

    def gemm_acc(self, xq, wq, K):
        M, N = xq.shape[0], wq.shape[0]
        acc = np.zeros((M, N), np.int32)
        self.l.or_gemm_i8_acc(_ptr(acc), _ptr(np.ascontiguousarray(xq)), xq.shape[1],
                              _ptr(np.ascontiguousarray(wq)), wq.shape[1], M, N, K)
        return acc

    def dense_linear_i8_ref(self, xq, ascale, wq, wscale, bias, K):
        M, N = xq.shape[0], wq.shape[0]
        out = np.zeros((M, N), np.float32)
        self.l.or_dense_linear_i8_ref(_ptr(out), _ptr(np.ascontiguousarray(xq)), xq.shape[1],
                                      _ptr(np.ascontiguousarray(ascale, np.float32)),
                                      _ptr(np.ascontiguousarray(wq)), wq.shape[1],
                                      _ptr(np.ascontiguousarray(wscale, np.float32)),
                                      _ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)), M, N, K)
        return out

    def conv2d_i8(self, x, wq, wscale, bias, Cout, k, stride, pad, clip=1.0):
        x = np.ascontiguousarray(x, np.float32)
        H, W, Cin = x.shape
        Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
        out = np.zeros((Ho, Wo, Cout), np.float32)
        xs = np.zeros(H * W * Cin, np.int8)
        rs = np.zeros(k * k * Cin, np.int8)
        self.l.or_conv2d_i8(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(wq)), wq.shape[1],
                            _ptr(np.ascontiguousarray(wscale, np.float32)),
                            _ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                            H, W, Cin, Cout, k, stride, pad, clip, _ptr(xs), _ptr(rs))
        return out


class Reference:
    def __init__(self, path: str = REFERENCE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        l = ctypes.CDLL(path)
        self.path = path
        l.ref_nn_linear_forward.restype = I32
        l.ref_nn_linear_forward.argtypes = [VP, VP, I32, I32, VP, I32, VP, I32]
        l.ref_int8_gemm_available.restype = I32
        l.ref_i8_kpad.restype = I32
        l.ref_i8_kpad.argtypes = [I32]
        l.ref_packed_i8_words.restype = ctypes.c_ulonglong
        l.ref_packed_i8_words.argtypes = [I32, I32]
        l.ref_pack_weights_i8.argtypes = [VP, VP, VP, I32, I32]
        l.ref_quantize_act_i8.argtypes = [VP, VP, VP, I32, I32]
        l.ref_dense_linear_i8.argtypes = [VP, VP, VP, VP, VP, I32, I32, I32, VP, VP]
        l.ref_dense_linear_i8_pre.argtypes = [VP, VP, VP, VP, VP, VP, I32, I32, I32]
        l.ref_dense_linear_i8_ref.argtypes = [VP, VP, VP, VP, VP, VP, I32, I32, I32]
        l.ref_conv2d_i8.argtypes = [VP, VP, VP, VP, VP, I32, I32, I32, I32, I32, I32, I32]
        l.ref_layernorm.argtypes = [VP, VP, VP, VP, I32, I32, F32]
        l.ref_gqa_attention_masked.argtypes = [VP, VP, VP, VP, I32, I32, I32, I32, I32, F32, VP]
        l.ref_maxpool2d_relu.argtypes = [VP, VP, I32, I32, I32, I32, I32, I32]
        l.ref_relu.argtypes = [VP, I32]
        l.ref_dense_linear.argtypes = [VP, VP, VP, VP, I32, I32, I32]
        l.ref_rmsnorm.argtypes = [VP, VP, VP, I32, I32, F32]
        l.ref_rope_neox.argtypes = [VP, VP, I32, I32, I32, F32]
        l.ref_silu_gate.argtypes = [VP, VP, VP, I32]
        for n in ("silu", "gelu_tanh", "gelu_erf", "mish"):
            getattr(l, f"ref_{n}").argtypes = [VP, I32]
        l.ref_groupnorm.argtypes = [VP, VP, VP, VP, I32, I32, I32, F32, I32]
        l.ref_spatial_softmax.argtypes = [VP, VP, VP, I32, I32]
        l.ref_im2col1d.argtypes = [VP, VP, I32, I32, I32, I32, I32, I32]
        l.ref_conv_transpose1d.argtypes = [VP, VP, VP, VP, I32, I32, I32, I32, I32, I32]
        l.vla_act_load.restype = VP
        l.vla_act_load.argtypes = [ctypes.c_char_p]
        l.vla_act_free.argtypes = [VP]
        for n in ("chunk", "action_dim", "state_dim", "n_cams", "img_h", "img_w"):
            getattr(l, f"vla_act_{n}").restype = I32
            getattr(l, f"vla_act_{n}").argtypes = [VP]
        l.vla_act_predict.restype = I32
        l.vla_act_predict.argtypes = [VP, VP, VP, I32, VP]
        self.l = l

    def kpad(self, K):
        return self.l.ref_i8_kpad(K)

    def nn_linear_forward(self, W, bias, x, int8=True):
        """The reference's nn::Linear (Role::Gemm): init, init_int8 when asked, forward.
        Returns (out [seq, N], whether the layer took the int8 kernel)."""
        W = np.ascontiguousarray(W, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        N, K = W.shape
        out = np.zeros((x.shape[0], N), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        q = self.l.ref_nn_linear_forward(_ptr(W), _ptr(b), N, K, _ptr(x), x.shape[0], _ptr(out), 1 if int8 else 0)
        return out, bool(q)

    def pack_weights_i8(self, W):
        W = np.ascontiguousarray(W, np.float32)
        N, K = W.shape
        words = self.l.ref_packed_i8_words(N, K)
        buf = np.zeros(words * 4, np.int8)
        s = np.zeros(N, np.float32)
        self.l.ref_pack_weights_i8(_ptr(W), _ptr(buf), _ptr(s), N, K)
        return buf, s

    def quantize_act_i8(self, x):
        x = np.ascontiguousarray(x, np.float32)
        seq, K = x.shape
        q = np.zeros((seq, self.kpad(K)), np.int8)
        s = np.zeros(seq, np.float32)
        self.l.ref_quantize_act_i8(_ptr(x), _ptr(q), _ptr(s), seq, K)
        return q, s

    def dense_linear_i8_ref(self, xq, ascale, panels, wscale, bias, N, K):
        seq = xq.shape[0]
        out = np.zeros((seq, N), np.float32)
        self.l.ref_dense_linear_i8_ref(_ptr(out), _ptr(np.ascontiguousarray(xq)), _ptr(ascale), _ptr(panels),
                                       _ptr(wscale), _ptr(bias), seq, N, K)
        return out

    def dense_linear_i8(self, x, panels, wscale, bias, N):
        x = np.ascontiguousarray(x, np.float32)
        seq, K = x.shape
        out = np.zeros((seq, N), np.float32)
        xq = np.zeros((seq, self.kpad(K)), np.int8)
        s = np.zeros(seq, np.float32)
        self.l.ref_dense_linear_i8(_ptr(out), _ptr(x), _ptr(panels), _ptr(wscale), _ptr(bias), seq, N, K, _ptr(xq),
                                   _ptr(s))
        return out

    def conv2d_i8(self, x, panels, wscale, bias, Cout, k, stride, pad):
        x = np.ascontiguousarray(x, np.float32)
        H, W, Cin = x.shape
        Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
        out = np.zeros((Ho, Wo, Cout), np.float32)
        self.l.ref_conv2d_i8(_ptr(out), _ptr(x), _ptr(panels), _ptr(wscale), _ptr(bias), H, W, Cin, Cout, k, stride,
                             pad)
        return out

    def layernorm(self, x, w, b, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self.l.ref_layernorm(_ptr(out), _ptr(x), _ptr(w), _ptr(b), x.shape[0], x.shape[1], eps)
        return out

    def attention(self, Q, K, V, n_q, n_kv, head_dim, scale, mask=None):
        seq_q, seq_k = Q.shape[0], K.shape[0]
        out = np.zeros((seq_q, n_q * head_dim), np.float32)
        self.l.ref_gqa_attention_masked(_ptr(out), _ptr(np.ascontiguousarray(Q)), _ptr(np.ascontiguousarray(K)),
                                        _ptr(np.ascontiguousarray(V)), seq_q, seq_k, n_q, n_kv, head_dim, scale,
                                        _ptr(mask))
        return out

    def maxpool2d_relu(self, x, k=3, stride=2, pad=1):
        x = np.ascontiguousarray(x, np.float32)
        H, W, C = x.shape
        Ho, Wo = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
        out = np.zeros((Ho, Wo, C), np.float32)
        self.l.ref_maxpool2d_relu(_ptr(out), _ptr(x), H, W, C, k, stride, pad)
        return out

    def dense_linear(self, x, W, b):
        x = np.ascontiguousarray(x, np.float32)
        seq, K = x.shape
        N = W.shape[0]
        out = np.zeros((seq, N), np.float32)
        self.l.ref_dense_linear(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(W, np.float32)), _ptr(b), seq, N, K)
        return out

    # --- lm / conv ops of the other policy families (src/ops/lm_ops.h, conv_ops.h)
    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        self.l.ref_rmsnorm(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(w, np.float32)), x.shape[0], x.shape[1], eps)
        return out

    def rope_neox(self, x, pos, n_heads, head_dim, base):
        x = np.array(x, np.float32, copy=True, order="C")
        pos = np.ascontiguousarray(pos, np.int32)
        self.l.ref_rope_neox(_ptr(x), _ptr(pos), x.shape[0], n_heads, head_dim, base)
        return x

    def activation(self, name, x, u=None):
        x = np.array(x, np.float32, copy=True, order="C").ravel()
        if name == "silu_gate":
            out = np.zeros_like(x)
            self.l.ref_silu_gate(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(u, np.float32).ravel()), x.size)
            return out
        getattr(self.l, f"ref_{name}")(_ptr(x), x.size)
        return x

    def groupnorm(self, x, scale, bias, groups, eps, fuse_relu=False):
        x = np.ascontiguousarray(x, np.float32)
        P, C = x.shape
        out = np.zeros_like(x)
        self.l.ref_groupnorm(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(scale, np.float32)),
                             _ptr(np.ascontiguousarray(bias, np.float32)), P, C, groups, eps, 1 if fuse_relu else 0)
        return out

    def spatial_softmax(self, x, grid):
        x = np.ascontiguousarray(x, np.float32)
        P, C = x.shape
        out = np.zeros((C, 2), np.float32)
        self.l.ref_spatial_softmax(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(grid, np.float32)), P, C)
        return out

    def im2col1d(self, x, k, stride, pad):
        x = np.ascontiguousarray(x, np.float32)
        T, Cin = x.shape
        Tout = (T + 2 * pad - k) // stride + 1
        col = np.zeros((Tout, k * Cin), np.float32)
        self.l.ref_im2col1d(_ptr(col), _ptr(x), T, Cin, k, stride, pad, Tout)
        return col

    def conv_transpose1d(self, x, W, b, k, stride, pad):
        x = np.ascontiguousarray(x, np.float32)
        T, Cin = x.shape
        Cout = W.shape[-1]
        Tout = (T - 1) * stride - 2 * pad + k
        out = np.zeros((Tout, Cout), np.float32)
        self.l.ref_conv_transpose1d(_ptr(out), _ptr(x), _ptr(np.ascontiguousarray(W, np.float32)),
                                    _ptr(b) if b is not None else None, T, Cin, Cout, k, stride, pad)
        return out

    # --- policy level (the reference's own vla_act_* ABI)
    def act_predict(self, model_dir, frames, state, unnormalize=True):
        h = self.l.vla_act_load(model_dir.encode())
        if not h:
            raise RuntimeError("reference vla_act_load failed")
        try:
            chunk, ad = self.l.vla_act_chunk(h), self.l.vla_act_action_dim(h)
            out = np.zeros((chunk, ad), np.float32)
            fr = np.ascontiguousarray(frames, np.uint8)
            st = np.ascontiguousarray(state, np.float32)
            rc = self.l.vla_act_predict(h, _ptr(fr), _ptr(st), 1 if unnormalize else 0, _ptr(out))
            if rc != 0:
                raise RuntimeError(f"reference vla_act_predict rc={rc}")
            return out
        finally:
            self.l.vla_act_free(h)


    def dp_predict(self, model_dir, frames, state, noise, unnormalize=True):
        """The reference's vla_diffusion_predict (src/models/diffusion/diffusion_capi.cpp:57-72)
        on one query: frames [n_obs*n_cams, H, W, 3] uint8, state [n_obs, state_dim],
        noise [1 + steps, horizon, action_dim]; returns actions [n_action_steps, action_dim]."""
        l = self.l
        l.vla_diffusion_load.restype = VP
        l.vla_diffusion_load.argtypes = [ctypes.c_char_p]
        l.vla_diffusion_free.argtypes = [VP]
        for name in ("chunk", "action_dim"):
            getattr(l, f"vla_diffusion_{name}").argtypes = [VP]
        l.vla_diffusion_predict.argtypes = [VP, VP, VP, I32, VP, VP]
        h = l.vla_diffusion_load(model_dir.encode())
        if not h:
            raise RuntimeError("reference vla_diffusion_load failed")
        try:
            out = np.zeros((l.vla_diffusion_chunk(h), l.vla_diffusion_action_dim(h)), np.float32)
            fr = np.ascontiguousarray(frames, np.uint8)
            st = np.ascontiguousarray(state, np.float32)
            nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
            rc = l.vla_diffusion_predict(h, _ptr(fr), _ptr(st), 1 if unnormalize else 0, _ptr(out), _ptr(nz))
            if rc != 0:
                raise RuntimeError(f"reference vla_diffusion_predict rc={rc}")
            return out
        finally:
            l.vla_diffusion_free(h)


    def octo_predict(self, model_dir, tok_dir, primary, wrist, tmask, instruction, noise, z, seed=0,
                     unnormalize=True):
        """The reference's vla_octo_predict_ex (src/models/octo/octo_capi.cpp:40-58) on one
        query: primary [wnd, 256, 256, 3], wrist [wnd, 128, 128, 3] or None, tmask [wnd];
        noise [flat] and z [steps, flat], or both None (drawn from seed);
        returns actions [horizon, action_dim]."""
        l = self.l
        l.vla_octo_load.restype = VP
        l.vla_octo_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        l.vla_octo_free.argtypes = [VP]
        for name in ("horizon", "action_dim"):
            getattr(l, f"vla_octo_{name}").argtypes = [VP]
        l.vla_octo_predict_ex.argtypes = [VP, VP, VP, I32, VP, ctypes.c_char_p, VP, VP, ctypes.c_uint64, I32, VP]
        h = l.vla_octo_load(model_dir.encode(), tok_dir.encode())
        if not h:
            raise RuntimeError("reference vla_octo_load failed")
        try:
            out = np.zeros((l.vla_octo_horizon(h), l.vla_octo_action_dim(h)), np.float32)
            p = np.ascontiguousarray(primary, np.uint8)
            w = None if wrist is None else np.ascontiguousarray(wrist, np.uint8)
            tm = np.ascontiguousarray(tmask, np.uint8)
            nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
            zz = None if z is None else np.ascontiguousarray(z, np.float32)
            rc = l.vla_octo_predict_ex(h, _ptr(p), _ptr(w), p.shape[0], _ptr(tm), instruction.encode(), _ptr(nz),
                                       _ptr(zz), seed, 1 if unnormalize else 0, _ptr(out))
            if rc != 0:
                raise RuntimeError(f"reference vla_octo_predict_ex rc={rc}")
            return out
        finally:
            l.vla_octo_free(h)

    def octo_readout(self, model_dir, tok_dir, primary, wrist, tmask, instruction, d):
        """The readout embedding [d] the reference's diffusion head reads (ref_octo_shim.cpp)."""
        l = self.l
        l.ref_octo_readout.argtypes = [ctypes.c_char_p, ctypes.c_char_p, VP, VP, I32, VP, ctypes.c_char_p, VP]
        l.ref_octo_readout.restype = I32
        out = np.zeros(d, np.float32)
        p = np.ascontiguousarray(primary, np.uint8)
        w = None if wrist is None else np.ascontiguousarray(wrist, np.uint8)
        rc = l.ref_octo_readout(model_dir.encode(), tok_dir.encode(), _ptr(p), _ptr(w), p.shape[0],
                                _ptr(np.ascontiguousarray(tmask, np.uint8)), instruction.encode(), _ptr(out))
        if rc != 0:
            raise RuntimeError("ref_octo_readout failed")
        return out

    def t5_tokenize(self, tok_dir, text, max_len=16):
        """The reference tokenizer's ids of `text` (ref_octo_shim.cpp)."""
        l = self.l
        l.ref_t5_tokenize.argtypes = [ctypes.c_char_p, ctypes.c_char_p, I32, VP]
        l.ref_t5_tokenize.restype = I32
        ids = np.zeros(max_len, np.int32)
        if l.ref_t5_tokenize(tok_dir.encode(), text.encode(), max_len, _ptr(ids)) != 0:
            raise RuntimeError("ref_t5_tokenize failed")
        return ids

    def _smolvla_bind(self):
        l = self.l
        l.vla_smolvla_load.restype = VP
        l.vla_smolvla_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        l.vla_smolvla_free.argtypes = [VP]
        for name in ("chunk", "action_dim", "tok_maxlen"):
            getattr(l, f"vla_smolvla_{name}").argtypes = [VP]
        l.vla_smolvla_tokenize.argtypes = [VP, ctypes.c_char_p, VP, VP]
        l.vla_smolvla_predict_rtc.argtypes = [VP, VP, I32, I32, I32, VP, VP, I32, VP, VP, ctypes.c_uint64, VP, VP,
                                              I32, VP, F32]
        return l

    def smolvla_predict(self, model_dir, frames, instruction, state, noise, seed=0, prev=None, weights=None,
                        max_guidance=0.0):
        """The reference's vla_smolvla_tokenize + vla_smolvla_predict_rtc
        (src/models/smolvla/smolvla_capi.cpp:94-165) on one query: frames
        [n_views, h, w, 3] uint8 at the camera's resolution, the instruction
        string, raw state, noise [chunk, max_action_dim] or None (drawn from
        seed), optional RTC guidance (prev [n_prev, action_dim], weights
        [chunk]); returns actions [chunk, action_dim]."""
        l = self._smolvla_bind()
        h = l.vla_smolvla_load(model_dir.encode(), (model_dir + "/tok").encode())
        if not h:
            raise RuntimeError("reference vla_smolvla_load failed")
        try:
            n = l.vla_smolvla_tok_maxlen(h)
            ids, mask = np.zeros(n, np.int32), np.zeros(n, np.int32)
            if l.vla_smolvla_tokenize(h, instruction.encode(), _ptr(ids), _ptr(mask)) < 0:
                raise RuntimeError("reference vla_smolvla_tokenize failed")
            out = np.zeros((l.vla_smolvla_chunk(h), l.vla_smolvla_action_dim(h)), np.float32)
            fr = np.ascontiguousarray(frames, np.uint8)
            st = np.ascontiguousarray(state, np.float32)
            nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
            pv = None if prev is None else np.ascontiguousarray(prev, np.float32)
            wt = None if weights is None else np.ascontiguousarray(weights, np.float32)
            rc = l.vla_smolvla_predict_rtc(h, _ptr(fr), fr.shape[0], fr.shape[1], fr.shape[2], _ptr(ids), _ptr(mask),
                                           n, _ptr(st), _ptr(nz), seed, _ptr(out), _ptr(pv),
                                           0 if pv is None else pv.shape[0], _ptr(wt), max_guidance)
            if rc != 0:
                raise RuntimeError(f"reference vla_smolvla_predict_rtc rc={rc}")
            return out
        finally:
            l.vla_smolvla_free(h)

    def smolvla_tokenize(self, model_dir, text):
        """(ids, mask, n) of the reference's vla_smolvla_tokenize."""
        l = self._smolvla_bind()
        h = l.vla_smolvla_load(model_dir.encode(), (model_dir + "/tok").encode())
        if not h:
            raise RuntimeError("reference vla_smolvla_load failed")
        try:
            n = l.vla_smolvla_tok_maxlen(h)
            ids, mask = np.zeros(n, np.int32), np.zeros(n, np.int32)
            k = l.vla_smolvla_tokenize(h, text.encode(), _ptr(ids), _ptr(mask))
            return ids, mask, k
        finally:
            l.vla_smolvla_free(h)

    def dp_global_cond(self, model_dir, frames, state):
        """The global conditioning vector the reference builds for one DP query (ref_dp_shim.cpp)."""
        l = self.l
        l.ref_dp_global_cond.argtypes = [ctypes.c_char_p, VP, VP, VP]
        l.ref_dp_global_cond.restype = I32
        st = np.ascontiguousarray(state, np.float32)
        out = np.zeros(1 << 16, np.float32)
        rc = l.ref_dp_global_cond(model_dir.encode(), _ptr(np.ascontiguousarray(frames, np.uint8)), _ptr(st),
                                  _ptr(out))
        if rc != 0:
            raise RuntimeError("ref_dp_global_cond failed")
        return out

    def dp_backbone_stage(self, model_dir, frames, s, cam, stage):
        """One ResNet stage map of frame (s, cam) in the reference's DP encoder (ref_dp_shim.cpp)."""
        l = self.l
        l.ref_dp_backbone_stage.argtypes = [ctypes.c_char_p, VP, I32, I32, I32, VP, I64]
        l.ref_dp_backbone_stage.restype = I64
        out = np.zeros(1 << 24, np.float32)
        n = l.ref_dp_backbone_stage(model_dir.encode(), _ptr(np.ascontiguousarray(frames, np.uint8)), s, cam,
                                    stage, _ptr(out), out.size)
        if n < 0:
            raise RuntimeError("ref_dp_backbone_stage failed")
        return out[:n].copy()


def restated() -> Restated:
    return Restated()


def reference() -> Reference | None:
    """The compiled reference, or None when oracle/_ref was not built here."""
    try:
        return Reference()
    except (FileNotFoundError, OSError):
        return None


def reference_cuda() -> Reference | None:
    """The reference over this repository's CUDA backend, or None when not built."""
    try:
        return Reference(REFERENCE_CUDA_SO)
    except (FileNotFoundError, OSError):
        return None


class XorShift:
    """The reference op tests' generator (tests/test_ops.cpp:31-35): 24-bit uniform floats."""

    def __init__(self, seed: int = 0x243F6A8885A308D3):
        self.state = seed & 0xFFFFFFFFFFFFFFFF

    def uniform(self, n: int, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
        out = np.empty(n, np.float32)
        s = self.state
        M = 0xFFFFFFFFFFFFFFFF
        lo32, span = np.float32(lo), np.float32(hi) - np.float32(lo)
        for i in range(n):
            s ^= (s << 13) & M
            s ^= s >> 7
            s ^= (s << 17) & M
            r = np.float32((s >> 40) & 0xFFFFFF) / np.float32(16777216.0)
            out[i] = lo32 + span * r
        self.state = s
        return out
