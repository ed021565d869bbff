"""vla_simd_b200: the B200 (sm_100a) backend of vla.simd's W8A8 policy path.

The product is ``libvla_simd_b200.so`` (CUDA kernels + the C ABI of
``include/vla_simd.h`` and ``include/vla_simd_cuda.h``). This package only loads
it with ctypes and mirrors the reference's Python-side interface:

* :class:`ActPolicy` - the reference server's ``ActEngine`` binding
  (vla_simd/policy_server.py:276-307): uint8 frames + state in, actions out.
* :class:`DiffusionPolicy` - the ``vla_diffusion_*`` ABI: an observation
  history (frames + states) and the sampler's noise in, an action chunk out;
  optionally a batch of independent queries per call.
* :class:`SmolvlaPolicy` - the ``vla_smolvla_*`` ABI: camera frames, an
  instruction, the robot state and the flow-matching noise in, an action chunk
  out (optionally with real-time-chunking guidance, and batches of queries).
* :class:`OctoPolicy` - the ``vla_octo_*`` ABI: a window of primary / wrist
  frames, a language instruction and the DDPM noise in, an action chunk out;
  optionally a batch of independent queries per call.
* ``ops`` - device-pointer wrappers over the op-level ABI taking torch CUDA
  tensors (torch is only the allocator / stream provider here).

There is no CPU fallback: importing works without a GPU, but every call needs
the compiled library and a B200, and fails loudly otherwise.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

__all__ = ["LIB_PATH", "lib", "ActPolicy", "DiffusionPolicy", "VlaError"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libvla_simd_b200.so")

VLA_OK, VLA_ERR_ARG, VLA_ERR_SHAPE, VLA_ERR_EXCEPTION, VLA_ERR_DEVICE = 0, -1, -2, -3, -4
EPI_RELU, EPI_ADD, EPI_ADD_RELU, EPI_ACC = 1, 2, 4, 8

U8P = ctypes.POINTER(ctypes.c_uint8)
F32P = ctypes.POINTER(ctypes.c_float)
VP = ctypes.c_void_p
I32, I64, F32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float


class VlaError(RuntimeError):
    def __init__(self, what: str, code: int):
        super().__init__(f"{what} failed with vla_status {code}")
        self.code = code


# name -> (restype, argtypes) for every symbol the two headers declare
SIGNATURES = {
    "vla_abi_version": (I32, []),
    "vla_backend_name": (ctypes.c_char_p, []),
    "vla_int8_available": (I32, []),
    "vla_act_load": (VP, [ctypes.c_char_p]),
    "vla_act_free": (None, [VP]),
    "vla_act_chunk": (I32, [VP]),
    "vla_act_action_dim": (I32, [VP]),
    "vla_act_state_dim": (I32, [VP]),
    "vla_act_n_cams": (I32, [VP]),
    "vla_act_img_h": (I32, [VP]),
    "vla_act_img_w": (I32, [VP]),
    "vla_act_predict": (I32, [VP, U8P, F32P, I32, F32P]),
    "vla_cuda_i8_ld": (I64, [I32]),
    "vla_cuda_device_status": (I32, []),
    "vla_cuda_quantize_act_i8": (I32, [VP, VP, VP, I32, I32, I64, VP]),
    "vla_cuda_quantize_span_i8": (I32, [VP, VP, I64, ctypes.c_float, VP]),
    "vla_cuda_pack_weights_i8": (I32, [VP, VP, VP, I32, I32, I64, VP]),
    "vla_cuda_dense_linear_i8_pre": (I32, [VP, VP, VP, VP, VP, VP, I32, I32, I32, I64, I64, VP]),
    "vla_cuda_dense_linear_i8": (I32, [VP, VP, VP, VP, VP, I32, I32, I32, I64, VP, VP, VP]),
    "vla_cuda_dense_linear_i8_noalloc": (I32, [VP, VP, VP, VP, VP, I32, I32, I32, I64, VP]),
    "vla_cuda_gemm_i8": (I32, [VP, I64, VP, I64, VP, I32, VP, I64, VP, VP, VP, I64, I32, I32, I32, I32, VP, I32,
                               I32, VP]),
    "vla_cuda_gemm_i8_rowq_supported": (I32, [I32, I32, I32]),
    "vla_cuda_gemm_i8_rowq": (I32, [VP, I64, VP, VP, I64, VP, VP, I64, VP, VP, I32, I32, I32, I32, VP, VP, VP]),
    "vla_cuda_gemm_i8_splitk": (I32, [VP, I64, VP, I64, VP, VP, I64, VP, VP, VP, I64, I32, I32, I32, I32, VP, I64, VP,
                                      I32, VP]),
    "vla_cuda_conv2d_i8": (I32, [VP, VP, I32, I32, I32, I32, VP, I64, VP, VP, I32, I32, I32, I32, F32, I32, VP, VP,
                                 VP, VP, VP]),
    "vla_cuda_layernorm": (I32, [VP, VP, VP, VP, I32, I32, F32, VP]),
    "vla_cuda_gqa_attention": (I32, [VP, VP, VP, VP, I32, I32, I32, I32, I32, F32, VP, VP]),
    "vla_cuda_gqa_attention_tc": (I32, [VP, VP, VP, VP, I32, I32, I32, I32, I32, F32, VP, VP]),
    "vla_cuda_maxpool2d_relu": (I32, [VP, VP, I32, I32, I32, I32, I32, I32, I32, VP]),
    "vla_cuda_rmsnorm": (I32, [VP, VP, VP, I32, I32, F32, VP]),
    "vla_cuda_rope_neox": (I32, [VP, VP, I32, I32, I32, F32, VP]),
    "vla_cuda_silu_gate": (I32, [VP, VP, VP, I64, VP]),
    "vla_cuda_silu": (I32, [VP, VP, I64, VP]),
    "vla_cuda_gelu_tanh": (I32, [VP, VP, I64, VP]),
    "vla_cuda_gelu_erf": (I32, [VP, VP, I64, VP]),
    "vla_cuda_relu": (I32, [VP, VP, I64, VP]),
    "vla_cuda_mish": (I32, [VP, VP, I64, VP]),
    "vla_cuda_groupnorm_scratch_bytes": (ctypes.c_uint64, [I32]),
    "vla_cuda_groupnorm": (I32, [VP, VP, VP, VP, I32, I32, I32, F32, I32, VP, VP]),
    "vla_cuda_spatial_softmax": (I32, [VP, VP, VP, I32, I32, VP]),
    "vla_cuda_im2col1d": (I32, [VP, VP, I32, I32, I32, I32, I32, I32, VP]),
    "vla_cuda_conv_transpose1d": (I32, [VP, VP, VP, VP, I32, I32, I32, I32, I32, I32, VP]),
    "vla_cuda_dense_linear_f32": (I32, [VP, VP, VP, VP, I32, I32, I32, VP]),
    "vla_tcpu_int8_gemm_available": (I32, []),
    "vla_tcpu_i8_kpad": (I32, [I32]),
    "vla_tcpu_packed_i8_words": (ctypes.c_uint64, [I32, I32]),
    "vla_tcpu_pack_weights_i8": (I32, [VP, VP, VP, I32, I32]),
    "vla_tcpu_i8_rowsums": (VP, [VP, I32, I32]),
    "vla_tcpu_quantize_span_i8": (I32, [VP, VP, ctypes.c_uint64, ctypes.c_float]),
    "vla_tcpu_dense_linear_i8_ref": (I32, [VP, VP, VP, VP, VP, VP, I32, I32, I32]),
    "vla_tcpu_quantize_act_i8": (I32, [VP, VP, VP, I32, I32]),
    "vla_tcpu_dense_linear_i8_pre": (I32, [VP, VP, VP, VP, VP, VP, I32, I32, I32]),
    "vla_tcpu_dense_linear_i8": (I32, [VP, VP, VP, VP, VP, I32, I32, I32, VP, VP]),
    "vla_diffusion_load": (VP, [ctypes.c_char_p]),
    "vla_diffusion_load_batch": (VP, [ctypes.c_char_p, I32]),
    "vla_diffusion_free": (None, [VP]),
    "vla_diffusion_chunk": (I32, [VP]),
    "vla_diffusion_horizon": (I32, [VP]),
    "vla_diffusion_action_dim": (I32, [VP]),
    "vla_diffusion_state_dim": (I32, [VP]),
    "vla_diffusion_n_cams": (I32, [VP]),
    "vla_diffusion_n_obs_steps": (I32, [VP]),
    "vla_diffusion_img_h": (I32, [VP]),
    "vla_diffusion_img_w": (I32, [VP]),
    "vla_diffusion_num_steps": (I32, [VP]),
    "vla_diffusion_is_ddim": (I32, [VP]),
    "vla_diffusion_predict": (I32, [VP, U8P, F32P, I32, F32P, F32P]),
    "vla_diffusion_predict_batch": (I32, [VP, I32, U8P, F32P, I32, F32P, F32P]),
    "vla_diffusion_device_buffers": (I32, [VP, VP, VP, VP, VP]),
    "vla_diffusion_enqueue": (I32, [VP, I32, VP, I32]),
    "vla_diffusion_kernels_per_step": (I32, [VP]),
    "vla_diffusion_int8_layers": (I32, [VP]),
    "vla_diffusion_global_cond": (I64, [VP, F32P, I64]),
    "vla_diffusion_debug_map": (I64, [VP, F32P, I64]),
    "vla_octo_load": (VP, [ctypes.c_char_p, ctypes.c_char_p]),
    "vla_octo_load_batch": (VP, [ctypes.c_char_p, ctypes.c_char_p, I32]),
    "vla_octo_free": (None, [VP]),
    "vla_octo_horizon": (I32, [VP]),
    "vla_octo_action_dim": (I32, [VP]),
    "vla_octo_max_window": (I32, [VP]),
    "vla_octo_num_steps": (I32, [VP]),
    "vla_octo_embed_dim": (I32, [VP]),
    "vla_octo_int8_layers": (I32, [VP]),
    "vla_octo_kernels_per_step": (I32, [VP]),
    "vla_octo_t5_runs": (I32, [VP]),
    "vla_octo_predict": (I32, [VP, U8P, U8P, I32, U8P, ctypes.c_char_p, ctypes.c_uint64, I32, F32P]),
    "vla_octo_predict_ex": (I32, [VP, U8P, U8P, I32, U8P, ctypes.c_char_p, F32P, F32P, ctypes.c_uint64, I32, F32P]),
    "vla_octo_predict_batch": (I32, [VP, I32, U8P, U8P, I32, U8P, ctypes.POINTER(ctypes.c_char_p), F32P, F32P,
                                     ctypes.POINTER(ctypes.c_uint64), I32, F32P]),
    "vla_octo_readout": (I64, [VP, F32P, I64]),
    "vla_t5_tokenize": (I32, [ctypes.c_char_p, ctypes.c_char_p, I32, ctypes.POINTER(ctypes.c_int32)]),
    "vla_smolvla_load": (VP, [ctypes.c_char_p, ctypes.c_char_p]),
    "vla_smolvla_load_batch": (VP, [ctypes.c_char_p, ctypes.c_char_p, I32]),
    "vla_smolvla_free": (None, [VP]),
    "vla_smolvla_chunk": (I32, [VP]),
    "vla_smolvla_action_dim": (I32, [VP]),
    "vla_smolvla_state_dim": (I32, [VP]),
    "vla_smolvla_n_views": (I32, [VP]),
    "vla_smolvla_img_size": (I32, [VP]),
    "vla_smolvla_tok_maxlen": (I32, [VP]),
    "vla_smolvla_int8_layers": (I32, [VP]),
    "vla_smolvla_kernels_per_step": (I32, [VP]),
    "vla_smolvla_tokenize": (I32, [VP, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]),
    "vla_smolvla_predict": (I32, [VP, U8P, I32, I32, I32, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), I32, F32P, F32P, ctypes.c_uint64, F32P]),
    "vla_smolvla_predict_rtc": (I32, [VP, U8P, I32, I32, I32, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), I32, F32P, F32P, ctypes.c_uint64, F32P,
                                      F32P, I32, F32P, ctypes.c_float]),
    "vla_smolvla_predict_batch": (I32, [VP, I32, U8P, I32, I32, I32, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32), I32, F32P, F32P,
                                        ctypes.POINTER(ctypes.c_uint64), F32P, F32P, I32, F32P, ctypes.c_float]),
    "vla_bpe_tokenize": (I32, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), I32]),
    "vla_octo_device_buffers": (I32, [VP, VP, VP, VP, VP, VP, VP]),
    "vla_octo_set_instruction": (I32, [VP, I32, ctypes.c_char_p]),
    "vla_octo_enqueue": (I32, [VP, I32, I32, I32, VP, I32]),
    "vla_act_device_buffers": (I32, [VP, VP, VP, VP]),
    "vla_act_enqueue": (I32, [VP, VP, I32]),
    "vla_act_kernels_per_step": (I32, [VP]),
    "vla_act_int8_layers": (I32, [VP]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library (built on first use if only the sources are present)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            from . import build as _build
            _build.build()
        l = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(code: int, what: str) -> None:
    if code != VLA_OK:
        raise VlaError(what, code)


class ActPolicy:
    """ctypes binding of the ACT C ABI, shaped like the reference's ActEngine.

    frames [n_cams, img_h, img_w, 3] uint8 + state [state_dim] (raw robot units)
    -> actions [chunk, action_dim] float32 (robot units unless unnormalize=False).
    """

    def __init__(self, model_dir: str):
        self.lib = lib()
        self.h = self.lib.vla_act_load(model_dir.encode())
        if not self.h:
            raise RuntimeError(f"vla_act_load failed for {model_dir}")
        for name in ("chunk", "action_dim", "state_dim", "n_cams", "img_h", "img_w"):
            setattr(self, name, int(getattr(self.lib, f"vla_act_{name}")(self.h)))

    def predict(self, frames: np.ndarray, state: np.ndarray, unnormalize: bool = True) -> np.ndarray:
        frames = np.ascontiguousarray(frames, np.uint8)
        if frames.shape != (self.n_cams, self.img_h, self.img_w, 3):
            raise ValueError(f"frames {frames.shape} != {(self.n_cams, self.img_h, self.img_w, 3)}")
        state = np.ascontiguousarray(np.asarray(state, np.float32).reshape(-1))
        if state.size != self.state_dim:
            raise ValueError(f"state has {state.size} values, the checkpoint wants {self.state_dim}")
        out = np.empty((self.chunk, self.action_dim), np.float32)
        rc = self.lib.vla_act_predict(self.h, frames.ctypes.data_as(U8P), state.ctypes.data_as(F32P),
                                      1 if unnormalize else 0, out.ctypes.data_as(F32P))
        check(rc, "vla_act_predict")
        return out

    def device_buffers(self):
        img, st, act = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        check(self.lib.vla_act_device_buffers(self.h, ctypes.byref(img), ctypes.byref(st), ctypes.byref(act)),
              "vla_act_device_buffers")
        return img.value, st.value, act.value

    def enqueue(self, stream_handle: int, unnormalize: bool = True) -> None:
        check(self.lib.vla_act_enqueue(self.h, ctypes.c_void_p(stream_handle), 1 if unnormalize else 0),
              "vla_act_enqueue")

    @property
    def kernels_per_step(self) -> int:
        return int(self.lib.vla_act_kernels_per_step(self.h))

    @property
    def int8_layers(self) -> int:
        return int(self.lib.vla_act_int8_layers(self.h))

    def close(self) -> None:
        if self.h:
            self.lib.vla_act_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def t5_tokenize(vocab_text: str, text: str, max_len: int = 16) -> np.ndarray:
    """Token ids of `text` under a T5 vocab.txt (the tokenizer Octo's handles
    use; host code, no GPU needed)."""
    ids = np.zeros(max_len, np.int32)
    rc = lib().vla_t5_tokenize(vocab_text.encode(), text.encode(), int(max_len),
                               ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)))
    check(rc, "vla_t5_tokenize")
    return ids


def bpe_tokenize(vocab_text: str, merges_text: str, text: str) -> np.ndarray:
    """Token ids of `text` under a byte-level BPE vocab.txt / merges.txt (the
    tokenizer SmolVLA's handles use; host code, no GPU needed)."""
    i32p = ctypes.POINTER(ctypes.c_int32)
    n = lib().vla_bpe_tokenize(vocab_text.encode(), merges_text.encode(), text.encode(), None, 0)
    check(min(int(n), 0), "vla_bpe_tokenize")
    ids = np.zeros(max(int(n), 1), np.int32)
    lib().vla_bpe_tokenize(vocab_text.encode(), merges_text.encode(), text.encode(), ids.ctypes.data_as(i32p),
                           ids.size)
    return ids[:int(n)]


class SmolvlaPolicy:
    """ctypes binding of the SmolVLA C ABI (include/vla_simd.h, the reference's
    vla_smolvla_* at src/models/smolvla/smolvla_capi.cpp:66-180).

    frames [n_views, h, w, 3] uint8 at the camera's resolution, an instruction
    string (tokenized by the handle), raw state [state_dim], and noise [chunk,
    32] or a seed -> actions [chunk, action_dim]; optional real-time-chunking
    guidance (prev [n_prev, action_dim], weights [chunk], max_guidance). With
    max_batch > 1, predict_batch takes the arrays with a leading batch axis.
    """

    def __init__(self, model_dir: str, tok_dir: str | None = None, max_batch: int = 1):
        self.lib = lib()
        tok_dir = tok_dir or os.path.join(model_dir, "tok")
        self.h = (self.lib.vla_smolvla_load(model_dir.encode(), tok_dir.encode()) if max_batch == 1
                  else self.lib.vla_smolvla_load_batch(model_dir.encode(), tok_dir.encode(), int(max_batch)))
        if not self.h:
            raise RuntimeError(f"vla_smolvla_load failed for {model_dir}")
        self.max_batch = int(max_batch)
        for name in ("chunk", "action_dim", "state_dim", "n_views", "img_size", "tok_maxlen"):
            setattr(self, name, int(getattr(self.lib, f"vla_smolvla_{name}")(self.h)))

    def tokenize(self, text: str):
        i32p = ctypes.POINTER(ctypes.c_int32)
        ids = np.zeros(self.tok_maxlen, np.int32)
        mask = np.zeros(self.tok_maxlen, np.int32)
        n = self.lib.vla_smolvla_tokenize(self.h, text.encode(), ids.ctypes.data_as(i32p), mask.ctypes.data_as(i32p))
        check(min(int(n), 0), "vla_smolvla_tokenize")
        return ids, mask

    def predict(self, frames, instruction: str, state, noise=None, seed: int = 0, prev=None, weights=None,
                max_guidance: float = 0.0) -> np.ndarray:
        return self.predict_batch(np.asarray(frames)[None], [instruction], np.asarray(state)[None],
                                  None if noise is None else np.asarray(noise)[None], [seed],
                                  None if prev is None else np.asarray(prev)[None],
                                  None if weights is None else np.asarray(weights)[None], max_guidance)[0]

    def predict_batch(self, frames, instructions, state, noise=None, seeds=None, prev=None, weights=None,
                      max_guidance: float = 0.0) -> np.ndarray:
        i32p = ctypes.POINTER(ctypes.c_int32)
        frames = np.ascontiguousarray(frames, np.uint8)
        b = frames.shape[0]
        if frames.ndim != 5 or frames.shape[1] != self.n_views or frames.shape[4] != 3:
            raise ValueError(f"frames {frames.shape}")
        toks = [self.tokenize(t) for t in instructions]
        ids = np.ascontiguousarray(np.stack([t[0] for t in toks]))
        mask = np.ascontiguousarray(np.stack([t[1] for t in toks]))
        state = np.ascontiguousarray(state, np.float32).reshape(b, self.state_dim)
        nz = None if noise is None else np.ascontiguousarray(noise, np.float32)
        sd = (ctypes.c_uint64 * b)(*[int(v) for v in (seeds if seeds is not None else range(b))])
        pv = None if prev is None else np.ascontiguousarray(prev, np.float32)
        wt = None if weights is None else np.ascontiguousarray(weights, np.float32)
        n_prev = 0 if pv is None else pv.shape[1]
        out = np.empty((b, self.chunk, self.action_dim), np.float32)
        p = lambda a, t: None if a is None else a.ctypes.data_as(t)
        rc = self.lib.vla_smolvla_predict_batch(self.h, b, frames.ctypes.data_as(U8P), self.n_views, frames.shape[2],
                                                frames.shape[3], ids.ctypes.data_as(i32p), mask.ctypes.data_as(i32p),
                                                self.tok_maxlen, state.ctypes.data_as(F32P), p(nz, F32P), sd,
                                                out.ctypes.data_as(F32P), p(pv, F32P), n_prev, p(wt, F32P),
                                                float(max_guidance))
        check(rc, "vla_smolvla_predict_batch")
        return out

    @property
    def kernels_per_step(self) -> int:
        return int(self.lib.vla_smolvla_kernels_per_step(self.h))

    @property
    def int8_layers(self) -> int:
        return int(self.lib.vla_smolvla_int8_layers(self.h))

    def close(self) -> None:
        if self.h:
            self.lib.vla_smolvla_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OctoPolicy:
    """ctypes binding of the Octo C ABI (include/vla_simd.h, the reference's
    vla_octo_* at src/models/octo/octo_capi.cpp:19-58).

    primary [wnd, 256, 256, 3] and wrist [wnd, 128, 128, 3] (or None) uint8,
    timestep_mask [wnd], an instruction string, and either noise [horizon *
    action_dim] with z [steps, horizon * action_dim] or a seed -> actions
    [horizon, action_dim]. With max_batch > 1, predict_batch takes the arrays
    with a leading batch axis and a list of instructions.
    """

    def __init__(self, model_dir: str, tok_dir: str | None = None, max_batch: int = 1):
        self.lib = lib()
        tok_dir = tok_dir or os.path.join(model_dir, "tok")
        self.h = (self.lib.vla_octo_load(model_dir.encode(), tok_dir.encode()) if max_batch == 1
                  else self.lib.vla_octo_load_batch(model_dir.encode(), tok_dir.encode(), int(max_batch)))
        if not self.h:
            raise RuntimeError(f"vla_octo_load failed for {model_dir}")
        self.max_batch = int(max_batch)
        for name in ("horizon", "action_dim", "max_window", "num_steps", "embed_dim"):
            setattr(self, name, int(getattr(self.lib, f"vla_octo_{name}")(self.h)))
        self.flat = self.horizon * self.action_dim

    def _arrays(self, primary, wrist, tmask, noise, z, lead):
        primary = np.ascontiguousarray(primary, np.uint8)
        if primary.ndim != len(lead) + 4 or primary.shape[len(lead) + 1:] != (256, 256, 3):
            raise ValueError(f"primary {primary.shape}")
        wnd = primary.shape[len(lead)]
        if wrist is not None:
            wrist = np.ascontiguousarray(wrist, np.uint8)
            if wrist.shape != lead + (wnd, 128, 128, 3):
                raise ValueError(f"wrist {wrist.shape}")
        tmask = np.ascontiguousarray(tmask, np.uint8)
        if tmask.shape != lead + (wnd,):
            raise ValueError(f"timestep mask {tmask.shape}")
        if (noise is None) != (z is None):
            raise ValueError("noise and z go together")
        n = int(np.prod(lead, dtype=np.int64)) if lead else 1
        if noise is not None:
            noise = np.ascontiguousarray(noise, np.float32)
            z = np.ascontiguousarray(z, np.float32)
            if noise.size != n * self.flat or z.size != n * self.num_steps * self.flat:
                raise ValueError("noise / z size")
        return primary, wrist, tmask, noise, z, wnd

    @staticmethod
    def _p(a, t):
        return None if a is None else a.ctypes.data_as(t)

    def predict(self, primary, wrist, tmask, instruction: str, noise=None, z=None, seed: int = 0,
                unnormalize: bool = True) -> np.ndarray:
        primary, wrist, tmask, noise, z, wnd = self._arrays(primary, wrist, tmask, noise, z, ())
        out = np.empty((self.horizon, self.action_dim), np.float32)
        rc = self.lib.vla_octo_predict_ex(self.h, self._p(primary, U8P), self._p(wrist, U8P), wnd,
                                          self._p(tmask, U8P), instruction.encode(), self._p(noise, F32P),
                                          self._p(z, F32P), int(seed), 1 if unnormalize else 0,
                                          out.ctypes.data_as(F32P))
        check(rc, "vla_octo_predict_ex")
        return out

    def predict_batch(self, primary, wrist, tmask, instructions, noise=None, z=None, seeds=None,
                      unnormalize: bool = True) -> np.ndarray:
        b = int(np.asarray(primary).shape[0])
        primary, wrist, tmask, noise, z, wnd = self._arrays(primary, wrist, tmask, noise, z, (b,))
        if len(instructions) != b:
            raise ValueError("one instruction per query")
        ins = (ctypes.c_char_p * b)(*[s.encode() for s in instructions])
        sd = None
        if noise is None:
            sd = (ctypes.c_uint64 * b)(*[int(v) for v in (seeds if seeds is not None else range(b))])
        out = np.empty((b, self.horizon, self.action_dim), np.float32)
        rc = self.lib.vla_octo_predict_batch(self.h, b, self._p(primary, U8P), self._p(wrist, U8P), wnd,
                                             self._p(tmask, U8P), ins, self._p(noise, F32P), self._p(z, F32P), sd,
                                             1 if unnormalize else 0, out.ctypes.data_as(F32P))
        check(rc, "vla_octo_predict_batch")
        return out

    def readout(self) -> np.ndarray:
        """The last query batch's readout embeddings [batch, embed_dim] (a parity tap)."""
        out = np.empty(self.max_batch * self.embed_dim, np.float32)
        n = int(self.lib.vla_octo_readout(self.h, out.ctypes.data_as(F32P), out.size))
        if n < 0:
            raise RuntimeError("vla_octo_readout failed")
        return out[:n].reshape(-1, self.embed_dim).copy()

    def device_buffers(self):
        ptrs = [ctypes.c_void_p() for _ in range(6)]
        check(self.lib.vla_octo_device_buffers(self.h, *[ctypes.byref(p) for p in ptrs]), "vla_octo_device_buffers")
        return tuple(p.value for p in ptrs)

    def set_instruction(self, b: int, instruction: str) -> None:
        check(self.lib.vla_octo_set_instruction(self.h, int(b), instruction.encode()), "vla_octo_set_instruction")

    def enqueue(self, batch: int, wnd: int, wrist: bool, stream_handle: int, unnormalize: bool = True) -> None:
        check(self.lib.vla_octo_enqueue(self.h, int(batch), int(wnd), 1 if wrist else 0,
                                        ctypes.c_void_p(stream_handle), 1 if unnormalize else 0), "vla_octo_enqueue")

    @property
    def kernels_per_step(self) -> int:
        return int(self.lib.vla_octo_kernels_per_step(self.h))

    @property
    def int8_layers(self) -> int:
        return int(self.lib.vla_octo_int8_layers(self.h))

    @property
    def t5_runs(self) -> int:
        return int(self.lib.vla_octo_t5_runs(self.h))

    def close(self) -> None:
        if self.h:
            self.lib.vla_octo_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DiffusionPolicy:
    """ctypes binding of the Diffusion Policy C ABI (include/vla_simd.h, the
    reference's vla_diffusion_* at src/models/diffusion/diffusion_capi.cpp:23-72).

    frames [n_obs_steps * n_cams, img_h, img_w, 3] uint8 (oldest step first,
    cameras inside a step), state [n_obs_steps, state_dim], noise
    [1 + num_steps, horizon, action_dim] (None: start from zeros) ->
    actions [chunk, action_dim]. With max_batch > 1, predict_batch takes the
    same arrays with a leading batch axis.
    """

    def __init__(self, model_dir: str, max_batch: int = 1):
        self.lib = lib()
        self.h = (self.lib.vla_diffusion_load(model_dir.encode()) if max_batch == 1
                  else self.lib.vla_diffusion_load_batch(model_dir.encode(), int(max_batch)))
        if not self.h:
            raise RuntimeError(f"vla_diffusion_load failed for {model_dir}")
        self.max_batch = int(max_batch)
        for name in ("chunk", "horizon", "action_dim", "state_dim", "n_cams", "n_obs_steps", "img_h", "img_w",
                     "num_steps", "is_ddim"):
            setattr(self, name, int(getattr(self.lib, f"vla_diffusion_{name}")(self.h)))

    def _args(self, frames, state, noise, lead):
        frames = np.ascontiguousarray(frames, np.uint8)
        want = lead + (self.n_obs_steps * self.n_cams, self.img_h, self.img_w, 3)
        if frames.shape != want:
            raise ValueError(f"frames {frames.shape} != {want}")
        state = np.ascontiguousarray(np.asarray(state, np.float32))
        if state.size != int(np.prod(lead, dtype=np.int64)) * self.n_obs_steps * self.state_dim:
            raise ValueError(f"state has {state.size} values")
        nz = None
        if noise is not None:
            nz = np.ascontiguousarray(np.asarray(noise, np.float32))
            if nz.size != int(np.prod(lead, dtype=np.int64)) * (1 + self.num_steps) * self.horizon * self.action_dim:
                raise ValueError(f"noise has {nz.size} values")
        return frames, state, nz

    def predict(self, frames, state, noise=None, unnormalize: bool = True) -> np.ndarray:
        frames, state, nz = self._args(frames, state, noise, ())
        out = np.empty((self.chunk, self.action_dim), np.float32)
        rc = self.lib.vla_diffusion_predict(self.h, frames.ctypes.data_as(U8P), state.ctypes.data_as(F32P),
                                            1 if unnormalize else 0, out.ctypes.data_as(F32P),
                                            None if nz is None else nz.ctypes.data_as(F32P))
        check(rc, "vla_diffusion_predict")
        return out

    def predict_batch(self, frames, state, noise=None, unnormalize: bool = True) -> np.ndarray:
        b = int(np.asarray(frames).shape[0])
        frames, state, nz = self._args(frames, state, noise, (b,))
        out = np.empty((b, self.chunk, self.action_dim), np.float32)
        rc = self.lib.vla_diffusion_predict_batch(self.h, b, frames.ctypes.data_as(U8P), state.ctypes.data_as(F32P),
                                                  1 if unnormalize else 0, out.ctypes.data_as(F32P),
                                                  None if nz is None else nz.ctypes.data_as(F32P))
        check(rc, "vla_diffusion_predict_batch")
        return out

    def device_buffers(self):
        fr, st, nz, act = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
        check(self.lib.vla_diffusion_device_buffers(self.h, ctypes.byref(fr), ctypes.byref(st), ctypes.byref(nz),
                                                    ctypes.byref(act)), "vla_diffusion_device_buffers")
        return fr.value, st.value, nz.value, act.value

    def enqueue(self, batch: int, stream_handle: int, unnormalize: bool = True) -> None:
        check(self.lib.vla_diffusion_enqueue(self.h, int(batch), ctypes.c_void_p(stream_handle),
                                             1 if unnormalize else 0), "vla_diffusion_enqueue")

    def global_cond(self) -> np.ndarray:
        """The last query batch's global conditioning vectors (a parity tap)."""
        out = np.empty(self.max_batch * 4096 * 16, np.float32)
        n = int(self.lib.vla_diffusion_global_cond(self.h, out.ctypes.data_as(F32P), out.size))
        if n < 0:
            raise RuntimeError("vla_diffusion_global_cond failed")
        return out[:n].copy()

    def debug_map(self, cap: int = 1 << 24) -> np.ndarray:
        """The first encoder's map after the ResNet stage VLA_DP_DEBUG_STAGE names (a parity tap)."""
        out = np.empty(cap, np.float32)
        n = int(self.lib.vla_diffusion_debug_map(self.h, out.ctypes.data_as(F32P), out.size))
        if n < 0:
            raise RuntimeError("vla_diffusion_debug_map failed")
        return out[:n].copy()

    @property
    def kernels_per_step(self) -> int:
        return int(self.lib.vla_diffusion_kernels_per_step(self.h))

    @property
    def int8_layers(self) -> int:
        return int(self.lib.vla_diffusion_int8_layers(self.h))

    def close(self) -> None:
        if self.h:
            self.lib.vla_diffusion_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
