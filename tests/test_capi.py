"""The C-ABI library without a GPU: it loads, exports every entry point the
headers in include/ declare, and rejects bad arguments before touching a device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        names |= set(re.findall(r"VLA_API[^;(]*?\b(vla_\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol():
    import vla_simd_b200
    lib = vla_simd_b200.lib()
    declared = _declared()
    assert len(declared) >= 30
    missing = [n for n in sorted(declared) if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding table covers them all
    assert declared == set(vla_simd_b200.SIGNATURES)


def test_abi_identity():
    import vla_simd_b200
    lib = vla_simd_b200.lib()
    assert lib.vla_abi_version() == 1          # the reference server requires 1
    assert lib.vla_backend_name() == b"cuda-sm100a"
    assert lib.vla_tcpu_i8_kpad(147) == 148 and lib.vla_tcpu_i8_kpad(512) == 512
    assert lib.vla_cuda_i8_ld(147) == 160 and lib.vla_cuda_i8_ld(3200) == 3200
    assert lib.vla_tcpu_packed_i8_words(16, 3) == (16 * 4 + 16 * 4) // 4


def test_argument_checks_need_no_device():
    import vla_simd_b200 as v
    lib = v.lib()
    # NULL handles
    assert lib.vla_act_chunk(None) == 0
    assert lib.vla_act_predict(None, None, None, 1, None) == v.VLA_ERR_ARG
    # shapes rejected before any launch
    assert lib.vla_cuda_gemm_i8(None, 16, None, 16, None, 1, None, 16, None, None, None, 0, 1, 16, 16, 0, None, 1, 0,
                                None) == v.VLA_ERR_ARG
    fake = ctypes.c_void_p(16)
    # K beyond the int32 headroom bound of nn::Linear::init_int8
    bigk = 2**31 // (255 * 127) + 1
    assert lib.vla_cuda_gemm_i8(fake, 16, fake, bigk + 16, fake, 1, fake, bigk + 16, fake, None, None, 0, 1, 16, bigk,
                                0, None, 1, 0, None) == v.VLA_ERR_ARG
    # ldx < K
    assert lib.vla_cuda_gemm_i8(fake, 16, fake, 8, fake, 1, fake, 16, fake, None, None, 0, 1, 16, 16, 0, None, 1, 0,
                                None) == v.VLA_ERR_ARG
    # unknown epilogue bit
    assert lib.vla_cuda_gemm_i8(fake, 16, fake, 16, fake, 1, fake, 16, fake, None, None, 0, 1, 16, 16, 64, None, 1, 0,
                                None) == v.VLA_ERR_ARG
    assert lib.vla_cuda_gqa_attention(fake, fake, fake, fake, 4, 4, 3, 2, 64, 1.0, None, None) == v.VLA_ERR_ARG
    assert lib.vla_cuda_gqa_attention(fake, fake, fake, fake, 4, 4, 2, 2, 32, 1.0, None, None) == v.VLA_ERR_ARG
    assert lib.vla_cuda_layernorm(fake, fake, fake, None, 1, 4096, 1e-5, None) == v.VLA_ERR_ARG
    assert lib.vla_tcpu_pack_weights_i8(fake, fake, fake, 15, 4) == v.VLA_ERR_ARG


def test_load_failures_return_null(tmp_path):
    import vla_simd_b200
    lib = vla_simd_b200.lib()
    assert not lib.vla_act_load(None)
    assert not lib.vla_act_load(str(tmp_path / "missing").encode())
