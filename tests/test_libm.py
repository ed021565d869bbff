"""The host C library's float expf / log1pf / expm1f / tanhf, restated in
vla_simd_b200/csrc/libm_f32.h for the kernels, against the host library itself
on every one of the 2^32 float bit patterns (the restatement compiled as host C
with -ffp-contract=off into the oracle library), plus the reference's scalar
Mish tail v * tanhf(log1pf(expf(v))) (src/hal/common/eltwise.cpp:244-248)
composed from them. A NaN matches any NaN."""
import ctypes
from concurrent.futures import ThreadPoolExecutor

import pytest

FUNCS = {"expf": 0, "log1pf": 1, "expm1f": 2, "tanhf": 3, "mish": 4}


@pytest.fixture(scope="module")
def lib():
    from oracle import oracle
    oracle.restated()   # builds the oracle library if needed
    l = ctypes.CDLL(oracle.RESTATED_SO)
    l.or_libm_mismatches.restype = ctypes.c_uint64
    l.or_libm_mismatches.argtypes = [ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint32)]
    return l


@pytest.mark.parametrize("name", list(FUNCS))
def test_restated_libm_equals_host_on_all_inputs(lib, name):
    def run(chunk):
        first = ctypes.c_uint32(0)
        bad = lib.or_libm_mismatches(FUNCS[name], chunk << 27, 1 << 27, ctypes.byref(first))
        return bad, first.value
    with ThreadPoolExecutor(8) as ex:
        res = list(ex.map(run, range(32)))
    bad = [(n, hex(f)) for n, f in res if n]
    assert not bad, f"{name}: {sum(n for n, _ in bad)} mismatches, first at {bad[0][1]}"
