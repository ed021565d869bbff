// TEST INFRASTRUCTURE ONLY: a TCPU_HAL_CUDA backend translation unit for the
// reference. It defines every function of the reference's int8 op API
// (vla.simd src/ops/quant_ops.h:40-92) on top of libvla_simd_b200.so's
// host-pointer C ABI (vla_tcpu_*, include/vla_simd_cuda.h), and oracle/Makefile
// links it with the reference's own unmodified sources - all of them except
// the two files that define these functions for the CPU
// (src/hal/common/gemm_i8.cpp, src/hal/avx2/gemm_i8.cpp) - into
// oracle/_ref/libvla_ref_cuda.so. So the reference's nn::Linear
// (src/nn/linear.cpp:66-134), its int8 convolutions (src/hal/common/conv.cpp:444-526,
// which quantize through quantize_span_i8) and its whole ACT / Diffusion Policy
// / Octo / SmolVLA models run their int8 layers on the B200 with no change to
// their code; the tests compare them with the CPU build (oracle/_ref/libvla_ref.so).
//
// The reference's ops return void and assert their preconditions
// (src/hal/common/gemm_i8.cpp:61, src/hal/avx2/gemm_i8.cpp:127); here a call the
// library refuses ends the process with the status, which is the same contract.
#include "ops/quant_ops.h"

#include "../include/vla_simd_cuda.h"

#include <cstdio>
#include <cstdlib>

namespace {

void must(int32_t status, const char* what) {
    if (status == VLA_OK) return;
    std::fprintf(stderr, "TCPU_HAL_CUDA backend: %s failed with status %d\n", what, status);
    std::abort();
}

}  // namespace

namespace tcpu {

bool int8_gemm_available() { return vla_tcpu_int8_gemm_available() != 0; }

int i8_kpad(int K) { return vla_tcpu_i8_kpad(K); }

size_t packed_i8_words(int N, int K) { return static_cast<size_t>(vla_tcpu_packed_i8_words(N, K)); }

void pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int N, int K) {
    must(vla_tcpu_pack_weights_i8(W, Wq, wscale, N, K), "pack_weights_i8");
}

const int32_t* i8_rowsums(const int8_t* Wq, int N, int K) { return vla_tcpu_i8_rowsums(Wq, N, K); }

void dense_linear_i8(float* out, const float* x, const int8_t* Wq, const float* wscale, const float* bias, int seq,
                     int N, int K, int8_t* xq_scratch, float* ascale_scratch) {
    must(vla_tcpu_dense_linear_i8(out, x, Wq, wscale, bias, seq, N, K, xq_scratch, ascale_scratch),
         "dense_linear_i8");
}

void quantize_act_i8(const float* x, int8_t* xq, float* ascale, int seq, int K) {
    must(vla_tcpu_quantize_act_i8(x, xq, ascale, seq, K), "quantize_act_i8");
}

void quantize_span_i8(const float* x, int8_t* q, size_t n, float inv) {
    must(vla_tcpu_quantize_span_i8(x, q, n, inv), "quantize_span_i8");
}

void dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq, const float* wscale,
                         const float* bias, int seq, int N, int K) {
    must(vla_tcpu_dense_linear_i8_pre(out, xq, ascale, Wq, wscale, bias, seq, N, K), "dense_linear_i8_pre");
}

void dense_linear_i8_ref(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq, const float* wscale,
                         const float* bias, int seq, int N, int K) {
    must(vla_tcpu_dense_linear_i8_ref(out, xq, ascale, Wq, wscale, bias, seq, N, K), "dense_linear_i8_ref");
}

}  // namespace tcpu

extern "C" int ref_backend_is_cuda(void) { return 1; }
