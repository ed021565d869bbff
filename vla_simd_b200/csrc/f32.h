// Host-side interface of the fp32 layer path (f32.cu).
#pragma once
#include <cuda_runtime.h>

namespace vsb {

// out [M][ldo] = A [M][lda] * W[N][ldw]^T + bias, epilogue modes as gemm_i8.h.
cudaError_t gemm_f32(const float* A, long long lda, const float* W, long long ldw, const float* bias, float* out,
                     long long ldo, const float* res, long long ldr, int M, int N, int K, int mode,
                     unsigned int* amax, int amax_rows, cudaStream_t st);

// fp32 im2col of F NHWC frames: col [F*Ho*Wo][k*k*C].
cudaError_t im2col_f32(const float* x, int F, int H, int W, int C, int k, int stride, int pad, int Ho, int Wo,
                       float* col, cudaStream_t st);

}  // namespace vsb
