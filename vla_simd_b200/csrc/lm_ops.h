// Host-side interface of the lm / conv ops of the other policy families (lm_ops.cu).
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

namespace vsb {

enum : int { kActRelu = 0, kActSiluGate = 1, kActSilu = 2, kActGeluTanh = 3, kActGeluErf = 4, kActMish = 5 };

// RMSNorm; with q, also the per-row int8 copy of out (q [seq][ldq], zero past
// hidden) and its scales, as quantize_rows would make them.
cudaError_t rmsnorm(const float* x, const float* w, float* out, int seq, int hidden, float eps, cudaStream_t st,
                    int8_t* q = nullptr, long long ldq = 0, float* qscale = nullptr);
cudaError_t rope_neox(float* x, const int* pos, int seq, int n_heads, int head_dim, float base, cudaStream_t st);
// out = act(x) (u: silu_gate's second operand); out may alias x
cudaError_t activation(int kind, float* out, const float* x, const float* u, long long n, cudaStream_t st);
size_t groupnorm_scratch_bytes(int C);
cudaError_t groupnorm(const float* x, const float* scale, const float* bias, float* out, int n_pixels, int C,
                      int groups, float eps, bool fuse_relu, void* scratch, cudaStream_t st);
cudaError_t spatial_softmax(const float* x, const float* grid, float* out, int n_pixels, int C, cudaStream_t st);
cudaError_t im2col1d(const float* x, float* col, int T, int Cin, int k, int stride, int pad, int Tout,
                     cudaStream_t st);
cudaError_t conv_transpose1d(const float* x, const float* W, const float* bias, float* out, int T, int Cin, int Cout,
                             int k, int stride, int pad, cudaStream_t st);

}  // namespace vsb
