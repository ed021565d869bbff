// Host-side interface of the quantization kernels (quant.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vsb {

// Most frames one im2col / space-to-depth launch quantizes (per-frame scales
// are staged in shared memory).
constexpr int kMaxConvFrames = 256;

// Per-row symmetric int8 quantization of x [M][ldx] (K valid columns), optional
// fp32 addend added first. q [M][ldq] is zero past K. Optional second output
// q2/scale2 quantizes x itself (without the addend) in the same pass.
cudaError_t quantize_rows(const float* x, long long ldx, const float* addend, long long ld_add, int M, int K,
                          int8_t* q, long long ldq, float* scale, int8_t* q2, long long ldq2, float* scale2,
                          cudaStream_t st);

// int8 im2col of F NHWC frames with the per-frame per-tensor scale derived from
// amax_bits[f] (float bits) and clip; col [F*Ho*Wo][ldc], rscale [F*Ho*Wo].
cudaError_t im2col_i8(const float* x, int F, int H, int W, int C, int k, int stride, int pad, int Ho, int Wo,
                      long long ldc, const unsigned int* amax_bits, float clip, int8_t* col, float* rscale,
                      cudaStream_t st);

// Per-frame int8 quantization of F frames of per_frame floats with the scale
// im2col_i8 uses (from amax_bits[f] and clip): q has x's layout, fscale [F].
// The input of the implicit-GEMM convolution.
cudaError_t quantize_frames_i8(const float* x, int F, long long per_frame, const unsigned int* amax_bits, float clip,
                               int8_t* q, float* fscale, cudaStream_t st);

// Stride-2 convolution over C <= 4 channels with a k <= 8 filter as a
// stride-1 conv of kt = ceil(k/2) rows and 1 column over 64 channels
// (space to depth): s2d_quantize_i8 writes the int8 input
// q [F][Ho + kt - 1][Wo][64] and fscale [F] (scale as im2col_i8), and
// s2d_repack_weights_host re-indexes packed weights Wq [N][ldw] (K order
// ky, kx, c) into [N][64 * kt] (zero for the taps the conv does not have).
bool s2d_conv_supported(int C, int k, int stride);
cudaError_t s2d_quantize_i8(const float* x, int F, int H, int W, int C, int k, int pad, int Ho, int Wo,
                            const unsigned int* amax_bits, float clip, int8_t* q, float* fscale, cudaStream_t st);
void s2d_repack_weights_host(const int8_t* Wq, int N, int k, int C, long long ldw, int8_t* out);

// atomicMax of |x| (float bits) per slot of per_slot consecutive elements.
cudaError_t absmax_slots(const float* x, long long n, long long per_slot, unsigned int* amax_bits,
                         cudaStream_t st);

// Reference CPU panel layout [N/16][Kp/4][16][4] -> device rows [N][ldw].
cudaError_t unpack_panels_i8(const int8_t* panels, int N, int K, int8_t* rows, long long ldw, cudaStream_t st);
// q[i] = rne(clamp(x[i] * inv, +-127)) over n elements (tcpu::quantize_span_i8).
cudaError_t quantize_span_i8(const float* x, int8_t* q, long long n, float inv, cudaStream_t st);
// The inverse: device rows [N][ldw] -> panels [N/16][Kp/4][16][4] + int32 row
// sums [N] right after them (the reference's pack_weights_i8 output layout).
cudaError_t pack_panels_i8(const int8_t* rows, long long ldw, int N, int K, int8_t* panels, cudaStream_t st);

}  // namespace vsb
