// fp32 path for layers a model leaves out of W8A8 (an ACT_INT8 bit cleared):
// im2col in fp32 and a shared-memory-tiled CUDA-core GEMM with the same
// epilogue options as the int8 kernel (bias, ReLU, residual add, residual add +
// ReLU, absmax tap). Summation order differs from the CPU's packed kernels, so
// these layers match the reference to fp32 rounding, not bit for bit.
#include "sm100.cuh"
#include "launch.cuh"
#include "f32.h"
#include "gemm_i8.h"

namespace vsb {

constexpr int kFT = 64;   // output tile
constexpr int kFK = 16;   // k step

__global__ void __launch_bounds__(256)
gemm_f32_kernel(const float* __restrict__ A, long long lda, const float* __restrict__ W, long long ldw,
                const float* __restrict__ bias, float* __restrict__ out, long long ldo,
                const float* __restrict__ res, long long ldr, int M, int N, int K, int mode,
                unsigned int* __restrict__ amax, int amax_rows) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    __shared__ float sA[kFK][kFT + 4];
    __shared__ float sW[kFK][kFT + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * kFT, n0 = blockIdx.x * kFT;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kFK) {
        for (int i = threadIdx.x; i < kFT * kFK; i += 256) {
            const int r = i / kFK, kk = i - r * kFK;
            const int m = m0 + r, n = n0 + r, k = k0 + kk;
            sA[kk][r] = (m < M && k < K) ? A[(long long)m * lda + k] : 0.0f;
            sW[kk][r] = (n < N && k < K) ? W[(long long)n * ldw + k] : 0.0f;
        }
        __syncthreads();
        #pragma unroll
        for (int kk = 0; kk < kFK; ++kk) {
            float a[4], w[4];
            #pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = sA[kk][ty + 16 * i]; w[i] = sW[kk][tx + 16 * i]; }
            #pragma unroll
            for (int i = 0; i < 4; ++i)
                #pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], w[j], acc[i][j]);
        }
        __syncthreads();
    }
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty + 16 * i;
        if (m >= M) continue;
        float tmax = 0.0f;
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx + 16 * j;
            if (n >= N) continue;
            float v = acc[i][j] + (bias ? bias[n] : 0.0f);
            if (mode & kEpiRelu) v = (v < 0.0f) ? 0.0f : v;
            if (mode & kEpiAdd) v = res[(long long)m * ldr + n] + v;
            if (mode & kEpiAddRelu) { v = v + res[(long long)m * ldr + n]; v = v > 0.0f ? v : 0.0f; }
            out[(long long)m * ldo + n] = v;
            tmax = fmaxf(tmax, fabsf(v));
        }
        if (amax) atomicMax(&amax[m / amax_rows], __float_as_uint(tmax));
    }
}

cudaError_t gemm_f32(const float* A, long long lda, const float* W, long long ldw, const float* bias, float* out,
                     long long ldo, const float* res, long long ldr, int M, int N, int K, int mode,
                     unsigned int* amax, int amax_rows, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    dim3 grid((N + kFT - 1) / kFT, (M + kFT - 1) / kFT);
    {
        const cudaError_t le_ = launch_k(gemm_f32_kernel, grid, 256, 0, st,
                                         A, lda, W, ldw, bias, out, ldo, res, ldr, M, N, K, mode, amax,
                                          amax_rows > 0 ? amax_rows : 1);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

__global__ void im2col_f32_kernel(const float* __restrict__ x, int F, int H, int W, int C, int k, int stride, int pad,
                                  int Ho, int Wo, int K, float* __restrict__ col) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long total = (long long)F * Ho * Wo * K;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long row = t / K;
        const int kk = static_cast<int>(t - row * K);
        const int npix = Ho * Wo;
        const int f = static_cast<int>(row / npix);
        const int pix = static_cast<int>(row - (long long)f * npix);
        const int oy = pix / Wo, ox = pix - oy * Wo;
        const int tap = kk / C, ci = kk - tap * C;
        const int ky = tap / k, kx = tap - ky * k;
        const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
        float v = 0.0f;
        if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = x[(((long long)f * H + iy) * W + ix) * C + ci];
        col[t] = v;
    }
}

cudaError_t im2col_f32(const float* x, int F, int H, int W, int C, int k, int stride, int pad, int Ho, int Wo,
                       float* col, cudaStream_t st) {
    const long long total = (long long)F * Ho * Wo * k * k * C;
    if (total <= 0) return cudaErrorInvalidValue;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    {
        const cudaError_t le_ = launch_k(im2col_f32_kernel, (int)blocks, 256, 0, st,
                                         x, F, H, W, C, k, stride, pad, Ho, Wo, k * k * C, col);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace vsb
