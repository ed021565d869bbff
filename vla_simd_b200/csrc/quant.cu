// Symmetric int8 quantizers (memory-bound kernels).
//
// Row quantizer (activations per token, weights per output row): the same
// arithmetic as the reference's quantize_act_i8 / pack_weights_i8
// (src/hal/common/gemm_i8.cpp:49-54, :76, :150-152):
//   s   = amax > 0 ? max(amax / 127, FLT_MIN) : 1
//   q   = clamp(rne(x * (1/s)), -127, 127)
// with IEEE division (__fdiv_rn) and an explicitly rounded multiply, so the
// int8 values and scales are bit-identical to the CPU's.
//
// Per-tensor quantization for convolutions (src/hal/common/conv.cpp:444-466)
// happens inside the im2col kernel: the producer of the conv input has already
// accumulated its absmax (per frame) into a float-bits slot, so im2col reads
// fp32, quantizes with the frame's scale and writes the int8 patch rows once.
#include "sm100.cuh"
#include "launch.cuh"
#include "quant.h"

#include <cfloat>

namespace vsb {

__device__ __forceinline__ float row_scale(float amax) {
    return amax > 0.0f ? fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN) : 1.0f;
}

__device__ __forceinline__ int8_t q8(float v, float inv) {
    // round, then clamp to +-127; the same as clamping in fp32 first (x.5 at
    // the edge rounds outward either way), which keeps the rounding in the
    // exact small-range form. NaN quantizes to 0 as a plain conversion would.
    float t = __fmul_rn(v, inv);
    t = t != t ? 0.0f : fminf(fmaxf(t, -127.0f), 127.0f);
    return static_cast<int8_t>(f2i_rn_small(t));
}

// fp32 clamp first, then round: quantize_span_i8 (src/hal/common/gemm_i8.cpp:177-207),
// where a clip factor < 1 lets x*inv exceed 127.
__device__ __forceinline__ int8_t q8_span(float v, float inv) {
    float t = __fmul_rn(v, inv);
    t = fminf(fmaxf(t, -127.0f), 127.0f);
    return static_cast<int8_t>(f2i_rn_small(t));
}

// One warp per row (two rows per 64-thread block). x [M][ldx] (+ optional
// addend [M][lda_] added first, in fp32, like ActTransformer::encode's
// xq = x + pos). Writes q [M][ldq] (zero past K) and scale [M]. A second output
// pair (q2/s2) quantizes x without the addend in the same pass. float4 loads /
// 4-byte int8 stores when every row is 16-byte aligned and K % 4 == 0.
template <bool VEC>
__global__ void __launch_bounds__(64)
quantize_rows_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ addend, long long lda_,
                     int M, int K, int8_t* __restrict__ q, long long ldq, float* __restrict__ scale,
                     int8_t* __restrict__ q2, long long ldq2, float* __restrict__ scale2) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int row = blockIdx.x * 2 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const float* xr = x + (long long)row * ldx;
    const float* ar = addend ? addend + (long long)row * lda_ : nullptr;
    float m1 = 0.0f, m2 = 0.0f;
    // unrolled so several rows' loads are in flight (a 3200-wide row is 25
    // vector loads per lane)
    if (VEC) {
        #pragma unroll 8
        for (int k = 4 * lane; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + k);
            m2 = fmaxf(m2, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            if (ar) {
                const float4 t = *reinterpret_cast<const float4*>(ar + k);
                m1 = fmaxf(m1, fmaxf(fmaxf(fabsf(__fadd_rn(v.x, t.x)), fabsf(__fadd_rn(v.y, t.y))),
                                     fmaxf(fabsf(__fadd_rn(v.z, t.z)), fabsf(__fadd_rn(v.w, t.w)))));
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) {
            const float v = xr[k];
            m2 = fmaxf(m2, fabsf(v));
            if (ar) m1 = fmaxf(m1, fabsf(__fadd_rn(v, ar[k])));
        }
    }
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        m1 = fmaxf(m1, __shfl_xor_sync(0xFFFFFFFFu, m1, off));
        m2 = fmaxf(m2, __shfl_xor_sync(0xFFFFFFFFu, m2, off));
    }
    if (!ar) m1 = m2;
    const float s1 = row_scale(m1), inv1 = __fdiv_rn(1.0f, s1);
    const float s2 = row_scale(m2), inv2 = __fdiv_rn(1.0f, s2);
    int8_t* qr = q + (long long)row * ldq;
    int8_t* qr2 = q2 ? q2 + (long long)row * ldq2 : nullptr;
    if (VEC) {
        #pragma unroll 4
        for (int k = 4 * lane; k < K; k += 128) {
            const float4 v = *reinterpret_cast<const float4*>(xr + k);
            if (ar) {
                const float4 t = *reinterpret_cast<const float4*>(ar + k);
                *reinterpret_cast<char4*>(qr + k) =
                    make_char4(q8(__fadd_rn(v.x, t.x), inv1), q8(__fadd_rn(v.y, t.y), inv1),
                               q8(__fadd_rn(v.z, t.z), inv1), q8(__fadd_rn(v.w, t.w), inv1));
            } else {
                *reinterpret_cast<char4*>(qr + k) = make_char4(q8(v.x, inv1), q8(v.y, inv1), q8(v.z, inv1), q8(v.w, inv1));
            }
            if (qr2)
                *reinterpret_cast<char4*>(qr2 + k) = make_char4(q8(v.x, inv2), q8(v.y, inv2), q8(v.z, inv2), q8(v.w, inv2));
        }
        for (long long k = K + 4 * lane; k < ldq; k += 128) *reinterpret_cast<char4*>(qr + k) = make_char4(0, 0, 0, 0);
        if (qr2)
            for (long long k = K + 4 * lane; k < ldq2; k += 128) *reinterpret_cast<char4*>(qr2 + k) = make_char4(0, 0, 0, 0);
    } else {
        for (long long k = lane; k < ldq; k += 32)
            qr[k] = k < K ? q8(ar ? __fadd_rn(xr[k], ar[k]) : xr[k], inv1) : 0;
        if (qr2)
            for (long long k = lane; k < ldq2; k += 32) qr2[k] = k < K ? q8(xr[k], inv2) : 0;
    }
    if (lane == 0) {
        scale[row] = s1;
        if (scale2) scale2[row] = s2;
    }
}

// im2col + per-tensor quantization. x: F frames of NHWC fp32 [H][W][C];
// amax_bits[f] = float bits of frame f's absmax; clip = TCPU_I8_CLIP semantics.
// col [F*Ho*Wo][ldc] int8, patch element order (ky, kx, ci) as the reference's
// im2col_panel (src/hal/common/conv.cpp:142-156), zero for taps outside the
// image and past K. rscale[row] = the frame's scale (one per output row, so the
// GEMM epilogue reads a per-row scale).
// C % 16 == 0: one thread per 16-byte group of an output row (16 channels of
// one tap); 32-bit index math; the per-frame scale computed once per block.
__global__ void __launch_bounds__(256)
im2col_i8_kernel(const float* __restrict__ x, int F, int H, int W, int C, int k, int stride, int pad, int Ho,
                 int Wo, int K, int ldc, const unsigned int* __restrict__ amax_bits, float clip,
                 int8_t* __restrict__ col, float* __restrict__ rscale) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    __shared__ float s_inv[kMaxConvFrames], s_scale[kMaxConvFrames];
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const float amax = __uint_as_float(amax_bits[i]);
        const float s = amax > 0.0f ? fmaxf(__fdiv_rn(__fmul_rn(amax, clip), 127.0f), FLT_MIN) : 1.0f;
        s_scale[i] = s;
        s_inv[i] = __fdiv_rn(1.0f, s);
    }
    __syncthreads();
    const int groups = ldc >> 4;
    const int cg = C >> 4;                       // 16-channel groups per tap
    const int npix = Ho * Wo;
    const int total = F * npix * groups;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int row = t / groups;
        const int g = t - row * groups;
        const int f = row / npix;
        const int pix = row - f * npix;
        const float inv = s_inv[f];
        if (g == 0) rscale[row] = s_scale[f];
        char4 out[4];
        const int oy = pix / Wo, ox = pix - oy * Wo;
        const int tap = g / cg, ci = (g - tap * cg) * 16;
        const int ky = tap / k, kx = tap - ky * k;
        const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
        const bool in = g * 16 < K && iy >= 0 && iy < H && ix >= 0 && ix < W;
        const float4* src = reinterpret_cast<const float4*>(x + (((long long)f * H + (in ? iy : 0)) * W +
                                                                 (in ? ix : 0)) * C + (in ? ci : 0));
        float4 v[4];
        #pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = in ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        #pragma unroll
        for (int i = 0; i < 4; ++i)   // zero taps (padding, past K) quantize to 0
            out[i] = make_char4(q8_span(v[i].x, inv), q8_span(v[i].y, inv), q8_span(v[i].z, inv), q8_span(v[i].w, inv));
        reinterpret_cast<int4*>(col + (long long)row * ldc)[g] = *reinterpret_cast<int4*>(out);
    }
}

// im2col for channel counts that are not a multiple of 16 (the 3-channel
// stem): one thread per 16-byte group of an output row, like the kernel
// above, but element by element: the group's first patch element e = 16g is
// split into (tap, channel) once, then (ky, kx, ci) advance incrementally.
// One 16-byte store per thread (a row's groups are consecutive threads).
__global__ void __launch_bounds__(256)
im2col_i8_bytes_kernel(const float* __restrict__ x, int F, int H, int W, int C, int k, int stride, int pad, int Ho,
                       int Wo, int K, int ldc, const unsigned int* __restrict__ amax_bits, float clip,
                       int8_t* __restrict__ col, float* __restrict__ rscale) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    __shared__ float s_inv[kMaxConvFrames], s_scale[kMaxConvFrames];
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const float amax = __uint_as_float(amax_bits[i]);
        const float s = amax > 0.0f ? fmaxf(__fdiv_rn(__fmul_rn(amax, clip), 127.0f), FLT_MIN) : 1.0f;
        s_scale[i] = s;
        s_inv[i] = __fdiv_rn(1.0f, s);
    }
    __syncthreads();
    const int groups = ldc >> 4;
    const int npix = Ho * Wo;
    const int total = F * npix * groups;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int row = t / groups;
        const int g = t - row * groups;
        const int f = row / npix;
        const int pix = row - f * npix;
        const float inv = s_inv[f];
        if (g == 0) rscale[row] = s_scale[f];
        const int oy = pix / Wo, ox = pix - oy * Wo;
        const int e0 = 16 * g;
        int tap = e0 / C;
        int ci = e0 - tap * C;
        int ky = tap / k, kx = tap - ky * k;
        const float* xf = x + (long long)f * H * W * C;
        // all 16 gathers first (addresses and predicates, then the loads),
        // so they are in flight together; then quantize and pack
        int off[16];
        bool ok[16];
        #pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
            ok[i] = e0 + i < K && iy >= 0 && iy < H && ix >= 0 && ix < W;
            off[i] = (iy * W + ix) * C + ci;
            if (++ci == C) {
                ci = 0;
                if (++kx == k) { kx = 0; ++ky; }
            }
        }
        float v[16];
        #pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = ok[i] ? xf[off[i]] : 0.0f;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        #pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int8_t q = ok[i] ? q8_span(v[i], inv) : 0;
            w[i >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(q)) << (8 * (i & 3));
        }
        reinterpret_cast<int4*>(col + (long long)row * ldc)[g] =
            make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]), static_cast<int>(w[2]), static_cast<int>(w[3]));
    }
}

// Per-frame quantization for the implicit-GEMM convolution: F frames of
// per_frame contiguous floats (NHWC) -> int8 with the scale the im2col path
// uses (frame absmax slot -> s = max(amax * clip / 127, FLT_MIN), 1 if the
// frame is all zero), fscale[f] = s. blockIdx.y = frame; 4 floats per thread
// when per_frame % 4 == 0.
__global__ void quantize_frames_i8_kernel(const float* __restrict__ x, long long per_frame,
                                          const unsigned int* __restrict__ amax_bits, float clip,
                                          int8_t* __restrict__ q, float* __restrict__ fscale, int vec) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int f = blockIdx.y;
    __shared__ float s_inv;
    if (threadIdx.x == 0) {   // the frame's scale once per block
        const float amax = __uint_as_float(amax_bits[f]);
        const float s = amax > 0.0f ? fmaxf(__fdiv_rn(__fmul_rn(amax, clip), 127.0f), FLT_MIN) : 1.0f;
        s_inv = __fdiv_rn(1.0f, s);
        if (blockIdx.x == 0) fscale[f] = s;
    }
    __syncthreads();
    const float inv = s_inv;
    const float* xf = x + (long long)f * per_frame;
    int8_t* qf = q + (long long)f * per_frame;
    const long long stride = (long long)gridDim.x * blockDim.x;
    if (vec) {
        #pragma unroll 4
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; 4 * i < per_frame; i += stride) {
            const float4 v = reinterpret_cast<const float4*>(xf)[i];
            reinterpret_cast<char4*>(qf)[i] =
                make_char4(q8_span(v.x, inv), q8_span(v.y, inv), q8_span(v.z, inv), q8_span(v.w, inv));
        }
    } else {
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < per_frame; i += stride)
            qf[i] = q8_span(xf[i], inv);
    }
}

cudaError_t quantize_frames_i8(const float* x, int F, long long per_frame, const unsigned int* amax_bits, float clip,
                               int8_t* q, float* fscale, cudaStream_t st) {
    if (F <= 0 || per_frame <= 0 || F > 65535) return cudaErrorInvalidValue;
    const int vec = per_frame % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                    ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    const long long items = vec ? per_frame / 4 : per_frame;
    long long bx = (items + 255) / 256;
    if (bx > 148 * 4) bx = 148 * 4;
    const cudaError_t e = launch_k(quantize_frames_i8_kernel, dim3((unsigned)bx, (unsigned)F), 256, 0, st, x,
                                   per_frame, amax_bits, clip, q, fscale, vec);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Space-to-depth quantization for a stride-2 convolution over C <= 4
// channels (the 7x7/2 stem). With ky = 2t + dy and kx = 2u + dx the stride-2
// conv is a stride-1 conv of kt = ceil(k/2) rows and one column over
//   q[f][by][ox][u*16 + (dy*2 + dx)*C + c] = quant(x[f][2by + dy - pad][2(ox + u) + dx - pad][c])
// (zero outside the image, in bytes 4C..15 of a group and in groups u >= kt),
// 64 channels per pixel, by in [0, Hb = Ho + kt - 1). The weights are
// re-indexed the same way once at load, so every int32 sum, and the output,
// is the im2col path's. One thread per 16-byte group (a pixel's u), scale as
// im2col_i8 (frame absmax slot, clip), fscale [F] = the frame scales.
template <int C>
__global__ void __launch_bounds__(256)
s2d_quantize_i8_kernel(const float* __restrict__ x, int F, int H, int W, int pad, int Hb, int Wo, int kt,
                       const unsigned int* __restrict__ amax_bits, float clip, int8_t* __restrict__ q,
                       float* __restrict__ fscale) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    __shared__ float s_inv[kMaxConvFrames];
    for (int i = threadIdx.x; i < F; i += blockDim.x) {
        const float amax = __uint_as_float(amax_bits[i]);
        const float s = amax > 0.0f ? fmaxf(__fdiv_rn(__fmul_rn(amax, clip), 127.0f), FLT_MIN) : 1.0f;
        s_inv[i] = __fdiv_rn(1.0f, s);
        if (blockIdx.x == 0) fscale[i] = s;
    }
    __syncthreads();
    const int total = F * Hb * Wo * 4;
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < total; t += gridDim.x * blockDim.x) {
        const int u = t & 3;
        const int pix = t >> 2;
        const int ox = pix % Wo, r = pix / Wo;
        const int by = r % Hb, f = r / Hb;
        const float inv = s_inv[f];
        const int iy0 = 2 * by - pad, ix0 = 2 * (ox + u) - pad;
        const float* xf = x + (long long)f * H * W * C;
        // all loads first (predicated), then quantize and pack
        float v[4 * C];
        bool ok[4 * C];
        #pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int iy = iy0 + (d >> 1), ix = ix0 + (d & 1);
            const bool in = u < kt && iy >= 0 && iy < H && ix >= 0 && ix < W;
            #pragma unroll
            for (int c = 0; c < C; ++c) {
                ok[d * C + c] = in;
                v[d * C + c] = in ? xf[(iy * W + ix) * C + c] : 0.0f;
            }
        }
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        #pragma unroll
        for (int i = 0; i < 4 * C; ++i) {
            const int8_t b = ok[i] ? q8_span(v[i], inv) : 0;
            w[i >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(b)) << (8 * (i & 3));
        }
        reinterpret_cast<int4*>(q)[t] =
            make_int4(static_cast<int>(w[0]), static_cast<int>(w[1]), static_cast<int>(w[2]), static_cast<int>(w[3]));
    }
}

cudaError_t s2d_quantize_i8(const float* x, int F, int H, int W, int C, int k, int pad, int Ho, int Wo,
                            const unsigned int* amax_bits, float clip, int8_t* q, float* fscale, cudaStream_t st) {
    const int kt = (k + 1) / 2;
    const int Hb = Ho + kt - 1;
    if (!s2d_conv_supported(C, k, 2) || F <= 0 || F > kMaxConvFrames || H <= 0 || W <= 0 || Ho <= 0 || Wo <= 0 || pad < 0 ||
        (reinterpret_cast<uintptr_t>(q) & 15) || (long long)F * Hb * Wo * 4 >= (1LL << 31) ||
        (long long)H * W * C >= (1LL << 31))
        return cudaErrorInvalidValue;
    const long long total = (long long)F * Hb * Wo * 4;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    cudaError_t e = cudaSuccess;
    switch (C) {
        case 1: e = launch_k(s2d_quantize_i8_kernel<1>, (int)blocks, 256, 0, st, x, F, H, W, pad, Hb, Wo, kt, amax_bits,
                             clip, q, fscale); break;
        case 2: e = launch_k(s2d_quantize_i8_kernel<2>, (int)blocks, 256, 0, st, x, F, H, W, pad, Hb, Wo, kt, amax_bits,
                             clip, q, fscale); break;
        case 3: e = launch_k(s2d_quantize_i8_kernel<3>, (int)blocks, 256, 0, st, x, F, H, W, pad, Hb, Wo, kt, amax_bits,
                             clip, q, fscale); break;
        default: e = launch_k(s2d_quantize_i8_kernel<4>, (int)blocks, 256, 0, st, x, F, H, W, pad, Hb, Wo, kt,
                              amax_bits, clip, q, fscale); break;
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

bool s2d_conv_supported(int C, int k, int stride) {
    return stride == 2 && C >= 1 && C <= 4 && k >= 1 && k <= 8;
}

void s2d_repack_weights_host(const int8_t* Wq, int N, int k, int C, long long ldw, int8_t* out) {
    const int kt = (k + 1) / 2;
    const long long ldo = 64LL * kt;
    for (int o = 0; o < N; ++o) {
        int8_t* row = out + (long long)o * ldo;
        for (long long j = 0; j < ldo; ++j) row[j] = 0;
        for (int ky = 0; ky < k; ++ky)
            for (int kx = 0; kx < k; ++kx)
                for (int c = 0; c < C; ++c)
                    row[(ky >> 1) * 64 + (kx >> 1) * 16 + ((ky & 1) * 2 + (kx & 1)) * C + c] =
                        Wq[(long long)o * ldw + ((long long)ky * k + kx) * C + c];
    }
}

// Per-slot absmax of a contiguous tensor: slot = blockIdx.y covers elements
// [slot*per_slot, (slot+1)*per_slot); one atomic per block.
__global__ void absmax_kernel(const float* __restrict__ x, long long per_slot,
                              unsigned int* __restrict__ amax_bits) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const float* xs = x + (long long)blockIdx.y * per_slot;
    float v = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < per_slot;
         i += (long long)gridDim.x * blockDim.x)
        v = fmaxf(v, fabsf(xs[i]));
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    __shared__ float wmax[32];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, wmax[w]);
        atomicMax(&amax_bits[blockIdx.y], __float_as_uint(m));
    }
}

// The reference's CPU panel layout [N/16][Kp/4][16][4] (src/hal/common/gemm_i8.cpp:30-43,
// :79-84) -> device rows [N][ldw] (zero past K).
__global__ void unpack_panels_kernel(const int8_t* __restrict__ panels, int N, int K, int8_t* __restrict__ rows,
                                     long long ldw) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int Kp = (K + 3) & ~3, KG = Kp / 4;
    const long long total = (long long)N * ldw;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int n = static_cast<int>(i / ldw);
        const int k = static_cast<int>(i - (long long)n * ldw);
        int8_t v = 0;
        if (k < K) v = panels[((long long)((n / 16) * KG + k / 4) * 16 + (n % 16)) * 4 + (k % 4)];
        rows[i] = v;
    }
}

cudaError_t unpack_panels_i8(const int8_t* panels, int N, int K, int8_t* rows, long long ldw, cudaStream_t st) {
    if (N <= 0 || K <= 0 || N % 16 || ldw < K) return cudaErrorInvalidValue;
    const long long total = (long long)N * ldw;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    {
        const cudaError_t le_ = launch_k(unpack_panels_kernel, (int)blocks, 256, 0, st,
                                         panels, N, K, rows, ldw);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// q[i] = q8_span(x[i], inv): tcpu::quantize_span_i8 over a flat span.
__global__ void quantize_span_kernel(const float* __restrict__ x, int8_t* __restrict__ q, long long n, float inv) {
    pdl_wait();
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        q[i] = q8_span(x[i], inv);
}

cudaError_t quantize_span_i8(const float* x, int8_t* q, long long n, float inv, cudaStream_t st) {
    if (n < 0) return cudaErrorInvalidValue;
    if (n == 0) return cudaSuccess;
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    {
        const cudaError_t le_ = launch_k(quantize_span_kernel, (int)blocks, 256, 0, st, x, q, n, inv);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// Device rows [N][ldw] -> the reference's CPU panel layout [N/16][Kp/4][16][4]
// followed by the int32 row sums (src/hal/common/gemm_i8.cpp:30-43, :79-89):
// thread = one 4-byte group (n, k/4) of the panels; group k/4 == 0 also sums
// its row (the row sums are exact integer adds in any order).
__global__ void pack_panels_kernel(const int8_t* __restrict__ rows, long long ldw, int N, int K,
                                   int8_t* __restrict__ panels) {
    pdl_wait();
    pdl_trigger();
    const int Kp = (K + 3) & ~3, KG = Kp / 4;
    const long long groups = (long long)N * KG;
    int32_t* rowsum = reinterpret_cast<int32_t*>(panels + (long long)N * Kp);
    for (long long g = blockIdx.x * (long long)blockDim.x + threadIdx.x; g < groups;
         g += (long long)gridDim.x * blockDim.x) {
        const int n = static_cast<int>(g / KG), kg = static_cast<int>(g - (long long)n * KG);
        const int8_t* r = rows + (long long)n * ldw;
        char4 v;
        v.x = 4 * kg + 0 < K ? r[4 * kg + 0] : 0;
        v.y = 4 * kg + 1 < K ? r[4 * kg + 1] : 0;
        v.z = 4 * kg + 2 < K ? r[4 * kg + 2] : 0;
        v.w = 4 * kg + 3 < K ? r[4 * kg + 3] : 0;
        *reinterpret_cast<char4*>(panels + ((long long)((n / 16) * KG + kg) * 16 + (n % 16)) * 4) = v;
        if (kg == 0) {
            int32_t sum = 0;
            for (int k = 0; k < K; ++k) sum += r[k];
            rowsum[n] = sum;
        }
    }
}

cudaError_t pack_panels_i8(const int8_t* rows, long long ldw, int N, int K, int8_t* panels, cudaStream_t st) {
    if (N <= 0 || K <= 0 || N % 16 || ldw < K || (reinterpret_cast<uintptr_t>(panels) & 3)) return cudaErrorInvalidValue;
    const long long groups = (long long)N * ((K + 3) / 4);
    long long blocks = (groups + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    {
        const cudaError_t le_ = launch_k(pack_panels_kernel, (int)blocks, 256, 0, st, rows, ldw, N, K, panels);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t quantize_rows(const float* x, long long ldx, const float* addend, long long ld_add, int M, int K,
                          int8_t* q, long long ldq, float* scale, int8_t* q2, long long ldq2, float* scale2,
                          cudaStream_t st) {
    if (M <= 0 || K <= 0 || ldq < K || (q2 && ldq2 < K)) return cudaErrorInvalidValue;
    const uintptr_t fa = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(addend);
    const uintptr_t qa = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(q2);
    const bool vec = (K % 4 == 0) && (fa & 15) == 0 && (qa & 3) == 0 && (ldx % 4 == 0) &&
                     (!addend || ld_add % 4 == 0) && (ldq % 4 == 0) && (!q2 || ldq2 % 4 == 0);
    const int blocks = (M + 1) / 2;
    if (vec)
        {
            const cudaError_t le_ = launch_k(quantize_rows_kernel<true>, blocks, 64, 0, st,
                                             x, ldx, addend, ld_add, M, K, q, ldq, scale, q2, ldq2, scale2);
            if (le_ != cudaSuccess) return le_;
        }
    else
        {
            const cudaError_t le_ = launch_k(quantize_rows_kernel<false>, blocks, 64, 0, st,
                                             x, ldx, addend, ld_add, M, K, q, ldq, scale, q2, ldq2, scale2);
            if (le_ != cudaSuccess) return le_;
        }
    return cudaGetLastError();
}

cudaError_t im2col_i8(const float* x, int F, int H, int W, int C, int k, int stride, int pad, int Ho, int Wo,
                      long long ldc, const unsigned int* amax_bits, float clip, int8_t* col, float* rscale,
                      cudaStream_t st) {
    const int K = k * k * C;
    if (ldc < K || (ldc & 15) || F <= 0 || F > kMaxConvFrames || (long long)F * H * W * C >= (1LL << 31) ||
        (long long)F * Ho * Wo * (ldc / 16) >= (1LL << 31))
        return cudaErrorInvalidValue;
    const bool v16 = (C % 16 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(col) & 15) == 0);
    const long long rows = (long long)F * Ho * Wo;
    const int threads = 256;
    if (v16) {
        long long blocks = (rows * (ldc / 16) + threads - 1) / threads;
        if (blocks > 148 * 32) blocks = 148 * 32;
        const cudaError_t le_ = launch_k(im2col_i8_kernel, (int)blocks, threads, 0, st, x, F, H, W, C, k, stride, pad,
                                         Ho, Wo, K, (int)ldc, amax_bits, clip, col, rscale);
        if (le_ != cudaSuccess) return le_;
    } else {
        if ((reinterpret_cast<uintptr_t>(col) & 15)) return cudaErrorInvalidValue;
        long long blocks = (rows * (ldc / 16) + threads - 1) / threads;
        if (blocks > 148 * 32) blocks = 148 * 32;
        const cudaError_t le_ = launch_k(im2col_i8_bytes_kernel, (int)blocks, threads, 0, st, x, F, H, W, C, k,
                                         stride, pad, Ho, Wo, K, (int)ldc, amax_bits, clip, col, rscale);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t absmax_slots(const float* x, long long n, long long per_slot, unsigned int* amax_bits,
                         cudaStream_t st) {
    if (n <= 0 || per_slot <= 0 || n % per_slot) return cudaErrorInvalidValue;
    const int threads = 256;
    long long bx = (per_slot + threads - 1) / threads;
    if (bx > 296) bx = 296;
    dim3 grid((unsigned)bx, (unsigned)(n / per_slot));
    {
        const cudaError_t le_ = launch_k(absmax_kernel, grid, threads, 0, st,
                                         x, per_slot, amax_bits);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace vsb
