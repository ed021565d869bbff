// Norms, positional encoding, activations and the diffusion-policy conv ops of
// the reference's other policy families (src/ops/lm_ops.h, src/ops/conv_ops.h),
// on the GPU. Each kernel evaluates the reference's formula in its order:
//   - where the reference is deterministic fp32/fp64 arithmetic (RMSNorm's
//     sequential double sum, the SIMD bodies of the activations with their
//     Cephes exp, GroupNorm's per-channel sweeps, conv_transpose1d's fixed
//     accumulation order, im2col1d) the results are the reference's bits;
//   - where the reference calls the C library's float functions (silu, and
//     the scalar tails of silu_gate / gelu_tanh / mish past its 8-lane loops)
//     they are glibc's expf / tanhf / log1pf restated (libm_f32.h, bit-equal
//     to the host library on all 2^32 inputs), so those results are the
//     reference's bits too;
//   - spatial_softmax's expf and RoPE's double sin/cos use the device's own
//     functions and agree to the reference tests' tolerances.
// Compiled into kernels.cu after nn.cu (ref_exp, the reference's Cephes exp).
#include "lm_ops.h"
#include "libm_f32.h"

namespace vsb {

// ------------------------------------------------------------------ RMSNorm
// src/hal/common/norms.cpp:19-35: ss = sum over h in order of (double)x*x,
// inv = (float)(1/sqrt(ss/H + eps)), out = x*inv*w. One CTA per row: its
// threads load the row and the weights once (every load issued before any is
// used) and form the exact double products in shared memory; thread 0 adds
// them in the reference's order, which is the row's critical path (H dependent
// double adds).
//
// Optional fused output (q != nullptr): the per-row int8 quantization of the
// normalized row for the next W8A8 GEMM (quantize_rows' arithmetic: absmax
// scale, q8), so the GEMM needs no quantizer launch of its own.
constexpr int kRmsThreads = 128;

__global__ void __launch_bounds__(kRmsThreads)
rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out, int seq,
               int hidden, float eps, int8_t* __restrict__ q, long long ldq, float* __restrict__ qscale) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    extern __shared__ double rms_sq[];                                  // [hidden] squares
    float* xs = reinterpret_cast<float*>(rms_sq + hidden);              // [hidden] x, then the output row
    float* ws = xs + hidden;                                            // [hidden] weights
    __shared__ float s_red[kRmsThreads / 32];
    __shared__ float s_inv;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* xr = x + (long long)t * hidden;
    if (hidden % 4 == 0 && ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(w)) & 15) == 0) {
        #pragma unroll 4
        for (int h = 4 * tid; h < hidden; h += 4 * kRmsThreads) {
            const float4 v = *reinterpret_cast<const float4*>(xr + h);
            const float4 g = *reinterpret_cast<const float4*>(w + h);
            *reinterpret_cast<float4*>(xs + h) = v;
            *reinterpret_cast<float4*>(ws + h) = g;
            *reinterpret_cast<double2*>(rms_sq + h) = make_double2((double)v.x * (double)v.x, (double)v.y * (double)v.y);
            *reinterpret_cast<double2*>(rms_sq + h + 2) =
                make_double2((double)v.z * (double)v.z, (double)v.w * (double)v.w);
        }
    } else {
        #pragma unroll 4
        for (int h = tid; h < hidden; h += kRmsThreads) {
            const float v = xr[h];
            xs[h] = v;
            ws[h] = w[h];
            rms_sq[h] = (double)v * (double)v;
        }
    }
    __syncthreads();
    if (tid == 0) {
        // the next 16 squares are loaded while the current 16 are added, so
        // the chain runs at the double-add latency
        double ss = 0.0;
        int h = 0;
        double2 cur[8], nxt[8];
        const int h16 = hidden & ~15;
        if (h16) {
            #pragma unroll
            for (int u = 0; u < 8; ++u) cur[u] = reinterpret_cast<const double2*>(rms_sq)[u];
        }
        for (; h < h16; h += 16) {
            if (h + 16 < h16) {
                #pragma unroll
                for (int u = 0; u < 8; ++u) nxt[u] = reinterpret_cast<const double2*>(rms_sq + h + 16)[u];
            }
            #pragma unroll
            for (int u = 0; u < 8; ++u) { ss = __dadd_rn(ss, cur[u].x); ss = __dadd_rn(ss, cur[u].y); }
            #pragma unroll
            for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
        }
        for (; h < hidden; ++h) ss = __dadd_rn(ss, rms_sq[h]);
        s_inv = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)hidden), (double)eps)));
    }
    __syncthreads();
    const float inv = s_inv;
    float* orow = out + (long long)t * hidden;
    float am = 0.0f;
    for (int h = tid; h < hidden; h += kRmsThreads) {
        const float v = __fmul_rn(__fmul_rn(xs[h], inv), ws[h]);
        orow[h] = v;
        xs[h] = v;          // read back below by this same thread only
        am = fmaxf(am, fabsf(v));
    }
    if (!q) return;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, off));
    if ((tid & 31) == 0) s_red[tid >> 5] = am;
    __syncthreads();
    #pragma unroll
    for (int i = 0; i < kRmsThreads / 32; ++i) am = fmaxf(am, s_red[i]);
    const float sc = row_scale(am), iv = __fdiv_rn(1.0f, sc);
    int8_t* qr = q + (long long)t * ldq;
    for (long long h = tid; h < ldq; h += kRmsThreads) qr[h] = h < hidden ? q8(xs[h], iv) : 0;
    if (tid == 0) qscale[t] = sc;
}

cudaError_t rmsnorm(const float* x, const float* w, float* out, int seq, int hidden, float eps, cudaStream_t st,
                    int8_t* q, long long ldq, float* qscale) {
    if (seq <= 0 || hidden <= 0 || hidden > 6144 || (q && (ldq < hidden || !qscale))) return cudaErrorInvalidValue;
    const size_t smem = (sizeof(double) + 2 * sizeof(float)) * (size_t)hidden;
    static bool attr = false;
    if (!attr && smem > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)((sizeof(double) + 2 * sizeof(float)) * 6144));
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const cudaError_t e = launch_k(rmsnorm_kernel, seq, kRmsThreads, smem, st, x, w, out, seq, hidden, eps,
                                   q, ldq, qscale);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------------- RoPE NeoX
// src/hal/common/norms.cpp:37-67: theta_0 = pos[t], theta_{i+1} = theta_i *
// theta_scale in double (theta_scale = base^(-2/head_dim), computed on the
// host with the C library's pow like the reference); each head's pair
// (x[i], x[i+half]) rotates by (cos, sin)(theta_i) in double, rounded once to
// float. Thread = (token, i); the theta chain is walked to i in order.
__global__ void rope_neox_kernel(float* __restrict__ x, const int* __restrict__ pos, int seq, int n_heads,
                                 int head_dim, double theta_scale) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int t = blockIdx.x;
    const int half = head_dim / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        double theta = (double)pos[t];
        for (int j = 0; j < i; ++j) theta = __dmul_rn(theta, theta_scale);
        double s, c;
        sincos(theta, &s, &c);
        for (int hh = 0; hh < n_heads; ++hh) {
            float* v = x + ((long long)t * n_heads + hh) * head_dim;
            const double x0 = v[i], x1 = v[i + half];
            v[i] = (float)__fma_rn(x0, c, -__dmul_rn(x1, s));
            v[i + half] = (float)__fma_rn(x0, s, __dmul_rn(x1, c));
        }
    }
}

cudaError_t rope_neox(float* x, const int* pos, int seq, int n_heads, int head_dim, float base, cudaStream_t st) {
    if (seq <= 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2) return cudaErrorInvalidValue;
    const double theta_scale = std::pow((double)base, -2.0 / head_dim);
    const int threads = head_dim / 2 < 256 ? ((head_dim / 2 + 31) / 32) * 32 : 256;
    const cudaError_t e = launch_k(rope_neox_kernel, seq, threads, 0, st, x, pos, seq, n_heads, head_dim, theta_scale);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// -------------------------------------------------------------- activations
// The reference's SIMD bodies (src/hal/common/eltwise.cpp), element by
// element: IEEE divisions, its fma contractions and its Cephes exp.
// `tail`: the element lies past the reference's 8-lane loop, where it runs
// its scalar form with the C library's float functions (eltwise.cpp:52-53,
// :92-93, :244-248); silu is that scalar form everywhere (:67-73).
__device__ __forceinline__ float act_eval(int kind, float v, float u, bool tail) {
    switch (kind) {
        case kActRelu:   // :209-214
            return v < 0.0f ? 0.0f : v;
        case kActSiluGate: {   // :29-47 x / (1 + exp(0 - x)) * u
            const float e = tail ? lf_expf(-v) : ref_exp(__fsub_rn(0.0f, v));
            return __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, e)), u);
        }
        case kActSilu: {   // :67-73 x / (1 + expf(-x))
            return __fdiv_rn(v, __fadd_rn(1.0f, lf_expf(-v)));
        }
        case kActGeluTanh: {
            const float c = 0.7978845608028654f;
            if (tail) {   // :92-93 0.5 v (1 + tanhf(c (v + 0.044715 v^3))), the add contracted
                const float a = __fmul_rn(__fmul_rn(0.044715f, v), v);
                const float t = lf_tanhf(__fmul_rn(c, __fmaf_rn(a, v, v)));
                return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, t));
            }
            // :75-91 v * sigmoid(2c (v + 0.044715 v^3))
            const float v3 = __fmul_rn(__fmul_rn(v, v), v);
            const float y = __fmul_rn(2.0f * c, __fmaf_rn(0.044715f, v3, v));
            const float e = ref_exp(__fsub_rn(0.0f, y));
            return __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, e)));
        }
        case kActGeluErf: {   // :158-183 Abramowitz-Stegun 7.1.26 erf
            const float p = 0.3275911f, a1 = 0.254829592f, a2 = -0.284496736f, a3 = 1.421413741f,
                        a4 = -1.453152027f, a5 = 1.061405429f;
            const float z = __fmul_rn(fabsf(v), 0.70710678118654752f);
            const float t = __fdiv_rn(1.0f, __fmaf_rn(p, z, 1.0f));
            float poly = __fmaf_rn(a5, t, a4);
            poly = __fmaf_rn(poly, t, a3);
            poly = __fmaf_rn(poly, t, a2);
            poly = __fmaf_rn(poly, t, a1);
            poly = __fmul_rn(poly, t);
            const float e = ref_exp(__fsub_rn(0.0f, __fmul_rn(z, z)));
            const float erf_abs = __fmaf_rn(-poly, e, 1.0f);
            const float erf = __int_as_float(__float_as_int(erf_abs) | (__float_as_int(v) & 0x80000000));
            return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erf));
        }
        default: {   // kActMish
            if (tail) return lf_mish(v);   // :244-248 v * tanhf(log1pf(expf(v))), identity softplus above 20
            // :224-243: v * tanh(softplus(v)) = v * m / (m + 2), m = e(e + 2)
            const float e = ref_exp(fminf(v, 20.0f));
            const float m = __fmul_rn(e, __fadd_rn(e, 2.0f));
            return __fmul_rn(v, __fdiv_rn(m, __fadd_rn(m, 2.0f)));
        }
    }
}

__global__ void activation_kernel(int kind, float* out, const float* x, const float* __restrict__ u, long long n) {
    // out may alias x (the reference's in-place activations): each element is
    // read, then written, by the same thread
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long body = n - n % 8;   // the reference's 8-lane loop covers [0, body)
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = act_eval(kind, x[i], u ? u[i] : 0.0f, i >= body);
}

cudaError_t activation(int kind, float* out, const float* x, const float* u, long long n, cudaStream_t st) {
    if (n <= 0 || kind < kActRelu || kind > kActMish || (kind == kActSiluGate && !u)) return cudaErrorInvalidValue;
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const cudaError_t e = launch_k(activation_kernel, (int)blocks, 256, 0, st, kind, out, x, u, n);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------------- GroupNorm
// src/hal/common/conv.cpp:227-318 over x [n_pixels][C]. Per channel, shifted
// by its first pixel K: S1 = sum (x - K), S2 = sum (x - K)^2 in double, pixels
// in order (the reference's sweep when C >= 16 x its threads; with fewer
// channels its per-thread partials reorder the sums - tolerance class). Per
// group: mean, the exact shifted variance, inv; A = inv*scale, B = bias -
// mean*inv*scale; out = x*A + B (fused into one fma as the reference's
// -ffp-contract=fast build does), optional ReLU.
__global__ void groupnorm_stats_kernel(const float* __restrict__ x, int n_pixels, int C, double* __restrict__ S1,
                                       double* __restrict__ S2) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const double K = x[c];
    double s1 = 0.0, s2 = 0.0;
    for (int p = 0; p < n_pixels; ++p) {
        const double d = __dsub_rn((double)x[(long long)p * C + c], K);
        s1 = __dadd_rn(s1, d);
        s2 = __fma_rn(d, d, s2);
    }
    S1[c] = s1;
    S2[c] = s2;
}

__global__ void groupnorm_affine_kernel(const float* __restrict__ x, const double* __restrict__ S1,
                                        const double* __restrict__ S2, const float* __restrict__ scale,
                                        const float* __restrict__ bias, int n_pixels, int C, int groups, float eps,
                                        float* __restrict__ A, float* __restrict__ B) {
    pdl_wait();     // S1 / S2 come from the statistics kernel
    pdl_trigger();
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= groups) return;
    const int gc = C / groups, c0 = g * gc, c1 = c0 + gc;
    const double np = (double)n_pixels, n = np * gc;
    double tot = 0.0;
    for (int c = c0; c < c1; ++c) tot = __dadd_rn(tot, __fma_rn(np, (double)x[c], S1[c]));
    const double mean = __ddiv_rn(tot, n);
    double ss = 0.0;
    for (int c = c0; c < c1; ++c) {
        const double dk = __dsub_rn((double)x[c], mean);
        const double t = __fma_rn(__dmul_rn(2.0, dk), S1[c], S2[c]);
        ss = __dadd_rn(ss, __fma_rn(__dmul_rn(np, dk), dk, t));
    }
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, n), (double)eps)));
    for (int c = c0; c < c1; ++c) {
        A[c] = (float)__dmul_rn(inv, (double)scale[c]);
        B[c] = (float)__fma_rn(-__dmul_rn(mean, inv), (double)scale[c], (double)bias[c]);
    }
}

__global__ void groupnorm_apply_kernel(const float* __restrict__ x, const float* __restrict__ A,
                                       const float* __restrict__ B, float* __restrict__ out, long long total, int C,
                                       int fuse_relu) {
    pdl_wait();     // A / B come from the affine kernel
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int c = static_cast<int>(i % C);
        const float v = __fmaf_rn(x[i], A[c], B[c]);
        out[i] = (fuse_relu && v < 0.0f) ? 0.0f : v;
    }
}

size_t groupnorm_scratch_bytes(int C) { return (size_t)C * (2 * sizeof(double) + 2 * sizeof(float)); }

cudaError_t groupnorm(const float* x, const float* scale, const float* bias, float* out, int n_pixels, int C,
                      int groups, float eps, bool fuse_relu, void* scratch, cudaStream_t st) {
    if (n_pixels <= 0 || C <= 0 || groups <= 0 || C % groups || !scratch ||
        (reinterpret_cast<uintptr_t>(scratch) & 7))
        return cudaErrorInvalidValue;
    double* S1 = static_cast<double*>(scratch);
    double* S2 = S1 + C;
    float* A = reinterpret_cast<float*>(S2 + C);
    float* B = A + C;
    cudaError_t e = launch_k(groupnorm_stats_kernel, (C + 127) / 128, 128, 0, st, x, n_pixels, C, S1, S2);
    if (e != cudaSuccess) return e;
    e = launch_k(groupnorm_affine_kernel, (groups + 63) / 64, 64, 0, st, x, (const double*)S1, (const double*)S2,
                 scale, bias, n_pixels, C, groups, eps, A, B);
    if (e != cudaSuccess) return e;
    const long long total = (long long)n_pixels * C;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    e = launch_k(groupnorm_apply_kernel, (int)blocks, 256, 0, st, x, (const float*)A, (const float*)B, out, total, C,
                 fuse_relu ? 1 : 0);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------- spatial softmax
// src/hal/common/conv.cpp:397-422: per channel of x [n_pixels][C], softmax
// over pixels with the max shift and the expected (x, y) of grid [n_pixels][2];
// sums in pixel order, the coordinate products fused (fma). The reference's
// exp is libm's expf; the device's stands in (tolerance class).
__global__ void spatial_softmax_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                                       float* __restrict__ out, int n_pixels, int C) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    float m = -INFINITY;
    for (int p = 0; p < n_pixels; ++p) {
        const float v = x[(long long)p * C + c];
        if (v > m) m = v;
    }
    float sum = 0.0f, ex = 0.0f, ey = 0.0f;
    for (int p = 0; p < n_pixels; ++p) {
        const float e = expf(__fsub_rn(x[(long long)p * C + c], m));
        sum = __fadd_rn(sum, e);
        ex = __fmaf_rn(e, grid[2 * p], ex);
        ey = __fmaf_rn(e, grid[2 * p + 1], ey);
    }
    const float inv = __fdiv_rn(1.0f, sum);
    out[2 * c] = __fmul_rn(ex, inv);
    out[2 * c + 1] = __fmul_rn(ey, inv);
}

cudaError_t spatial_softmax(const float* x, const float* grid, float* out, int n_pixels, int C, cudaStream_t st) {
    if (n_pixels <= 0 || C <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(spatial_softmax_kernel, (C + 127) / 128, 128, 0, st, x, grid, out, n_pixels, C);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ----------------------------------------------------------------- im2col1d
// src/hal/common/conv.cpp:334-347: col [Tout][k*Cin], row ot = the k input
// rows ot*stride - pad + kt (zeros outside [0, T)).
__global__ void im2col1d_kernel(const float* __restrict__ x, float* __restrict__ col, int T, int Cin, int k,
                                int stride, int pad, int Tout) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long K = (long long)k * Cin, total = (long long)Tout * K;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int ot = static_cast<int>(i / K);
        const int r = static_cast<int>(i - ot * K);
        const int kt = r / Cin, ci = r - kt * Cin;
        const int t = ot * stride - pad + kt;
        col[i] = (t >= 0 && t < T) ? x[(long long)t * Cin + ci] : 0.0f;
    }
}

cudaError_t im2col1d(const float* x, float* col, int T, int Cin, int k, int stride, int pad, int Tout,
                     cudaStream_t st) {
    if (T <= 0 || Cin <= 0 || k <= 0 || stride <= 0 || pad < 0 || Tout <= 0) return cudaErrorInvalidValue;
    const long long total = (long long)Tout * k * Cin;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const cudaError_t e = launch_k(im2col1d_kernel, (int)blocks, 256, 0, st, x, col, T, Cin, k, stride, pad, Tout);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// --------------------------------------------------------- conv_transpose1d
// src/hal/common/conv.cpp:349-395: out [Tout][Cout], Tout = (T-1)*stride -
// 2*pad + k, W [Cin][k][Cout]. Each output starts at its bias and adds
// x[t][ci] * W[ci][kt][co] (one fma each, zero inputs skipped) over kt from
// k-1 down to 0, then ci in order - the reference's accumulation order for
// that output. Thread = one output.
__global__ void conv_transpose1d_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                        const float* __restrict__ bias, float* __restrict__ out, int T, int Cin,
                                        int Cout, int k, int stride, int pad, int Tout) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long total = (long long)Tout * Cout;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int ot = static_cast<int>(i / Cout), co = static_cast<int>(i - (long long)ot * Cout);
        float acc = bias ? bias[co] : 0.0f;
        for (int kt = k - 1; kt >= 0; --kt) {
            const int num = ot + pad - kt;
            if (num < 0 || num % stride) continue;
            const int t = num / stride;
            if (t >= T) continue;
            const float* xt = x + (long long)t * Cin;
            for (int ci = 0; ci < Cin; ++ci) {
                const float v = xt[ci];
                if (v == 0.0f) continue;
                acc = __fmaf_rn(v, W[((long long)ci * k + kt) * Cout + co], acc);
            }
        }
        out[i] = acc;
    }
}

cudaError_t conv_transpose1d(const float* x, const float* W, const float* bias, float* out, int T, int Cin, int Cout,
                             int k, int stride, int pad, cudaStream_t st) {
    const int Tout = (T - 1) * stride - 2 * pad + k;
    if (T <= 0 || Cin <= 0 || Cout <= 0 || k <= 0 || stride <= 0 || pad < 0 || Tout <= 0) return cudaErrorInvalidValue;
    const long long total = (long long)Tout * Cout;
    long long blocks = (total + 127) / 128;
    if (blocks > 148 * 16) blocks = 148 * 16;
    const cudaError_t e = launch_k(conv_transpose1d_kernel, (int)blocks, 128, 0, st, x, W, bias, out, T, Cin, Cout, k,
                                   stride, pad, Tout);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace vsb
