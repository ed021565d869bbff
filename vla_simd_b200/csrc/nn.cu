// Non-GEMM kernels of the policy step: LayerNorm (+ fused int8 quantization of
// its output for the next W8A8 GEMM), scaled-dot-product attention, max-pool +
// ReLU, camera-frame normalization, and the two tiny fp32 linears ACT keeps in
// full precision (state projection K=6, action head N=6).
#include "sm100.cuh"
#include "nn.h"

#include <cfloat>
#include <cmath>

namespace vsb {

__device__ __forceinline__ float nn_row_scale(float amax) {
    return amax > 0.0f ? fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN) : 1.0f;
}

__device__ __forceinline__ int8_t nn_q8(float v, float inv) {
    int r = __float2int_rn(__fmul_rn(v, inv));
    r = r > 127 ? 127 : r;
    r = r < -127 ? -127 : r;
    return static_cast<int8_t>(r);
}

__device__ __forceinline__ double warp_sum_d(double v) {
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    return v;
}

__device__ __forceinline__ float warp_max_f(float v) {
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    return v;
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row, the row held in registers (H <= 32*VPL). Mean and variance
// accumulate in double, inv = (float)(1/sqrt(var/H + eps)), out = x_c*inv*w + b
// with x_c = (float)(x - mean): the reference's layernorm
// (src/hal/common/norms.cpp:69-97). The affine tail is written as
// fma(x_c*inv, w, b), the contraction the reference's -ffp-contract=fast build
// produces for that expression.
//
// Optional fused outputs, each a per-row int8 quantization of the normalized
// row for the next W8A8 GEMM: q1 of (out + addend) and q2 of out.
template <int VPL>
__global__ void layernorm_kernel(const float* __restrict__ x, float* __restrict__ out, const float* __restrict__ w,
                                 const float* __restrict__ b, int M, int H, float eps,
                                 const float* __restrict__ addend,
                                 int8_t* __restrict__ q1, float* __restrict__ s1,
                                 int8_t* __restrict__ q2, float* __restrict__ s2, long long ldq) {
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const float* xr = x + (long long)row * H;
    float v[VPL];
    double sum = 0.0;
    #pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int h = lane + 32 * i;
        v[i] = h < H ? xr[h] : 0.0f;
        sum += (double)v[i];
    }
    const double mean = warp_sum_d(sum) / H;
    double var = 0.0;
    #pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int h = lane + 32 * i;
        if (h < H) {
            const double d = (double)v[i] - mean;
            var += d * d;
        }
    }
    var = warp_sum_d(var);
    const float inv = (float)(1.0 / sqrt(var / H + (double)eps));
    float* orow = out + (long long)row * H;
    float am1 = 0.0f, am2 = 0.0f;
    const float* ar = addend ? addend + (long long)row * H : nullptr;
    #pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int h = lane + 32 * i;
        if (h < H) {
            const float xc = (float)((double)v[i] - mean);
            const float y = b ? __fmaf_rn(__fmul_rn(xc, inv), w[h], b[h]) : __fmul_rn(__fmul_rn(xc, inv), w[h]);
            v[i] = y;
            orow[h] = y;
            am2 = fmaxf(am2, fabsf(y));
            if (ar) am1 = fmaxf(am1, fabsf(__fadd_rn(y, ar[h])));
        }
    }
    if (q1) {
        const float m = warp_max_f(ar ? am1 : am2);
        const float sc = nn_row_scale(m), iv = __fdiv_rn(1.0f, sc);
        int8_t* qr = q1 + (long long)row * ldq;
        #pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int h = lane + 32 * i;
            if (h < H) qr[h] = nn_q8(ar ? __fadd_rn(v[i], ar[h]) : v[i], iv);
        }
        for (int h = H + lane; h < ldq; h += 32) qr[h] = 0;
        if (lane == 0) s1[row] = sc;
    }
    if (q2) {
        const float m = warp_max_f(am2);
        const float sc = nn_row_scale(m), iv = __fdiv_rn(1.0f, sc);
        int8_t* qr = q2 + (long long)row * ldq;
        #pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int h = lane + 32 * i;
            if (h < H) qr[h] = nn_q8(v[i], iv);
        }
        for (int h = H + lane; h < ldq; h += 32) qr[h] = 0;
        if (lane == 0) s2[row] = sc;
    }
}

cudaError_t layernorm(const float* x, float* out, const float* w, const float* b, int M, int H, float eps,
                      const float* addend, int8_t* q1, float* s1, int8_t* q2, float* s2, long long ldq,
                      cudaStream_t st) {
    if (M <= 0 || H <= 0 || H > 2048 || ((q1 || q2) && ldq < H)) return cudaErrorInvalidValue;
    const int threads = 256;
    const int blocks = (M * 32 + threads - 1) / threads;
    if (H <= 512)
        layernorm_kernel<16><<<blocks, threads, 0, st>>>(x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
    else if (H <= 1024)
        layernorm_kernel<32><<<blocks, threads, 0, st>>>(x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
    else
        layernorm_kernel<64><<<blocks, threads, 0, st>>>(x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- attention
// softmax(Q K^T * scale + mask) V per head, fp32 throughout, flash-style
// (online max / sum over 64-key tiles, scores never leave shared memory).
// Semantics of the reference's gqa_attention_masked / _dense
// (src/hal/avx2/attn.cpp:266-447, src/hal/common/attn.cpp:22-41): grouped KV
// heads (kv = h / (n_q / n_kv)), an optional additive mask [seq_q][seq_k] whose
// -inf / lowest entries block a key, and a fully-blocked row -> the uniform mean
// of V over all seq_k keys.
//
// CTA = 128 threads = 32 queries x 64 keys per tile of one head; thread (ty, tx)
// owns query rows 4ty..4ty+3 and key columns tx, tx+16, tx+32, tx+48 of the
// score tile, and output dims tx, tx+16, tx+32, tx+48 of those rows.
constexpr int kAttQ = 32;
constexpr int kAttK = 64;
constexpr int kAttD = 64;

__global__ void __launch_bounds__(128)
attention_kernel(const float* __restrict__ Q, long long ldq, const float* __restrict__ K, long long ldk,
                 const float* __restrict__ V, long long ldv, float* __restrict__ O, long long ldo,
                 int seq_q, int seq_k, int n_q, int n_kv, float scale, const float* __restrict__ mask) {
    // dynamic shared memory (49.4 KB): Q tile, K^T tile (padded against bank
    // conflicts on the transposed store), V tile, probabilities
    extern __shared__ float att_smem[];
    float (*sQ)[kAttD] = reinterpret_cast<float (*)[kAttD]>(att_smem);
    float (*sKt)[kAttK + 1] = reinterpret_cast<float (*)[kAttK + 1]>(att_smem + kAttQ * kAttD);
    float (*sV)[kAttD] = reinterpret_cast<float (*)[kAttD]>(att_smem + kAttQ * kAttD + kAttD * (kAttK + 1));
    float (*sP)[kAttK] = reinterpret_cast<float (*)[kAttK]>(att_smem + kAttQ * kAttD + kAttD * (kAttK + 1) + kAttK * kAttD);

    const int h = blockIdx.y;
    const int kvh = h / (n_q / n_kv);
    const int q0 = blockIdx.x * kAttQ;
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;   // ty 0..7

    for (int i = tid; i < kAttQ * kAttD; i += 128) {
        const int r = i / kAttD, d = i - r * kAttD;
        const int q = q0 + r;
        sQ[r][d] = q < seq_q ? Q[(long long)q * ldq + (long long)h * kAttD + d] : 0.0f;
    }

    float m_i[4], l_i[4], acc[4][4];
    #pragma unroll
    for (int r = 0; r < 4; ++r) {
        m_i[r] = -INFINITY;
        l_i[r] = 0.0f;
        #pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
    }

    for (int k0 = 0; k0 < seq_k; k0 += kAttK) {
        __syncthreads();
        for (int i = tid; i < kAttK * kAttD; i += 128) {
            const int r = i / kAttD, d = i - r * kAttD;
            const int kk = k0 + r;
            sKt[d][r] = kk < seq_k ? K[(long long)kk * ldk + (long long)kvh * kAttD + d] : 0.0f;
            sV[r][d] = kk < seq_k ? V[(long long)kk * ldv + (long long)kvh * kAttD + d] : 0.0f;
        }
        __syncthreads();

        float s[4][4];
        #pragma unroll
        for (int r = 0; r < 4; ++r)
            #pragma unroll
            for (int c = 0; c < 4; ++c) s[r][c] = 0.0f;
        #pragma unroll 8
        for (int d = 0; d < kAttD; ++d) {
            float qv[4], kv[4];
            #pragma unroll
            for (int r = 0; r < 4; ++r) qv[r] = sQ[4 * ty + r][d];
            #pragma unroll
            for (int c = 0; c < 4; ++c) kv[c] = sKt[d][tx + 16 * c];
            #pragma unroll
            for (int r = 0; r < 4; ++r)
                #pragma unroll
                for (int c = 0; c < 4; ++c) s[r][c] = fmaf(qv[r], kv[c], s[r][c]);
        }

        #pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int q = q0 + 4 * ty + r;
            float tmax = -INFINITY;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int kk = k0 + tx + 16 * c;
                float v = s[r][c] * scale;
                if (kk >= seq_k) v = -INFINITY;
                else if (mask && q < seq_q) {
                    const float mv = mask[(long long)q * seq_k + kk];
                    v = (mv <= -FLT_MAX) ? -INFINITY : v + mv;
                }
                s[r][c] = v;
                tmax = fmaxf(tmax, v);
            }
            // the 16 threads of a row are lanes (ty&1)*16 .. +15 of one warp
            #pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, off));
            const float m_new = fmaxf(m_i[r], tmax);
            const float alpha = (m_i[r] == -INFINITY) ? 0.0f : expf(m_i[r] - m_new);
            float psum = 0.0f;
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float pv = (m_new == -INFINITY) ? 0.0f : expf(s[r][c] - m_new);
                sP[4 * ty + r][tx + 16 * c] = pv;
                psum += pv;
            }
            #pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xFFFFFFFFu, psum, off);
            l_i[r] = l_i[r] * alpha + psum;
            m_i[r] = m_new;
            #pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] *= alpha;
        }
        __syncwarp();
        // sP rows 4ty..4ty+3 are written and read by the same 16 threads
        // (half of one warp), so a warp barrier is enough here.
        const int kn = min(kAttK, seq_k - k0);
        for (int j = 0; j < kn; ++j) {
            float pv[4];
            #pragma unroll
            for (int r = 0; r < 4; ++r) pv[r] = sP[4 * ty + r][j];
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float vv = sV[j][tx + 16 * c];
                #pragma unroll
                for (int r = 0; r < 4; ++r) acc[r][c] = fmaf(pv[r], vv, acc[r][c]);
            }
        }
    }

    // fully-blocked rows: uniform mean of V over every key
    #pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int q = q0 + 4 * ty + r;
        if (q >= seq_q) continue;
        float* o = O + (long long)q * ldo + (long long)h * kAttD;
        if (m_i[r] == -INFINITY) {
            const float u = __fdiv_rn(1.0f, (float)seq_k);
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int d = tx + 16 * c;
                float a = 0.0f;
                for (int kk = 0; kk < seq_k; ++kk) a = fmaf(u, V[(long long)kk * ldv + (long long)kvh * kAttD + d], a);
                o[d] = a;
            }
        } else {
            const float invl = __fdiv_rn(1.0f, l_i[r]);
            #pragma unroll
            for (int c = 0; c < 4; ++c) o[tx + 16 * c] = acc[r][c] * invl;
        }
    }
}

cudaError_t attention(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                      float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, int head_dim, float scale,
                      const float* mask, cudaStream_t st) {
    if (head_dim != kAttD || seq_q <= 0 || seq_k <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv)
        return cudaErrorInvalidValue;
    constexpr size_t smem = sizeof(float) * (kAttQ * kAttD + kAttD * (kAttK + 1) + kAttK * kAttD + kAttQ * kAttK);
    static bool configured = false;
    if (!configured) {
        const cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    dim3 grid((seq_q + kAttQ - 1) / kAttQ, n_q);
    attention_kernel<<<grid, 128, smem, st>>>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask);
    return cudaGetLastError();
}

// --------------------------------------------------------- max-pool + ReLU
// src/hal/common/conv.cpp:192-225: max over the in-image taps, then the folded
// ReLU `!(o > 0) -> 0`. F frames of NHWC. Optional per-frame absmax tap for the
// next conv's per-tensor quantization.
__global__ void maxpool_relu_kernel(const float* __restrict__ x, float* __restrict__ out, int F, int H, int W, int C,
                                    int k, int stride, int pad, int Ho, int Wo, unsigned int* __restrict__ amax) {
    const long long total = (long long)F * Ho * Wo * C;
    const long long per_frame = (long long)Ho * Wo * C;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int f = static_cast<int>(i / per_frame);
        const long long r = i - f * per_frame;
        const int c = static_cast<int>(r % C);
        const int pix = static_cast<int>(r / C);
        const int oy = pix / Wo, ox = pix - oy * Wo;
        float o = -INFINITY;
        const float* xf = x + (long long)f * H * W * C;
        for (int ky = 0; ky < k; ++ky) {
            const int iy = oy * stride - pad + ky;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < k; ++kx) {
                const int ix = ox * stride - pad + kx;
                if (ix < 0 || ix >= W) continue;
                const float v = xf[((long long)iy * W + ix) * C + c];
                o = v > o ? v : o;
            }
        }
        if (!(o > 0.0f)) o = 0.0f;
        out[i] = o;
        if (amax) atomicMax(&amax[f], __float_as_uint(o));
    }
}

cudaError_t maxpool_relu(const float* x, float* out, int F, int H, int W, int C, int k, int stride, int pad,
                         int Ho, int Wo, unsigned int* amax, cudaStream_t st) {
    const long long total = (long long)F * Ho * Wo * C;
    if (total <= 0) return cudaErrorInvalidValue;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    maxpool_relu_kernel<<<(int)blocks, 256, 0, st>>>(x, out, F, H, W, C, k, stride, pad, Ho, Wo, amax);
    return cudaGetLastError();
}

// --------------------------------------------------- camera frame normalize
// uint8 HWC -> (p/255 - mean[c]) / (std[c] + eps), per camera f
// (src/models/act/act_model.cpp:116-121). mean/std are [F][3]. Per-frame absmax tap.
__global__ void normalize_frames_kernel(const uint8_t* __restrict__ img, float* __restrict__ out, int F, long long npx,
                                        const float* __restrict__ mean, const float* __restrict__ stdv, float eps,
                                        unsigned int* __restrict__ amax) {
    const long long per_frame = npx * 3;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < F * per_frame;
         i += (long long)gridDim.x * blockDim.x) {
        const int f = static_cast<int>(i / per_frame);
        const int c = static_cast<int>((i - f * per_frame) % 3);
        const float p = __fdiv_rn((float)img[i], 255.0f);
        const float v = __fdiv_rn(__fsub_rn(p, mean[f * 3 + c]), __fadd_rn(stdv[f * 3 + c], eps));
        out[i] = v;
        if (amax) {
            float a = fabsf(v);
            // frames are whole blocks apart only by chance: reduce per warp when uniform
            const unsigned fk = static_cast<unsigned>(f);
            const unsigned msk = __activemask();
            const unsigned f0 = __shfl_sync(msk, fk, __ffs(msk) - 1);
            if (msk == 0xFFFFFFFFu && __all_sync(msk, fk == f0)) {
                a = warp_max_f(a);
                if ((threadIdx.x & 31) == 0) atomicMax(&amax[f], __float_as_uint(a));
            } else {
                atomicMax(&amax[f], __float_as_uint(a));
            }
        }
    }
}

cudaError_t normalize_frames(const uint8_t* img, float* out, int F, long long npx, const float* mean,
                             const float* stdv, float eps, unsigned int* amax, cudaStream_t st) {
    const long long total = (long long)F * npx * 3;
    if (total <= 0) return cudaErrorInvalidValue;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    normalize_frames_kernel<<<(int)blocks, 256, 0, st>>>(img, out, F, npx, mean, stdv, eps, amax);
    return cudaGetLastError();
}

// ------------------------------------------------------ small fp32 linears
// out[m][n] = bias[n] + sum_k x[m][k] * W[n][k], one warp per output, k in
// order per lane then a fixed tree: fp32 dense_linear (src/hal/avx2/gemm.cpp:98-122)
// up to summation order. Optional elementwise affine on the result
// (out = out*post_mul[n] + post_add[n]: ACT's action unnormalization).
__global__ void linear_f32_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ W,
                                  const float* __restrict__ bias, float* __restrict__ out, long long ldo,
                                  int M, int N, int K, const float* __restrict__ post_mul,
                                  const float* __restrict__ post_add) {
    const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= M * N) return;
    const int m = gw / N, n = gw - m * N;
    const float* xr = x + (long long)m * ldx;
    const float* wr = W + (long long)n * K;
    float a = 0.0f;
    for (int k = lane; k < K; k += 32) a = fmaf(xr[k], wr[k], a);
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xFFFFFFFFu, a, off);
    if (lane == 0) {
        float v = a + (bias ? bias[n] : 0.0f);
        if (post_mul) v = fmaf(v, post_mul[n], post_add[n]);
        out[(long long)m * ldo + n] = v;
    }
}

cudaError_t linear_f32(const float* x, long long ldx, const float* W, const float* bias, float* out, long long ldo,
                       int M, int N, int K, const float* post_mul, const float* post_add, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    const long long threads = (long long)M * N * 32;
    linear_f32_kernel<<<(int)((threads + 255) / 256), 256, 0, st>>>(x, ldx, W, bias, out, ldo, M, N, K, post_mul,
                                                                      post_add);
    return cudaGetLastError();
}

// (state - mean) / (std + eps): ActModel::predict (src/models/act/act_model.cpp:151-153)
__global__ void normalize_state_kernel(const float* __restrict__ s, const float* __restrict__ mean,
                                       const float* __restrict__ stdv, float eps, float* __restrict__ out, int n) {
    const int i = threadIdx.x;
    if (i < n) out[i] = __fdiv_rn(__fsub_rn(s[i], mean[i]), __fadd_rn(stdv[i], eps));
}

cudaError_t normalize_state(const float* s, const float* mean, const float* stdv, float eps, float* out, int n,
                            cudaStream_t st) {
    if (n <= 0 || n > 1024) return cudaErrorInvalidValue;
    normalize_state_kernel<<<1, 1024, 0, st>>>(s, mean, stdv, eps, out, n);
    return cudaGetLastError();
}

// out = a + b, elementwise (fp32 inputs of fp32-path q/k projections)
__global__ void add_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                               long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

cudaError_t add_f32(const float* a, const float* b, float* out, long long n, cudaStream_t st) {
    if (n <= 0) return cudaErrorInvalidValue;
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    add_f32_kernel<<<(int)blocks, 256, 0, st>>>(a, b, out, n);
    return cudaGetLastError();
}

}  // namespace vsb
