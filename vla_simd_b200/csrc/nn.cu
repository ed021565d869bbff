// Non-GEMM kernels of the policy step: LayerNorm (+ fused int8 quantization of
// its output for the next W8A8 GEMM), scaled-dot-product attention, max-pool +
// ReLU, camera-frame normalization, and the two tiny fp32 linears ACT keeps in
// full precision (state projection K=6, action head N=6).
#include "sm100.cuh"
#include "launch.cuh"
#include "nn.h"
#include "quant.h"

#include <cfloat>
#include <cmath>
#include <cstdlib>

namespace vsb {

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("VLA_CUDA_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

__device__ __forceinline__ float nn_row_scale(float amax) {
    return amax > 0.0f ? fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN) : 1.0f;
}

__device__ __forceinline__ int8_t nn_q8(float v, float inv) {
    // round, then clamp to +-127; the same as clamping in fp32 first (x.5 at
    // the edge rounds outward either way), which keeps the rounding in the
    // exact small-range form. NaN quantizes to 0 as a plain conversion would.
    float t = __fmul_rn(v, inv);
    t = t != t ? 0.0f : fminf(fmaxf(t, -127.0f), 127.0f);
    return static_cast<int8_t>(f2i_rn_small(t));
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
template <int V4>
__global__ void __launch_bounds__(64)
layernorm_kernel(const float* __restrict__ x, float* __restrict__ out, const float* __restrict__ w,
                 const float* __restrict__ b, int M, int H, float eps, const float* __restrict__ addend,
                 int8_t* __restrict__ q1, float* __restrict__ s1, int8_t* __restrict__ q2, float* __restrict__ s2,
                 long long ldq) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    // one warp per row (two rows per 64-thread block, so a 602-row input spans
    // every SM); lane l holds float4 groups l, l+32, ... (H % 4 == 0)
    const int row = blockIdx.x * 2 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const int H4 = H >> 2;
    const float4* xr = reinterpret_cast<const float4*>(x + (long long)row * H);
    const float4* ar = addend ? reinterpret_cast<const float4*>(addend + (long long)row * H) : nullptr;
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* b4 = b ? reinterpret_cast<const float4*>(b) : nullptr;
    // the row, and (rows of up to 1024: registers allow) the affine / addend
    // operands of the output pass, all requested up front so their latency
    // overlaps the two reductions
    constexpr bool kHoist = V4 <= 8;
    constexpr int VH = kHoist ? V4 : 1;
    float4 v[V4], wv[VH], bv[VH], av[VH];
    #pragma unroll
    for (int i = 0; i < V4; ++i) {
        const int g = lane + 32 * i;
        const bool in = g < H4;
        v[i] = in ? xr[g] : make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (kHoist) {
            wv[i] = in ? w4[g] : make_float4(0.f, 0.f, 0.f, 0.f);
            bv[i] = (in && b4) ? b4[g] : make_float4(0.f, 0.f, 0.f, 0.f);
            av[i] = (in && ar) ? ar[g] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    double sum = 0.0;
    #pragma unroll
    for (int i = 0; i < V4; ++i) sum += (double)v[i].x + (double)v[i].y + (double)v[i].z + (double)v[i].w;
    const double mean = warp_sum_d(sum) / H;
    double var = 0.0;
    #pragma unroll
    for (int i = 0; i < V4; ++i) {
        if (lane + 32 * i < H4) {
            const double dx = (double)v[i].x - mean, dy = (double)v[i].y - mean;
            const double dz = (double)v[i].z - mean, dw = (double)v[i].w - mean;
            var += dx * dx + dy * dy + dz * dz + dw * dw;
        }
    }
    var = warp_sum_d(var);
    const float inv = (float)(1.0 / sqrt(var / H + (double)eps));
    float4* orow = reinterpret_cast<float4*>(out + (long long)row * H);
    float am1 = 0.0f, am2 = 0.0f;
    float4 a[V4];
    #pragma unroll
    for (int i = 0; i < V4; ++i) {
        const int g = lane + 32 * i;
        if (g < H4) {
            const float4 ww = kHoist ? wv[i % VH] : w4[g];
            const float4 bb = kHoist ? bv[i % VH] : (b4 ? b4[g] : make_float4(0.f, 0.f, 0.f, 0.f));
            float* e = reinterpret_cast<float*>(&v[i]);
            const float* we = reinterpret_cast<const float*>(&ww);
            const float* be = reinterpret_cast<const float*>(&bb);
            #pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float xc = (float)((double)e[c] - mean);
                e[c] = b4 ? __fmaf_rn(__fmul_rn(xc, inv), we[c], be[c]) : __fmul_rn(__fmul_rn(xc, inv), we[c]);
                am2 = fmaxf(am2, fabsf(e[c]));
            }
            orow[g] = v[i];
            if (ar) {
                const float4 t = kHoist ? av[i % VH] : ar[g];
                a[i] = make_float4(__fadd_rn(v[i].x, t.x), __fadd_rn(v[i].y, t.y), __fadd_rn(v[i].z, t.z),
                                   __fadd_rn(v[i].w, t.w));
                am1 = fmaxf(am1, fmaxf(fmaxf(fabsf(a[i].x), fabsf(a[i].y)), fmaxf(fabsf(a[i].z), fabsf(a[i].w))));
            }
        }
    }
    auto store_q = [&](int8_t* qbase, float* sbase, float m, bool use_a) {
        m = warp_max_f(m);
        const float sc = nn_row_scale(m), iv = __fdiv_rn(1.0f, sc);
        char4* qr = reinterpret_cast<char4*>(qbase + (long long)row * ldq);
        #pragma unroll
        for (int i = 0; i < V4; ++i) {
            const int g = lane + 32 * i;
            if (g < H4) {
                const float4 t = use_a ? a[i] : v[i];
                qr[g] = make_char4(nn_q8(t.x, iv), nn_q8(t.y, iv), nn_q8(t.z, iv), nn_q8(t.w, iv));
            }
        }
        for (long long h = H + 4 * lane; h < ldq; h += 128)
            *reinterpret_cast<char4*>(qbase + (long long)row * ldq + h) = make_char4(0, 0, 0, 0);
        if (lane == 0) sbase[row] = sc;
    };
    if (q1) store_q(q1, s1, ar ? am1 : am2, ar != nullptr);
    if (q2) store_q(q2, s2, am2, false);
}

// Scalar twin of layernorm_kernel for rows that are not float4-shaped
// (H % 4 != 0 or unaligned pointers): lane l holds elements l, l+32, ...
template <int VPL>
__global__ void __launch_bounds__(64)
layernorm_scalar_kernel(const float* __restrict__ x, float* __restrict__ out, const float* __restrict__ w,
                        const float* __restrict__ b, int M, int H, float eps, const float* __restrict__ addend,
                        int8_t* __restrict__ q1, float* __restrict__ s1, int8_t* __restrict__ q2,
                        float* __restrict__ s2, long long ldq) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int row = blockIdx.x * 2 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const float* xr = x + (long long)row * H;
    float v[VPL], a[VPL];
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
    for (int i = 0; i < VPL; ++i)
        if (lane + 32 * i < H) {
            const double d = (double)v[i] - mean;
            var += d * d;
        }
    var = warp_sum_d(var);
    const float inv = (float)(1.0 / sqrt(var / H + (double)eps));
    float am1 = 0.0f, am2 = 0.0f;
    #pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int h = lane + 32 * i;
        a[i] = 0.0f;
        if (h < H) {
            const float xc = (float)((double)v[i] - mean);
            v[i] = b ? __fmaf_rn(__fmul_rn(xc, inv), w[h], b[h]) : __fmul_rn(__fmul_rn(xc, inv), w[h]);
            out[(long long)row * H + h] = v[i];
            am2 = fmaxf(am2, fabsf(v[i]));
            if (addend) {
                a[i] = __fadd_rn(v[i], addend[(long long)row * H + h]);
                am1 = fmaxf(am1, fabsf(a[i]));
            }
        }
    }
    for (int pass = 0; pass < 2; ++pass) {
        int8_t* qb = pass == 0 ? q1 : q2;
        if (!qb) continue;
        const bool use_a = pass == 0 && addend;
        const float m = warp_max_f(use_a ? am1 : am2);
        const float sc = nn_row_scale(m), iv = __fdiv_rn(1.0f, sc);
        int8_t* qr = qb + (long long)row * ldq;
        #pragma unroll
        for (int i = 0; i < VPL; ++i) {
            const int h = lane + 32 * i;
            if (h < H) qr[h] = nn_q8(use_a ? a[i] : v[i], iv);
        }
        for (long long h = H + lane; h < ldq; h += 32) qr[h] = 0;
        if (lane == 0) (pass == 0 ? s1 : s2)[row] = sc;
    }
}

cudaError_t layernorm(const float* x, float* out, const float* w, const float* b, int M, int H, float eps,
                      const float* addend, int8_t* q1, float* s1, int8_t* q2, float* s2, long long ldq,
                      cudaStream_t st) {
    if (M <= 0 || H <= 0 || H > 2048 || ((q1 || q2) && ldq < H)) return cudaErrorInvalidValue;
    const uintptr_t f16 = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                          reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(b) |
                          reinterpret_cast<uintptr_t>(addend);
    const uintptr_t q4 = reinterpret_cast<uintptr_t>(q1) | reinterpret_cast<uintptr_t>(q2);
    const bool vec = (H % 4 == 0) && (f16 & 15) == 0 && (q4 & 3) == 0 && (ldq % 4 == 0);
    const int blocks = (M + 1) / 2;
    if (vec) {
        if (H <= 512)
            {
                const cudaError_t le_ = launch_k(layernorm_kernel<4>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
        else if (H <= 1024)
            {
                const cudaError_t le_ = launch_k(layernorm_kernel<8>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
        else
            {
                const cudaError_t le_ = launch_k(layernorm_kernel<16>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
    } else {
        if (H <= 512)
            {
                const cudaError_t le_ = launch_k(layernorm_scalar_kernel<16>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
        else if (H <= 1024)
            {
                const cudaError_t le_ = launch_k(layernorm_scalar_kernel<32>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
        else
            {
                const cudaError_t le_ = launch_k(layernorm_scalar_kernel<64>, blocks, 64, 0, st,
                                                 x, out, w, b, M, H, eps, addend, q1, s1, q2, s2, ldq);
                if (le_ != cudaSuccess) return le_;
            }
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- attention
// softmax(Q K^T * scale + mask) V per head, fp32, reproducing the reference
// x86 kernel's arithmetic (src/hal/avx2/attn.cpp:54-94, :134-162, :210-251)
// operation for operation, so the int8 quantizers that follow see the same
// bits as on the CPU:
//   score[j] = (fma chain over d = 0..63 of q[d]*k[d], from 0) * scale
//              (+ mask[j] for j below the row bound; -inf past it)
//   e[j]     = cephes_exp(score[j] - max)   (0 where score - max <= -87)
//   sum      = 8 lane sums (lane l adds e[l], e[l+8], ... in order), combined
//              ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))    (hsum8, simd.h:52-59)
//   p[j]     = e[j] * (1/sum)
//   out[d]   = fma chain over keys j = 0.. of p[j]*v[j][d], from 0
// A row whose every score is blocked (max <= lowest) gets the uniform mean of V
// (attn_uniform_row, :45-52). Grouped KV heads: kv = h / (n_q / n_kv).
//
// CTA = one head x QT queries, NT threads (16 x 128 at ACT shapes), the whole
// score rows in shared memory (row stride = 8 banks apart). Three phases, each
// a register-tiled loop whose per-output accumulation order is the reference's:
//   scores  thread = QT/(NT/32) queries x 2 keys of a 64-key tile; per d the
//           queries' Q^T values (broadcast) + one 8-byte K^T load feed the fmas
//   softmax 8 threads per row; thread t owns keys j = t (mod 8), i.e. exactly
//           the reference's AVX lane t: its max, exp, and in-order lane sum
//   A*V     thread = QT/(NT/16) queries x 4 dims; keys streamed in order through
//           64-key V tiles, one 16-byte V load per key
constexpr int kAttD = 64;
constexpr int kAttKT = 64;   // keys per shared K^T / V tile

// Independent sequences of one launch (grid z): element strides between them.
#define VSB_ATT_BATCH_OFFSET(bs)                 \
    do {                                         \
        const long long z_ = blockIdx.z;         \
        Q += z_ * (bs).q;                        \
        K += z_ * (bs).k;                        \
        V += z_ * (bs).v;                        \
        O += z_ * (bs).o;                        \
        if (mask) mask += z_ * (bs).mask;        \
    } while (0)

// The reference's Cephes-style exp (src/hal/avx2/simd.h:72-95), lane for lane.
__device__ __forceinline__ float ref_exp(float x) {
    const bool keep = !(x <= -87.0f);
    x = (88.3762626647949f < x) ? 88.3762626647949f : x;
    x = (-88.3762626647950f > x) ? -88.3762626647950f : x;
    float fx = __fmaf_rn(x, 1.44269504088896341f, 0.5f);
    // floor(fx) for |fx| < 2^22 (here |fx| <= 128) in plain fp32 adds: adding
    // and removing 1.5 * 2^23 rounds to the nearest integer exactly, then step
    // down if that went up. Equal to floorf, but on the fma pipe instead of
    // the narrow conversion unit (this exp runs once per attention score).
    constexpr float kRound = 12582912.0f;   // 1.5 * 2^23, bits 0x4B400000
    {
        const float r = __fsub_rn(__fadd_rn(fx, kRound), kRound);
        fx = r > fx ? __fsub_rn(r, 1.0f) : r;
    }
    x = __fmaf_rn(-fx, 0.693359375f, x);
    x = __fmaf_rn(-fx, -2.12194440e-4f, x);
    float y = 1.9875691500e-4f;
    y = __fmaf_rn(y, x, 1.3981999507e-3f);
    y = __fmaf_rn(y, x, 8.3334519073e-3f);
    y = __fmaf_rn(y, x, 4.1665795894e-2f);
    y = __fmaf_rn(y, x, 1.6666665459e-1f);
    y = __fmaf_rn(y, x, 5.0000001201e-1f);
    y = __fmaf_rn(y, __fmul_rn(x, x), __fadd_rn(x, 1.0f));
    const int n = __float_as_int(__fadd_rn(fx, kRound)) - 0x4B400000;   // (int)fx: fx is an integer
    y = __fmul_rn(y, __int_as_float((n + 127) << 23));
    return keep ? y : 0.0f;
}

__host__ __device__ constexpr int att_row_stride(int seq_k) {
    // ceil8(seq_k), rounded to whole bank rows, plus 8 so consecutive rows
    // start 8 banks apart (the softmax phase reads 4 rows per warp)
    return (((seq_k + 7) & ~7) + 31) / 32 * 32 + 8;
}

template <int QT, int NT>
__global__ void __launch_bounds__(NT)
attention_kernel(const float* __restrict__ Q, long long ldq, const float* __restrict__ K, long long ldk,
                 const float* __restrict__ V, long long ldv, float* __restrict__ O, long long ldo,
                 int seq_q, int seq_k, int n_q, int n_kv, float scale, const float* __restrict__ mask,
                 AttBatch bs) {
    VSB_ATT_BATCH_OFFSET(bs);
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    constexpr int QPT = QT / (NT / 32);    // queries per thread, score phase
    constexpr int QPT2 = QT / (NT / 16);   // queries per thread, A*V phase
    static_assert(QPT >= 2 && QPT % 2 == 0 && QPT2 >= 1, "attention tile shape");
    static_assert(NT >= 64 && (QT % (NT / 8) == 0 || NT / 8 >= QT), "softmax row groups");
    extern __shared__ __align__(16) float att_smem[];
    const int ss = att_row_stride(seq_k);
    const int skp = (seq_k + 7) & ~7;
    float* sS = att_smem;                         // [QT][ss] scores -> probabilities
    float* sQt = sS + QT * ss;                    // Q^T [64][QT]
    float* sT = sQt + kAttD * QT;                 // K^T [64][64] or V [64][64]

    const int h = blockIdx.y;
    const int kvh = h / (n_q / n_kv);
    const int q0 = blockIdx.x * QT;
    const int tid = threadIdx.x;
    const float NINF = __int_as_float(0xff800000);

    for (int i = tid; i < QT * kAttD; i += NT) {
        const int q = i % QT, d = i / QT;
        sQt[d * QT + q] = (q0 + q) < seq_q ? Q[(long long)(q0 + q) * ldq + (long long)h * kAttD + d] : 0.0f;
    }

    // ---- scores: thread (tq, tk) -> queries QPT*tq.., keys 2tk, 2tk+1 of the tile
    {
        const int tq = tid >> 5, tk = tid & 31;
        for (int k0 = 0; k0 < seq_k; k0 += kAttKT) {
            __syncthreads();
            // K^T tile: consecutive threads take consecutive keys (conflict-free stores)
            for (int i = tid; i < kAttKT * (kAttD / 4); i += NT) {
                const int key = i % kAttKT, dg = i / kAttKT;
                const int kk = k0 + key;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (kk < seq_k)
                    v = *reinterpret_cast<const float4*>(K + (long long)kk * ldk + (long long)kvh * kAttD + dg * 4);
                sT[(dg * 4 + 0) * kAttKT + key] = v.x;
                sT[(dg * 4 + 1) * kAttKT + key] = v.y;
                sT[(dg * 4 + 2) * kAttKT + key] = v.z;
                sT[(dg * 4 + 3) * kAttKT + key] = v.w;
            }
            __syncthreads();
            float acc[QPT][2];
            #pragma unroll
            for (int a = 0; a < QPT; ++a) { acc[a][0] = 0.0f; acc[a][1] = 0.0f; }
            #pragma unroll 4
            for (int d = 0; d < kAttD; ++d) {
                float qv[QPT];
                #pragma unroll
                for (int a = 0; a < QPT; a += 2) {
                    const float2 t = *reinterpret_cast<const float2*>(sQt + d * QT + QPT * tq + a);
                    qv[a] = t.x;
                    qv[a + 1] = t.y;
                }
                const float2 kv = *reinterpret_cast<const float2*>(sT + d * kAttKT + 2 * tk);
                #pragma unroll
                for (int a = 0; a < QPT; ++a) {
                    acc[a][0] = __fmaf_rn(qv[a], kv.x, acc[a][0]);
                    acc[a][1] = __fmaf_rn(qv[a], kv.y, acc[a][1]);
                }
            }
            const int kk = k0 + 2 * tk;
            if (kk < skp) {
                #pragma unroll
                for (int a = 0; a < QPT; ++a)
                    *reinterpret_cast<float2*>(sS + (QPT * tq + a) * ss + kk) =
                        make_float2(__fmul_rn(acc[a][0], scale), __fmul_rn(acc[a][1], scale));
            }
        }
    }
    __syncthreads();

    // ---- softmax rows: 8 threads per row, thread t = the reference's lane t
    {
        const int t = tid & 7;
        for (int r = tid >> 3; r < QT; r += NT / 8) {   // rows of 8 threads (whole warps leave together)
            const int q = q0 + r;
            float* srow = sS + r * ss;
            const float* mrow = (mask && q < seq_q) ? mask + (long long)q * seq_k : nullptr;
            // row bound: trailing `lowest` mask entries block keys (hal::row_bound).
            // The shuffle is outside any row-dependent branch: every lane of
            // the warp reaches it (rows past seq_q have no mask row).
            int last = seq_k - 1;
            if (mrow) {
                last = -1;
                for (int j = t; j < seq_k; j += 8)
                    if (mrow[j] != -FLT_MAX) last = j;
            }
            #pragma unroll
            for (int off = 4; off > 0; off >>= 1) last = max(last, __shfl_xor_sync(0xFFFFFFFFu, last, off));
            const int jmax = last + 1;
            float mx = NINF;
            for (int j = t; j < skp; j += 8) {
                float v = srow[j];
                if (j >= jmax) v = NINF;
                else if (mrow) v = __fadd_rn(v, mrow[j]);
                srow[j] = v;
                mx = fmaxf(mx, v);
            }
            #pragma unroll
            for (int off = 4; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, off));
            const bool degenerate = !(mx > -FLT_MAX);
            float lane_sum = 0.0f;
            if (!degenerate) {
                for (int j = t; j < skp; j += 8) {
                    const float e = ref_exp(__fsub_rn(srow[j], mx));
                    srow[j] = e;
                    lane_sum = __fadd_rn(lane_sum, e);
                }
            }
            float l[8];
            #pragma unroll
            for (int i = 0; i < 8; ++i) l[i] = __shfl_sync(0xFFFFFFFFu, lane_sum, (threadIdx.x & 24) | i);
            const float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                                        __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
            if (degenerate) {
                // fully blocked row: uniform weights over every key (attn_uniform_row)
                const float u = __fdiv_rn(1.0f, (float)seq_k);
                for (int j = t; j < skp; j += 8) srow[j] = j < seq_k ? u : 0.0f;
            } else {
                const float inv = __fdiv_rn(1.0f, sum);
                for (int j = t; j < skp; j += 8) srow[j] = __fmul_rn(srow[j], inv);
            }
        }
    }

    // ---- A*V: thread (tq2, td) -> queries QPT2*tq2.., dims 4td..4td+3, keys in order
    const int tq2 = tid >> 4, td = tid & 15;
    float o[QPT2][4];
    #pragma unroll
    for (int a = 0; a < QPT2; ++a)
        #pragma unroll
        for (int c = 0; c < 4; ++c) o[a][c] = 0.0f;
    for (int k0 = 0; k0 < seq_k; k0 += kAttKT) {
        __syncthreads();
        for (int i = tid; i < kAttKT * (kAttD / 4); i += NT) {
            const int key = i / (kAttD / 4), dg = i % (kAttD / 4);
            const int kk = k0 + key;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kk < seq_k)
                v = *reinterpret_cast<const float4*>(V + (long long)kk * ldv + (long long)kvh * kAttD + dg * 4);
            *reinterpret_cast<float4*>(sT + key * kAttD + dg * 4) = v;
        }
        __syncthreads();
        const int kn = min(kAttKT, seq_k - k0);
        for (int j = 0; j < kn; ++j) {
            const float4 vv = *reinterpret_cast<const float4*>(sT + j * kAttD + 4 * td);
            #pragma unroll
            for (int a = 0; a < QPT2; ++a) {
                const float pv = sS[(QPT2 * tq2 + a) * ss + k0 + j];
                o[a][0] = __fmaf_rn(pv, vv.x, o[a][0]);
                o[a][1] = __fmaf_rn(pv, vv.y, o[a][1]);
                o[a][2] = __fmaf_rn(pv, vv.z, o[a][2]);
                o[a][3] = __fmaf_rn(pv, vv.w, o[a][3]);
            }
        }
    }
    #pragma unroll
    for (int a = 0; a < QPT2; ++a) {
        const int q = q0 + QPT2 * tq2 + a;
        if (q < seq_q)
            *reinterpret_cast<float4*>(O + (long long)q * ldo + (long long)h * kAttD + 4 * td) =
                make_float4(o[a][0], o[a][1], o[a][2], o[a][3]);
    }
}

// ---- register-tiled variant (the default wherever its score rows fit)
// CTA = one head x QP = 8*QPT query rows, 256 threads (two warps per SM
// sub-partition), K and V streamed through 128-key tiles. Warp w, lane l:
//   scores  rows 4*QPT*(w&1) + QPT*(l/8) + a (a < QPT), keys 32*(w/2) + l%8 + 8i
//           (i < 4) of the tile: per 4 dims, QPT 16-byte Q loads (4 distinct
//           addresses per warp) and 4 16-byte K loads (8 consecutive rows)
//           feed 16*QPT fmas, one shared-memory wavefront per load;
//   softmax warp w takes rows QPT*w ..: row bound, masked max, exp and the
//           final scaling are elementwise over all 32 lanes; only the
//           reference's 8 in-order lane sums run 8 lanes per row;
//   A*V     the score phase's rows, dims 16*(w/2) + 2*(l%8) + {0,1}: per 4 keys, QPT
//           16-byte probability loads and 4 8-byte V loads feed 8*QPT fmas.
// K/V rows are 68 floats apart in shared memory (conflict-free 16-byte
// loads); tiles are double-buffered with cp.async. Every per-output
// accumulation runs in the reference's order (d = 0..63 for a score, keys in
// order for an output), so the results are the reference's bits.
constexpr int kAttRS = 68;   // floats per Q / K / V row in shared memory
constexpr int kAttTK = 128;  // keys per K / V tile

__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 :: "r"(smem_u32(sdst)), "l"(gsrc), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__host__ __device__ constexpr size_t att_tiled_smem(int qp, int seq_k) {
    return sizeof(float) * ((size_t)qp * att_row_stride(seq_k) + (size_t)qp * kAttRS + 2 * kAttTK * kAttRS);
}
// the same with every K (then V) tile resident at once (kv_all)
__host__ __device__ constexpr size_t att_tiled_smem_all(int qp, int seq_k) {
    return sizeof(float) * ((size_t)qp * att_row_stride(seq_k) + (size_t)qp * kAttRS +
                            (size_t)((seq_k + kAttTK - 1) / kAttTK) * kAttTK * kAttRS);
}

// Fused row quantization of a finished attention output tile (AttQuant): the
// CTA's O stores are made visible, its arrival counted; the last CTA of the
// query tile (one per head, gridDim.y of them) reads the tile's rows back
// through L2 and quantizes them as quantize_rows does. Warp w takes rows
// w + 8j (j < QPT); CH = 16-byte chunks per lane per row (rows of up to
// 128*CH columns), and the loads of RB rows are issued before any is used.
template <int QPT, int CH>
__device__ __forceinline__ void att_quant_rows(const float* O, long long ldo, int q0, int seq_q, int kdim,
                                               const AttQuant& qz) {
    constexpr int RB = 20 / CH < QPT ? 20 / CH : QPT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int8_t* qb = qz.q + (long long)blockIdx.z * qz.zq;
    float* sb = qz.scale + (long long)blockIdx.z * qz.zs;
    for (int j0 = 0; j0 < QPT; j0 += RB) {
        float4 v[RB][CH];
        #pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int q = q0 + warp + 8 * (j0 + b);
            const bool ok = j0 + b < QPT && q < seq_q;
            const float* orow = O + (long long)q * ldo;
            #pragma unroll
            for (int i = 0; i < CH; ++i) {
                const int k = 4 * lane + 128 * i;
                v[b][i] = (ok && k < kdim) ? __ldcg(reinterpret_cast<const float4*>(orow + k))
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        #pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int q = q0 + warp + 8 * (j0 + b);
            if (!(j0 + b < QPT && q < seq_q)) continue;     // warp-uniform
            float m = 0.0f;
            #pragma unroll
            for (int i = 0; i < CH; ++i)
                m = fmaxf(m, fmaxf(fmaxf(fabsf(v[b][i].x), fabsf(v[b][i].y)), fmaxf(fabsf(v[b][i].z), fabsf(v[b][i].w))));
            m = warp_max_f(m);
            const float sc = nn_row_scale(m), inv = __fdiv_rn(1.0f, sc);
            int8_t* qr = qb + (long long)q * qz.ldq;
            #pragma unroll
            for (int i = 0; i < CH; ++i) {
                const int k = 4 * lane + 128 * i;
                if (k < kdim)
                    *reinterpret_cast<char4*>(qr + k) = make_char4(nn_q8(v[b][i].x, inv), nn_q8(v[b][i].y, inv),
                                                                   nn_q8(v[b][i].z, inv), nn_q8(v[b][i].w, inv));
            }
            for (long long k = kdim + 4 * lane; k < qz.ldq; k += 128)
                *reinterpret_cast<char4*>(qr + k) = make_char4(0, 0, 0, 0);
            if (lane == 0) sb[q] = sc;
        }
    }
}

template <int QPT>
__device__ __forceinline__ void att_fused_quant(const float* O, long long ldo, int q0, int seq_q, int kdim,
                                                const AttQuant& qz) {
    // the barrier orders the CTA's stores before thread 0's fence, which makes
    // them visible device-wide before its arrival is counted (the pattern of a
    // cooperative grid barrier); the last arrival fences again before reading
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int* c = qz.counters + ((long long)blockIdx.z * gridDim.x + blockIdx.x);
        __threadfence();
        const unsigned int prev = atomicAdd(c, 1u);
        const int last = prev + 1 == gridDim.y;
        if (last) {
            atomicExch(c, 0u);   // every head of the tile has arrived: ready for the next launch
            __threadfence();
        }
        s_last = last;
    }
    __syncthreads();
    if (!s_last) return;
    if (kdim <= 512) att_quant_rows<QPT, 4>(O, ldo, q0, seq_q, kdim, qz);
    else if (kdim <= 768) att_quant_rows<QPT, 6>(O, ldo, q0, seq_q, kdim, qz);
    else att_quant_rows<QPT, 8>(O, ldo, q0, seq_q, kdim, qz);
}

template <int QPT>
__global__ void __launch_bounds__(256, 1)
attention_tiled_kernel(const float* __restrict__ Q, long long ldq, const float* __restrict__ K, long long ldk,
                       const float* __restrict__ V, long long ldv, float* __restrict__ O, long long ldo,
                       int seq_q, int seq_k, int n_q, int n_kv, float scale, const float* __restrict__ mask,
                       AttBatch bs, AttQuant qz, int kv_all) {
    VSB_ATT_BATCH_OFFSET(bs);
    constexpr int QP = 8 * QPT;
    constexpr int kTile = kAttTK * kAttRS;
    extern __shared__ __align__(16) float att_smem[];
    const int ss = att_row_stride(seq_k);
    const int skp = (seq_k + 7) & ~7;
    float* sS = att_smem;               // [QP][ss] scores -> probabilities
    float* sQ = sS + QP * ss;           // [QP][kAttRS]
    float* sKV = sQ + QP * kAttRS;      // [2][kAttTK][kAttRS] K tiles, then V tiles

    const int h = blockIdx.y;
    const int kvh = h / (n_q / n_kv);
    const int q0 = blockIdx.x * QP;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane & 7;
    const int r0 = (warp & 1) * (4 * QPT) + (lane >> 3) * QPT;   // this thread's first row
    const int c0 = (warp >> 1) * 32;                              // key offset (scores) in the tile
    const int d0 = (warp >> 1) * 16 + 2 * g;                      // first of two output dims
    const float NINF = __int_as_float(0xff800000);
    const float* Kh = K + (long long)kvh * kAttD;
    const float* Vh = V + (long long)kvh * kAttD;

    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();

    // Keys past every row's bound (trailing `lowest` mask entries, hal::row_bound)
    // are never read: their probabilities are 0 and an fma with 0 leaves a chain
    // unchanged, so the CTA stops at the largest bound of its rows (a fully
    // blocked row keeps every key: it takes the uniform mean of V).
    // Each row's bound is found once (kept for the softmax in s_rowlast), with
    // four of a lane's mask loads in flight at a time.
    __shared__ int s_kend;
    __shared__ int s_rowlast[QP];
    if (tid == 0) s_kend = mask ? 0 : seq_k;
    __syncthreads();
    if (mask) {
        for (int r = warp; r < QP; r += 8) {
            const int q = q0 + r;
            if (q >= seq_q) continue;
            const float* mr = mask + (long long)q * seq_k;
            int last = -1;
            #pragma unroll 4
            for (int j = lane; j < seq_k; j += 32)
                if (mr[j] != -FLT_MAX) last = j;
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) last = max(last, __shfl_xor_sync(0xFFFFFFFFu, last, off));
            if (lane == 0) {
                s_rowlast[r] = last;
                atomicMax(&s_kend, last < 0 ? seq_k : last + 1);
            }
        }
    }
    __syncthreads();
    const int kend = s_kend;
    const int skp_c = (kend + 7) & ~7;
    const int ntiles = (kend + kAttTK - 1) / kAttTK;

    // kAttTK rows x 16 chunks of 16 bytes; rows past seq_k are zero-filled
    auto load_tile = [&](const float* base, long long ld, int k0, float* dst) {
        for (int i = tid; i < kAttTK * 16; i += 256) {
            const int r = i >> 4, c = i & 15;
            const bool ok = k0 + r < seq_k;
            cp_async16(dst + r * kAttRS + c * 4, base + (long long)(ok ? k0 + r : 0) * ld + c * 4, ok ? 16 : 0);
        }
    };
    for (int i = tid; i < QP * 16; i += 256) {
        const int r = i >> 4, c = i & 15;
        const bool ok = q0 + r < seq_q;
        cp_async16(sQ + r * kAttRS + c * 4, Q + (long long)(ok ? q0 + r : 0) * ldq + (long long)h * kAttD + c * 4,
                   ok ? 16 : 0);
    }
    // kv_all (short query tiles, whose per-tile work is too short for a
    // double buffer to hide the next tile's load): every K tile in one group,
    // one wait; then every V tile, issued before the softmax
    if (kv_all) {
        for (int t = 0; t < ntiles; ++t) load_tile(Kh, ldk, t * kAttTK, sKV + t * kTile);
    } else {
        load_tile(Kh, ldk, 0, sKV);
    }
    cp_async_commit();
    if (kv_all) {
        cp_async_wait_all();
        __syncthreads();
    }

    // ---- scores
    for (int t = 0; t < ntiles; ++t) {
        const float* cur = sKV + (kv_all ? t : (t & 1)) * kTile + (c0 + g) * kAttRS;
        if (!kv_all) {
            if (t + 1 < ntiles) load_tile(Kh, ldk, (t + 1) * kAttTK, sKV + ((t + 1) & 1) * kTile);
            cp_async_commit();
            cp_async_wait_prev();       // tile t (and Q) have landed
            __syncthreads();
        }
        float acc[QPT][4];
        #pragma unroll
        for (int a = 0; a < QPT; ++a)
            #pragma unroll
            for (int i = 0; i < 4; ++i) acc[a][i] = 0.0f;
        #pragma unroll
        for (int d = 0; d < kAttD; d += 4) {
            float4 qv[QPT], kv[4];
            #pragma unroll
            for (int a = 0; a < QPT; ++a) qv[a] = *reinterpret_cast<const float4*>(sQ + (r0 + a) * kAttRS + d);
            #pragma unroll
            for (int i = 0; i < 4; ++i) kv[i] = *reinterpret_cast<const float4*>(cur + 8 * i * kAttRS + d);
            // d, d+1, d+2, d+3 in order per accumulator; consecutive fmas
            // touch different accumulators (no dependent back-to-back issue)
            #pragma unroll
            for (int a = 0; a < QPT; ++a)
                #pragma unroll
                for (int i = 0; i < 4; ++i) acc[a][i] = __fmaf_rn(qv[a].x, kv[i].x, acc[a][i]);
            #pragma unroll
            for (int a = 0; a < QPT; ++a)
                #pragma unroll
                for (int i = 0; i < 4; ++i) acc[a][i] = __fmaf_rn(qv[a].y, kv[i].y, acc[a][i]);
            #pragma unroll
            for (int a = 0; a < QPT; ++a)
                #pragma unroll
                for (int i = 0; i < 4; ++i) acc[a][i] = __fmaf_rn(qv[a].z, kv[i].z, acc[a][i]);
            #pragma unroll
            for (int a = 0; a < QPT; ++a)
                #pragma unroll
                for (int i = 0; i < 4; ++i) acc[a][i] = __fmaf_rn(qv[a].w, kv[i].w, acc[a][i]);
        }
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int key = t * kAttTK + c0 + g + 8 * i;
            if (key < skp) {
                #pragma unroll
                for (int a = 0; a < QPT; ++a) sS[(r0 + a) * ss + key] = __fmul_rn(acc[a][i], scale);
            }
        }
        if (!kv_all) __syncthreads();   // the buffer is refilled two tiles on
    }
    if (kv_all) {
        __syncthreads();                // every K read done: V takes its place
        for (int t = 0; t < ntiles; ++t) load_tile(Vh, ldv, t * kAttTK, sKV + t * kTile);
    } else {
        load_tile(Vh, ldv, 0, sKV);     // V tile 0 streams in during the softmax
    }
    cp_async_commit();

    // ---- softmax: warp w takes rows QPT*w + k (k < QPT), processed together
    // so every pass has QPT independent chains in flight
    {
        float* srow[QPT];
        const float* mrow[QPT];
        int jmax[QPT];
        float mx[QPT];
        #pragma unroll
        for (int k = 0; k < QPT; ++k) {
            const int r = QPT * warp + k;
            const int q = q0 + r;
            srow[k] = sS + r * ss;
            mrow[k] = (mask && q < seq_q) ? mask + (long long)q * seq_k : nullptr;
            // row bound: trailing `lowest` mask entries block keys (hal::row_bound)
            jmax[k] = mrow[k] ? s_rowlast[r] + 1 : seq_k;
            mx[k] = NINF;
        }
        // Each pass loads all of an iteration's elements before storing any:
        // the row pointers may alias as far as the compiler knows, so a
        // load-compute-store sequence per element would serialize on the
        // shared-memory latency (and on the exp chain).
        // (branch-free bodies: selects, so the QPT rows' chains interleave)
        if (mask) {
            for (int j = lane; j < skp_c; j += 32) {
                float v[QPT];
                #pragma unroll
                for (int k = 0; k < QPT; ++k) v[k] = srow[k][j];
                #pragma unroll
                for (int k = 0; k < QPT; ++k) {
                    const float mv = (mrow[k] && j < jmax[k]) ? mrow[k][j] : 0.0f;
                    v[k] = j >= jmax[k] ? NINF : (mrow[k] ? __fadd_rn(v[k], mv) : v[k]);
                    mx[k] = fmaxf(mx[k], v[k]);
                }
                #pragma unroll
                for (int k = 0; k < QPT; ++k) srow[k][j] = v[k];
            }
        } else {
            for (int j = lane; j < skp_c; j += 32) {
                float v[QPT];
                #pragma unroll
                for (int k = 0; k < QPT; ++k) v[k] = srow[k][j];
                #pragma unroll
                for (int k = 0; k < QPT; ++k) {
                    v[k] = j >= seq_k ? NINF : v[k];
                    mx[k] = fmaxf(mx[k], v[k]);
                }
                if (j >= seq_k) {
                    #pragma unroll
                    for (int k = 0; k < QPT; ++k) srow[k][j] = NINF;
                }
            }
        }
        #pragma unroll
        for (int k = 0; k < QPT; ++k)
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xFFFFFFFFu, mx[k], off));
        const float u = __fdiv_rn(1.0f, (float)seq_k);
        for (int j = lane; j < skp_c; j += 32) {
            float v[QPT];
            #pragma unroll
            for (int k = 0; k < QPT; ++k) v[k] = srow[k][j];
            #pragma unroll
            for (int k = 0; k < QPT; ++k) {
                // a fully blocked row (max <= lowest) takes uniform weights over
                // every key (attn_uniform_row); the scaling pass leaves it alone.
                // The exp is computed either way (no branch), then selected.
                const float e = ref_exp(__fsub_rn(v[k], mx[k]));
                v[k] = mx[k] > -FLT_MAX ? e : (j < seq_k ? u : 0.0f);
            }
            #pragma unroll
            for (int k = 0; k < QPT; ++k) srow[k][j] = v[k];
        }
        __syncwarp();
        // the reference's 8 lane sums: lane t adds e[t], e[t+8], ... in order,
        // combined ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7)). Lane l runs sum
        // (l % 8) of rows k = l/8, l/8 + 4 (two chains per lane).
        const int t = lane & 7, kk = lane >> 3;
        float s0 = 0.0f, s1 = 0.0f;
        const float* rowa = kk < QPT ? sS + (QPT * warp + kk) * ss : nullptr;
        const float* rowb = kk + 4 < QPT ? sS + (QPT * warp + kk + 4) * ss : nullptr;
        if (rowa && rowb) {
            #pragma unroll 4
            for (int j = t; j < skp_c; j += 8) { s0 = __fadd_rn(s0, rowa[j]); s1 = __fadd_rn(s1, rowb[j]); }
        } else if (rowa) {
            #pragma unroll 8
            for (int j = t; j < skp_c; j += 8) s0 = __fadd_rn(s0, rowa[j]);
        }
        float inv[QPT];
        #pragma unroll
        for (int k = 0; k < QPT; ++k) {
            float l[8];
            #pragma unroll
            for (int i = 0; i < 8; ++i) l[i] = __shfl_sync(0xFFFFFFFFu, k < 4 ? s0 : s1, 8 * (k & 3) + i);
            const float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                                        __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
            inv[k] = __fdiv_rn(1.0f, sum);
        }
        for (int j = lane; j < skp_c; j += 64) {
            const bool two = j + 32 < skp_c;
            float v[QPT], w[QPT];
            #pragma unroll
            for (int k = 0; k < QPT; ++k) {
                v[k] = srow[k][j];
                w[k] = two ? srow[k][j + 32] : 0.0f;
            }
            #pragma unroll
            for (int k = 0; k < QPT; ++k) {
                if (mx[k] > -FLT_MAX) {
                    srow[k][j] = __fmul_rn(v[k], inv[k]);
                    if (two) srow[k][j + 32] = __fmul_rn(w[k], inv[k]);
                }
            }
        }
    }

    // ---- A*V. For 32- and 40-row tiles, 128 threads take QPT rows x 4 dims
    // each (per 4 keys QPT + 4 16-byte loads feed 16*QPT fmas: 0.45 loaded
    // floats per fma at QPT = 5, against 0.7 for QPT rows x 2 dims over 256
    // threads); the other threads only load and synchronize. Shorter tiles:
    // QPT rows x 2 dims over all 256 threads. Keys in order per output either way.
    constexpr bool kPv4 = QPT >= 4;
    constexpr int PC = kPv4 ? 4 : 2;
    const bool pv_on = !kPv4 || tid < 128;
    const int pr0 = kPv4 ? QPT * (tid >> 4) : r0;
    const int pd0 = kPv4 ? 4 * (tid & 15) : d0;
    float o[QPT][PC];
    #pragma unroll
    for (int a = 0; a < QPT; ++a)
        #pragma unroll
        for (int c = 0; c < PC; ++c) o[a][c] = 0.0f;
    if (kv_all) {
        cp_async_wait_all();
        __syncthreads();                // also: the softmax is done
    }
    for (int t = 0; t < ntiles; ++t) {
        const float* cur = sKV + (kv_all ? t : (t & 1)) * kTile + pd0;
        if (!kv_all) {
            if (t + 1 < ntiles) load_tile(Vh, ldv, (t + 1) * kAttTK, sKV + ((t + 1) & 1) * kTile);
            cp_async_commit();
            cp_async_wait_prev();
            __syncthreads();            // also: the softmax is done before tile 0
        }
        const int k0 = t * kAttTK;
        const int kn = min(kAttTK, kend - k0);
        const float* prow = sS + pr0 * ss + k0;
        if (pv_on) {
            int j = 0;
            #pragma unroll 2
            for (; j + 4 <= kn; j += 4) {
                float4 pv[QPT];
                float vv[4][PC];
                #pragma unroll
                for (int a = 0; a < QPT; ++a) pv[a] = *reinterpret_cast<const float4*>(prow + a * ss + j);
                #pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if constexpr (kPv4) {
                        const float4 v4 = *reinterpret_cast<const float4*>(cur + (j + i) * kAttRS);
                        vv[i][0] = v4.x; vv[i][1] = v4.y; vv[i][2] = v4.z; vv[i][3] = v4.w;
                    } else {
                        const float2 v2 = *reinterpret_cast<const float2*>(cur + (j + i) * kAttRS);
                        vv[i][0] = v2.x; vv[i][1] = v2.y;
                    }
                }
                // keys j..j+3 in order per output; PC*QPT independent chains per key
                #pragma unroll
                for (int i = 0; i < 4; ++i)
                    #pragma unroll
                    for (int a = 0; a < QPT; ++a) {
                        const float pa = i == 0 ? pv[a].x : i == 1 ? pv[a].y : i == 2 ? pv[a].z : pv[a].w;
                        #pragma unroll
                        for (int c = 0; c < PC; ++c) o[a][c] = __fmaf_rn(pa, vv[i][c], o[a][c]);
                    }
            }
            for (; j < kn; ++j) {       // ragged tail: exactly seq_k keys enter each chain
                float vv[PC];
                #pragma unroll
                for (int c = 0; c < PC; ++c) vv[c] = cur[j * kAttRS + c];
                #pragma unroll
                for (int a = 0; a < QPT; ++a) {
                    const float pa = prow[a * ss + j];
                    #pragma unroll
                    for (int c = 0; c < PC; ++c) o[a][c] = __fmaf_rn(pa, vv[c], o[a][c]);
                }
            }
        }
        if (!kv_all) __syncthreads();
    }
    if (pv_on) {
        #pragma unroll
        for (int a = 0; a < QPT; ++a) {
            const int q = q0 + pr0 + a;
            if (q < seq_q) {
                float* dst = O + (long long)q * ldo + (long long)h * kAttD + pd0;
                #pragma unroll
                for (int c = 0; c < PC; c += 2) *reinterpret_cast<float2*>(dst + c) = make_float2(o[a][c], o[a][c + 1]);
            }
        }
    }
    if (qz.q) att_fused_quant<QPT>(O, ldo, q0, seq_q, n_q * kAttD, qz);
}

template <int QPT>
cudaError_t launch_attention_tiled(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                                   long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                                   float scale, const float* mask, const AttBatch& bs, cudaStream_t st,
                                   const AttQuant& qz = AttQuant{}) {
    dim3 grid((seq_q + 8 * QPT - 1) / (8 * QPT), n_q, bs.n);
    // K / V resident for short query tiles (8-16 rows) when the grid is one
    // CTA per SM at most (the larger footprint costs no co-residency then)
    static const int sms = [] {
        int d = 0, n = 0;
        cudaGetDevice(&d);
        return cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) == cudaSuccess ? n : 0;
    }();
    const long long ctas = (long long)grid.x * grid.y * grid.z;
    const int kv_all = QPT <= 2 && seq_k > kAttTK && ctas <= sms &&
                       att_tiled_smem_all(8 * QPT, seq_k) <= 227 * 1024 ? 1 : 0;
    const size_t smem = kv_all ? att_tiled_smem_all(8 * QPT, seq_k) : att_tiled_smem(8 * QPT, seq_k);
    static int configured = 0;
    if ((int)smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(attention_tiled_kernel<QPT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured = (int)smem;
    }
    const cudaError_t e = launch_k(attention_tiled_kernel<QPT>, grid, 256, smem, st, Q, ldq, K, ldk, V, ldv, O, ldo,
                                   seq_q, seq_k, n_q, n_kv, scale, mask, bs, qz, kv_all);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

template <int QT, int NT>
cudaError_t launch_attention(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                             long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                             float scale, const float* mask, const AttBatch& bs, size_t smem, cudaStream_t st) {
    static int configured = 0;
    if ((int)smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(attention_kernel<QT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
        configured = (int)smem;
    }
    dim3 grid((seq_q + QT - 1) / QT, n_q, bs.n);
    {
        const cudaError_t le_ = launch_k(attention_kernel<QT, NT>, grid, NT, smem, st,
                                         Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv,
                                                          scale, mask, bs);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

cudaError_t attention(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                      float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, int head_dim, float scale,
                      const float* mask, cudaStream_t st, const AttQuant* qz) {
    return attention_batched(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, head_dim, scale, mask,
                             AttBatch{}, st, qz);
}

// The exact kernels: the register-tiled one where its score rows fit (it
// fuses the row quantization when qz.q is set: *fused), else the one-pass
// kernel; the tensor-core kernel when VLA_ATT_TC=1.
static cudaError_t attention_select(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                                    long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                                    int head_dim, float scale, const float* mask, const AttBatch& bs, cudaStream_t st,
                                    const AttQuant& qz, bool* fused);

cudaError_t attention_batched(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                              long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                              int head_dim, float scale, const float* mask, const AttBatch& bs, cudaStream_t st,
                              const AttQuant* qz) {
    const bool quant = qz && qz->q;
    if (quant && (!qz->scale || qz->ldq < (long long)n_q * head_dim || (qz->ldq & 3) ||
                  (reinterpret_cast<uintptr_t>(qz->q) & 3) || (qz->zq & 3)))
        return cudaErrorInvalidValue;
    // fusable: rows of at most 1024 columns and a counter per query tile
    const bool fusable = quant && qz->counters && (long long)n_q * head_dim <= 1024 &&
                         (long long)((seq_q + 7) / 8) * bs.n <= qz->n_counters;
    bool fused = false;
    cudaError_t e = attention_select(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, head_dim, scale, mask,
                                     bs, st, fusable ? *qz : AttQuant{}, &fused);
    if (e != cudaSuccess || !quant || fused) return e;
    for (int z = 0; z < bs.n && e == cudaSuccess; ++z)
        e = quantize_rows(O + z * bs.o, ldo, nullptr, 0, seq_q, n_q * head_dim, qz->q + z * qz->zq, qz->ldq,
                          qz->scale + z * qz->zs, nullptr, 0, nullptr, st);
    return e;
}

static cudaError_t attention_select(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                                    long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                                    int head_dim, float scale, const float* mask, const AttBatch& bs, cudaStream_t st,
                                    const AttQuant& qz, bool* fused) {
    *fused = false;
    if (head_dim != kAttD || seq_q <= 0 || seq_k <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv || bs.n < 1 ||
        bs.n > 65535)
        return cudaErrorInvalidValue;
    if (((bs.q | bs.k | bs.v | bs.o) & 3) != 0) return cudaErrorInvalidValue;
    // 16-byte vector loads of Q/K/V/O rows
    if (((ldq | ldk | ldv | ldo) & 3) ||
        ((reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) | reinterpret_cast<uintptr_t>(V) |
          reinterpret_cast<uintptr_t>(O)) & 15))
        return cudaErrorInvalidValue;
    if (attention_tc_enabled())
        return attention_tc(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, st);
    const size_t ss = (size_t)att_row_stride(seq_k);
    auto need = [&](int qt) { return sizeof(float) * (qt * ss + (size_t)kAttD * qt + (size_t)kAttKT * kAttD); };
    // Register-tiled kernel: the query tile (8, 16 or 40 rows) that gives the
    // busiest SM the least work (ceil(CTAs / SMs) x rows x the tile's cost per
    // row). 602 queries x 8 heads: 40 rows, 128 CTAs in one wave; the
    // decoder's 100 queries: 8 rows, 104 CTAs; Octo's 690 x 12 heads: 40 rows.
    if (att_tiled_smem(8, seq_k) <= 227 * 1024) {
        int best_qpt = 0;
        long long best_rows = 0;
        static const int forced = [] {
            const char* e = std::getenv("VLA_ATT_QPT");   // tuning knob: 1, 2, 4 or 5 query rows per warp
            const int v = e ? std::atoi(e) : 0;
            return v == 1 || v == 2 || v == 4 || v == 5 ? v : 0;
        }();
        const bool fits40 = att_tiled_smem(40, seq_k) <= 227 * 1024;
        for (int qpt : {5, 4, 2, 1}) {
            if (att_tiled_smem(8 * qpt, seq_k) > 227 * 1024) continue;
            if (forced && qpt != forced) continue;
            // 32-row tiles only where 40 rows of scores do not fit (SigLIP's
            // 1024 keys: 367 vs 465 us on 16-row tiles); where both fit, the
            // 40-row tile measured faster (Octo's 690 keys: 3.01 vs 3.11 ms
            // per query), each CTA streaming all keys whatever its rows
            if (qpt == 4 && fits40 && !forced) continue;
            const long long ctas = (long long)((seq_q + 8 * qpt - 1) / (8 * qpt)) * n_q * bs.n;
            // rows on the busiest SM, weighted by the cost of a row at each
            // tile height (taller tiles reuse every loaded K / V value more:
            // 1.0 / 1.3 / 1.4 per row measured for 40 / 16 / 8 rows on Octo
            // shapes; 32 rows between, by the shared-memory load count per fma)
            const int w = qpt == 5 ? 10 : qpt == 4 ? 11 : qpt == 2 ? 13 : 14;
            const long long rows = (ctas + 147) / 148 * 8 * qpt * w;
            if (!best_qpt || rows < best_rows) { best_qpt = qpt; best_rows = rows; }
        }
        // The fused quantization runs on one CTA per query tile after the
        // tile's heads finish: measured against a separate quantize_rows
        // launch in a graph, it saves 0.5-2 us at 8-16 rows per tile (the
        // SmolVLA expert, ACT's decoder) and costs 1.3 us at 40 (ACT's
        // encoder), where the separate launch spreads the rows over more SMs.
        *fused = qz.q != nullptr && best_qpt <= 2;
        const AttQuant none;
        if (best_qpt == 5)
            return launch_attention_tiled<5>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, st, none);
        if (best_qpt == 4)
            return launch_attention_tiled<4>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, st, none);
        if (best_qpt == 2)
            return launch_attention_tiled<2>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, st, qz);
        return launch_attention_tiled<1>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, st, qz);
    }
    // Longer key ranges (> ~1100 keys): score rows of fewer queries per CTA.
    // 16 queries x 128 threads per CTA: measured fastest among 8..32 queries x
    // 64..512 threads at the ACT encoder shape (more work per thread beats
    // more warps). Fewer queries (the decoder's 100) would leave most SMs idle
    // with 16 per CTA: narrower query tiles until the grid covers the SMs.
    const long long ctas16 = (long long)((seq_q + 15) / 16) * n_q;
    const long long ctas8 = (long long)((seq_q + 7) / 8) * n_q;
    if (ctas16 >= 148 && need(16) <= 200 * 1024)
        return launch_attention<16, 128>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, need(16), st);
    if (ctas8 >= 148 && need(8) <= 220 * 1024)
        return launch_attention<8, 64>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, need(8), st);
    if (need(4) <= 220 * 1024)
        return launch_attention<4, 64>(Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, need(4), st);
    return cudaErrorInvalidValue;   // > ~13000 keys: not a shape any policy here has
}

// --------------------------------------------------------- max-pool + ReLU
// src/hal/common/conv.cpp:192-225: max over the in-image taps, then the folded
// ReLU `!(o > 0) -> 0`. F frames of NHWC. Optional per-frame absmax tap for the
// next conv's per-tensor quantization.
__global__ void maxpool_relu_kernel(const float* __restrict__ x, float* __restrict__ out, int F, int H, int W, int C,
                                    int k, int stride, int pad, int Ho, int Wo, int vw, unsigned int* __restrict__ amax) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    // blockIdx.y = frame, so a block's absmax goes to one slot: reduce in the
    // block, then one atomic per block. Thread = vw (4 or 1) channels of one
    // output pixel (4: C % 4 == 0 and 16-byte aligned tensors); 32-bit index
    // math.
    const int f = blockIdx.y;
    const int cg = C / vw;
    const int per_frame = Ho * Wo * cg;
    const float* xf = x + (long long)f * H * W * C;
    float* of = out + (long long)f * Ho * Wo * C;
    float bmax = 0.0f;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < per_frame; r += gridDim.x * blockDim.x) {
        const int pix = r / cg;
        const int c = (r - pix * cg) * vw;
        const int oy = pix / Wo, ox = pix - oy * Wo;
        float o[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (k == 3 && vw == 4) {
            // the ACT stem pool: all 9 taps' loads issued before the maxima
            // (out-of-image taps predicated off and kept at -inf)
            float4 t[9];
            #pragma unroll
            for (int ky = 0; ky < 3; ++ky)
                #pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
                    const bool in = iy >= 0 && iy < H && ix >= 0 && ix < W;
                    t[ky * 3 + kx] = in ? *reinterpret_cast<const float4*>(xf + (iy * W + ix) * C + c)
                                        : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                }
            #pragma unroll
            for (int i = 0; i < 9; ++i) {     // taps in the reference's (ky, kx) order
                o[0] = t[i].x > o[0] ? t[i].x : o[0];
                o[1] = t[i].y > o[1] ? t[i].y : o[1];
                o[2] = t[i].z > o[2] ? t[i].z : o[2];
                o[3] = t[i].w > o[3] ? t[i].w : o[3];
            }
        } else {
            for (int ky = 0; ky < k; ++ky) {
                const int iy = oy * stride - pad + ky;
                if (iy < 0 || iy >= H) continue;
                for (int kx = 0; kx < k; ++kx) {
                    const int ix = ox * stride - pad + kx;
                    if (ix < 0 || ix >= W) continue;
                    const float* src = xf + (iy * W + ix) * C + c;
                    if (vw == 4) {
                        const float4 v = *reinterpret_cast<const float4*>(src);
                        o[0] = v.x > o[0] ? v.x : o[0];
                        o[1] = v.y > o[1] ? v.y : o[1];
                        o[2] = v.z > o[2] ? v.z : o[2];
                        o[3] = v.w > o[3] ? v.w : o[3];
                    } else {
                        const float v = *src;
                        o[0] = v > o[0] ? v : o[0];
                    }
                }
            }
        }
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            if (!(o[e] > 0.0f)) o[e] = 0.0f;
            bmax = fmaxf(bmax, o[e]);
        }
        float* dst = of + pix * C + c;
        if (vw == 4) *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        else *dst = o[0];
    }
    if (amax) {
        bmax = warp_max_f(bmax);
        __shared__ float wm[32];
        if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = bmax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = 0.0f;
            for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, wm[i]);
            atomicMax(&amax[f], __float_as_uint(m));
        }
    }
}

cudaError_t maxpool_relu(const float* x, float* out, int F, int H, int W, int C, int k, int stride, int pad,
                         int Ho, int Wo, unsigned int* amax, cudaStream_t st) {
    if (F <= 0 || Ho <= 0 || Wo <= 0 || C <= 0 || (long long)H * W * C >= (1LL << 31) ||
        (long long)Ho * Wo * C >= (1LL << 31))
        return cudaErrorInvalidValue;
    const bool vec = C % 4 == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    const long long per_frame = (long long)Ho * Wo * (vec ? C / 4 : C);
    long long bx = (per_frame + 255) / 256;
    if (bx > 148 * 8) bx = 148 * 8;
    {
        const cudaError_t le_ = launch_k(maxpool_relu_kernel, dim3((unsigned)bx, (unsigned)F), 256, 0, st,
                                         x, out, F, H, W, C, k, stride, pad, Ho, Wo, vec ? 4 : 1, amax);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// --------------------------------------------------- camera frame normalize
// uint8 HWC -> (p/255 - mean[c]) / (std[c] + eps), per camera f
// (src/models/act/act_model.cpp:116-121). mean/std are [F][3]. Per-frame absmax tap.
__global__ void normalize_frames_kernel(const uint8_t* __restrict__ img, float* __restrict__ out, int F, int npx,
                                        const float* __restrict__ mean, const float* __restrict__ stdv, float eps,
                                        unsigned int* __restrict__ amax) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    // thread = one pixel of frame blockIdx.y (its 3 interleaved channels)
    const int f = blockIdx.y;
    const uint8_t* src = img + (long long)f * npx * 3;
    float* dst = out + (long long)f * npx * 3;
    float mu[3], den[3];
    #pragma unroll
    for (int c = 0; c < 3; ++c) {
        mu[c] = mean[f * 3 + c];
        den[c] = __fadd_rn(stdv[f * 3 + c], eps);
    }
    float bmax = 0.0f;
    for (int px = blockIdx.x * blockDim.x + threadIdx.x; px < npx; px += gridDim.x * blockDim.x) {
        #pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float p = __fdiv_rn(i2f_small(src[3 * px + c]), 255.0f);
            const float v = __fdiv_rn(__fsub_rn(p, mu[c]), den[c]);
            dst[3 * px + c] = v;
            bmax = fmaxf(bmax, fabsf(v));
        }
    }
    if (amax) {
        bmax = warp_max_f(bmax);
        __shared__ float wm[32];
        if ((threadIdx.x & 31) == 0) wm[threadIdx.x >> 5] = bmax;
        __syncthreads();
        if (threadIdx.x == 0) {
            float m = 0.0f;
            for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, wm[i]);
            atomicMax(&amax[f], __float_as_uint(m));
        }
    }
}

cudaError_t normalize_frames(const uint8_t* img, float* out, int F, long long npx, const float* mean,
                             const float* stdv, float eps, unsigned int* amax, cudaStream_t st) {
    if (npx <= 0 || F <= 0 || npx * 3 >= (1LL << 31)) return cudaErrorInvalidValue;
    long long bx = (npx + 255) / 256;
    if (bx > 148 * 8) bx = 148 * 8;
    {
        const cudaError_t le_ = launch_k(normalize_frames_kernel, dim3((unsigned)bx, (unsigned)F), 256, 0, st,
                                         img, out, F, (int)npx, mean, stdv, eps, amax);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// ------------------------------------------------------ small fp32 linears
// The reference's fp32 dense_linear (src/hal/avx2/gemm.cpp:98-122), reproduced
// per output: outputs in a whole block of 4 take mm_block4's order (two 8-lane
// accumulators over 16-wide k steps, an 8-wide step into the first, hsum8 of
// their sum, scalar fma tail; :33-86), the rest simd_dot's (four 8-lane chains
// over 32-wide steps; simd.h:12-40); then + bias. One thread per output - these
// are ACT's K=6 state projection and N=6 action head, where exact replication
// costs nothing. Optional post affine (action unnormalization):
// out = fma(out, post_mul[n], post_add[n]).
__device__ __forceinline__ float hsum8_ref(const float (&a)[8]) {
    return __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[4]), __fadd_rn(a[1], a[5])),
                     __fadd_rn(__fadd_rn(a[2], a[6]), __fadd_rn(a[3], a[7])));
}

__global__ void linear_f32_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ W,
                                  const float* __restrict__ bias, float* __restrict__ out, long long ldo,
                                  int M, int N, int K, const float* __restrict__ post_mul,
                                  const float* __restrict__ post_add) {
    // one warp per output; the reference's independent lane accumulators are
    // spread over the warp's lanes, then combined in its order
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const long long w = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
    if (w >= (long long)M * N) return;
    const int m = static_cast<int>(w / N), n = static_cast<int>(w - (long long)m * N);
    const float* xr = x + (long long)m * ldx;
    const float* wr = W + (long long)n * K;
    const bool block4 = n < N - N % 4;
    float acc = 0.0f;
    int kend;
    if (block4) {
        // lanes 0-7: a[l] (k % 16 == l), lanes 8-15: b[l-8] (k % 16 == l); 16-wide steps
        const int K16 = K & ~15;
        if (lane < 16) {
            // 8 steps' operands are loaded before their fmas: the chain waits
            // on one round of load latency per 8 steps, not per step
            int k = 0;
            for (; k + 128 <= K16; k += 128) {
                float xv[8], wv[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) { xv[u] = xr[k + 16 * u + lane]; wv[u] = wr[k + 16 * u + lane]; }
                #pragma unroll
                for (int u = 0; u < 8; ++u) acc = __fmaf_rn(xv[u], wv[u], acc);
            }
            for (; k < K16; k += 16) acc = __fmaf_rn(xr[k + lane], wr[k + lane], acc);
        }
        kend = K16;
        if (K - K16 >= 8) {                      // one 8-wide step into a
            if (lane < 8) acc = __fmaf_rn(xr[K16 + lane], wr[K16 + lane], acc);
            kend = K16 + 8;
        }
        // t[l] = a[l] + b[l]
        const float other = __shfl_down_sync(0xFFFFFFFFu, acc, 8);
        acc = __fadd_rn(acc, other);
    } else {
        // lanes 8j+l: chain j of lane l, 32-wide steps; then 8-wide steps into chain 0
        const int K32 = K & ~31;
        int k = 0;
        for (; k + 256 <= K32; k += 256) {
            float xv[8], wv[8];
            #pragma unroll
            for (int u = 0; u < 8; ++u) { xv[u] = xr[k + 32 * u + lane]; wv[u] = wr[k + 32 * u + lane]; }
            #pragma unroll
            for (int u = 0; u < 8; ++u) acc = __fmaf_rn(xv[u], wv[u], acc);
        }
        for (; k < K32; k += 32) acc = __fmaf_rn(xr[k + lane], wr[k + lane], acc);
        kend = K32;
        for (; kend + 8 <= K; kend += 8)
            if (lane < 8) acc = __fmaf_rn(xr[kend + lane], wr[kend + lane], acc);
        // c0[l] = (acc0[l] + acc1[l]) + (acc2[l] + acc3[l])
        const float a1 = __shfl_down_sync(0xFFFFFFFFu, acc, 8);
        const float a2 = __shfl_down_sync(0xFFFFFFFFu, acc, 16);
        const float a3 = __shfl_down_sync(0xFFFFFFFFu, acc, 24);
        acc = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
    }
    // hsum8 over lanes 0..7: ((l0+l4)+(l1+l5)) + ((l2+l6)+(l3+l7))
    float l[8];
    #pragma unroll
    for (int i = 0; i < 8; ++i) l[i] = __shfl_sync(0xFFFFFFFFu, acc, i);
    if (lane == 0) {
        float s = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                            __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
        // scalar tails: mm_block4's is contracted to fma by the reference's
        // -ffp-contract=fast build, simd_dot's stays a rounded multiply then add
        // (both established against the compiled reference on odd K)
        if (block4)
            for (int k = kend; k < K; ++k) s = __fmaf_rn(xr[k], wr[k], s);
        else
            for (int k = kend; k < K; ++k) s = __fadd_rn(s, __fmul_rn(xr[k], wr[k]));
        float v = bias ? __fadd_rn(s, bias[n]) : s;
        if (post_mul) v = __fmaf_rn(v, post_mul[n], post_add[n]);
        out[(long long)m * ldo + n] = v;
    }
}

// The same outputs for many rows (N % 4 == 0: every output takes mm_block4's
// order). CTA = 32 rows x 32 outputs; K streams through shared memory in
// chunks of up to kLtK (both operand chunks staged whole); a thread owns a
// 2 x 2 block of outputs and runs, per output, the 16 lane chains (a[l] over
// k = 16s + l, b[l] over 16s + 8 + l) across the chunks in k order, then the
// 8-wide step into a, t = a + b, hsum8, the fused scalar tail and + bias in
// registers: bit for bit the warp kernel's arithmetic, with each staged value
// feeding two outputs.
constexpr int kLtRows = 32;
constexpr int kLtK = 512;

__global__ void __launch_bounds__(256)
linear_f32_tiled_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ W,
                        const float* __restrict__ bias, float* __restrict__ out, long long ldo, int M, int N, int K,
                        const float* __restrict__ post_mul, const float* __restrict__ post_add) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    extern __shared__ __align__(16) float lt_smem[];
    const int kc_max = K < kLtK ? K : kLtK;
    const int ldk = ((kc_max + 3) & ~3) + 4;       // 16-byte rows, rows 4 banks apart
    float* sx = lt_smem;
    float* sw = lt_smem + kLtRows * ldk;
    const int m0 = blockIdx.y * kLtRows, n0 = blockIdx.x * kLtRows;
    const int tm = threadIdx.x >> 4, tn = threadIdx.x & 15;
    const float* xr[2] = {sx + tm * ldk, sx + (tm + 16) * ldk};
    const float* wr[2] = {sw + tn * ldk, sw + (tn + 16) * ldk};
    float acc[2][2][16];
    #pragma unroll
    for (int i = 0; i < 2; ++i)
        #pragma unroll
        for (int j = 0; j < 2; ++j)
            #pragma unroll
            for (int l = 0; l < 16; ++l) acc[i][j][l] = 0.0f;
    const int K16 = K & ~15;
    const bool vec = ((K | ldx) & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W)) & 15) == 0;
    int kc0 = 0;
    for (;;) {
        const int kcl = K - kc0 < kLtK ? K - kc0 : kLtK;    // kLtK is a multiple of 16: chunks keep the 16-steps whole
        if (vec) {                     // 16-byte loads, four rounds in flight per thread
            const int c4 = kcl >> 2;
            #pragma unroll 4
            for (int e = threadIdx.x; e < kLtRows * c4; e += blockDim.x) {
                const int r = e / c4, c = 4 * (e - r * c4);
                const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                const float4 xv = m0 + r < M ? *reinterpret_cast<const float4*>(x + (long long)(m0 + r) * ldx + kc0 + c) : z;
                const float4 wv = n0 + r < N ? *reinterpret_cast<const float4*>(W + (long long)(n0 + r) * K + kc0 + c) : z;
                *reinterpret_cast<float4*>(sx + r * ldk + c) = xv;
                *reinterpret_cast<float4*>(sw + r * ldk + c) = wv;
            }
        } else {
            #pragma unroll 4
            for (int e = threadIdx.x; e < kLtRows * kcl; e += blockDim.x) {
                const int r = e / kcl, c = e - r * kcl;
                sx[r * ldk + c] = m0 + r < M ? x[(long long)(m0 + r) * ldx + kc0 + c] : 0.0f;
                sw[r * ldk + c] = n0 + r < N ? W[(long long)(n0 + r) * K + kc0 + c] : 0.0f;
            }
        }
        __syncthreads();
        const int kend16 = (kc0 + kcl < K16 ? kc0 + kcl : K16) - kc0;
        for (int k = 0; k < kend16; k += 16) {
            #pragma unroll
            for (int q = 0; q < 4; ++q) {              // lanes 4q .. 4q+3 of the 16
                const float4 x0 = *reinterpret_cast<const float4*>(xr[0] + k + 4 * q);
                const float4 x1 = *reinterpret_cast<const float4*>(xr[1] + k + 4 * q);
                const float4 w0 = *reinterpret_cast<const float4*>(wr[0] + k + 4 * q);
                const float4 w1 = *reinterpret_cast<const float4*>(wr[1] + k + 4 * q);
                const float xv[2][4] = {{x0.x, x0.y, x0.z, x0.w}, {x1.x, x1.y, x1.z, x1.w}};
                const float wv[2][4] = {{w0.x, w0.y, w0.z, w0.w}, {w1.x, w1.y, w1.z, w1.w}};
                #pragma unroll
                for (int i = 0; i < 2; ++i)
                    #pragma unroll
                    for (int j = 0; j < 2; ++j)
                        #pragma unroll
                        for (int u = 0; u < 4; ++u)
                            acc[i][j][4 * q + u] = __fmaf_rn(xv[i][u], wv[j][u], acc[i][j][4 * q + u]);
            }
        }
        if (kc0 + kcl >= K) break;     // the last chunk (it holds k >= K16) stays staged
        kc0 += kcl;
        __syncthreads();               // every thread is done with this chunk
    }
    const int t16 = K16 - kc0;         // offset of K16 in the staged last chunk
    int kend = t16;
    if (K - K16 >= 8) {                  // one 8-wide step into a
        #pragma unroll
        for (int i = 0; i < 2; ++i)
            #pragma unroll
            for (int j = 0; j < 2; ++j)
                #pragma unroll
                for (int l = 0; l < 8; ++l)
                    acc[i][j][l] = __fmaf_rn(xr[i][t16 + l], wr[j][t16 + l], acc[i][j][l]);
        kend = t16 + 8;
    }
    #pragma unroll
    for (int i = 0; i < 2; ++i) {
        #pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int m = m0 + tm + 16 * i, n = n0 + tn + 16 * j;
            float t[8];
            #pragma unroll
            for (int l = 0; l < 8; ++l) t[l] = __fadd_rn(acc[i][j][l], acc[i][j][8 + l]);
            float sum = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[4]), __fadd_rn(t[1], t[5])),
                                  __fadd_rn(__fadd_rn(t[2], t[6]), __fadd_rn(t[3], t[7])));
            for (int k = kend; k < K - kc0; ++k) sum = __fmaf_rn(xr[i][k], wr[j][k], sum);
            if (m < M && n < N) {
                float v = bias ? __fadd_rn(sum, bias[n]) : sum;
                if (post_mul) v = __fmaf_rn(v, post_mul[n], post_add[n]);
                out[(long long)m * ldo + n] = v;
            }
        }
    }
}

cudaError_t linear_f32(const float* x, long long ldx, const float* W, const float* bias, float* out, long long ldo,
                       int M, int N, int K, const float* post_mul, const float* post_add, cudaStream_t st) {
    if (M <= 0 || N <= 0 || K <= 0) return cudaErrorInvalidValue;
    if (N % 4 == 0 && M >= kLtRows && (long long)M * N >= (1LL << 16)) {
        const int kc = K < kLtK ? K : kLtK;
        const size_t smem = sizeof(float) * 2 * kLtRows * (((kc + 3) & ~3) + 4);
        static bool attr = false;
        if (!attr) {
            cudaFuncSetAttribute(linear_f32_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            attr = true;
        }
        const dim3 grid((unsigned)((N + kLtRows - 1) / kLtRows), (unsigned)((M + kLtRows - 1) / kLtRows));
        const cudaError_t le_ = launch_k(linear_f32_tiled_kernel, grid, 256, smem, st, x, ldx, W, bias, out, ldo, M,
                                         N, K, post_mul, post_add);
        if (le_ != cudaSuccess) return le_;
        return cudaGetLastError();
    }
    const long long threads = (long long)M * N * 32;
    {
        const cudaError_t le_ = launch_k(linear_f32_kernel, (int)((threads + 255) / 256), 256, 0, st,
                                         x, ldx, W, bias, out, ldo, M, N, K, post_mul, post_add);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

// First kernel of an ACT step: zero the per-frame absmax slots and the decoder
// queries, place the latent token, and normalize the state,
// (state - mean) / (std + eps) as ActModel::predict (src/models/act/act_model.cpp:151-153).
// Doing this in a kernel keeps the captured step a single chain of kernels.
__global__ void act_prologue_kernel(unsigned int* __restrict__ zero_u32, int n_zero_u32, float* __restrict__ zero_f32,
                                    long long n_zero_f32, const float* __restrict__ init_f32,
                                    float* __restrict__ tok0, const float* __restrict__ latent,
                                    int d, const float* __restrict__ state, const float* __restrict__ mean,
                                    const float* __restrict__ stdv, float eps, float* __restrict__ state_n, int n) {
    pdl_wait();     // the previous step may still read these buffers
    pdl_trigger();
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = tid; i < n_zero_u32; i += stride) zero_u32[i] = 0u;
    for (long long i = tid; i < n_zero_f32; i += stride) zero_f32[i] = init_f32 ? init_f32[i] : 0.0f;
    for (long long i = tid; i < d; i += stride) tok0[i] = latent[i];
    for (long long i = tid; i < n; i += stride)
        state_n[i] = __fdiv_rn(__fsub_rn(state[i], mean[i]), __fadd_rn(stdv[i], eps));
}

cudaError_t act_prologue(unsigned int* zero_u32, int n_zero_u32, float* zero_f32, long long n_zero_f32,
                         const float* init_f32, float* tok0, const float* latent, int d, const float* state,
                         const float* mean, const float* stdv, float eps, float* state_n, int n, cudaStream_t st) {
    const cudaError_t le_ = launch_k(act_prologue_kernel, 64, 256, 0, st, zero_u32, n_zero_u32, zero_f32, n_zero_f32,
                                     init_f32, tok0, latent, d, state, mean, stdv, eps, state_n, n);
    if (le_ != cudaSuccess) return le_;
    return cudaGetLastError();
}

// out = a + b, elementwise (fp32 inputs of fp32-path q/k projections)
__global__ void add_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                               long long n) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

cudaError_t add_f32(const float* a, const float* b, float* out, long long n, cudaStream_t st) {
    if (n <= 0) return cudaErrorInvalidValue;
    long long blocks = (n + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    {
        const cudaError_t le_ = launch_k(add_f32_kernel, (int)blocks, 256, 0, st,
                                         a, b, out, n);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

}  // namespace vsb
