// Diffusion Policy kernels: observation preprocessing, GroupNorm over batched
// samples with fused Mish / FiLM / residual / ReLU epilogues, the 1D im2col of
// the conditional U-Net fused with its per-row int8 quantization, the cond
// encoder input, and the DDIM / DDPM reverse step. Compiled into kernels.cu
// after nn.cu and lm_ops.cu (ref_exp, nn_row_scale, nn_q8, warp_max_f).
//
// Arithmetic follows the reference build (-mavx2 -mfma -ffp-contract=fast):
// the contractions below (fma in GroupNorm's apply, FiLM, the scheduler step
// and the action unnormalization) are the ones its compiler emitted.
#include "sm100.cuh"
#include "launch.cuh"
#include "dp.h"
#include "libm_f32.h"   // glibc's float expf / log1pf / expm1f / tanhf, restated

namespace vsb {

namespace {

// Mish as the reference's 8-lane body (src/hal/common/eltwise.cpp:224-243):
// v * m / (m + 2), m = e(e + 2), e = exp(min(v, 20)) with its Cephes exp.
__device__ __forceinline__ float mish_lanes(float v) {
    const float e = ref_exp(fminf(v, 20.0f));
    const float m = __fmul_rn(e, __fadd_rn(e, 2.0f));
    return __fmul_rn(v, __fdiv_rn(m, __fadd_rn(m, 2.0f)));
}

// the host library's expf (libm_f32.h: bit-identical to it on all 2^32 inputs)
__device__ __forceinline__ float libm_expf(float x) { return lf_expf(x); }

__device__ __forceinline__ float block_max_256(float v, float* sh) {
    v = warp_max_f(v);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float m = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0f;
        m = warp_max_f(m);
        if (threadIdx.x == 0) sh[0] = m;
    }
    __syncthreads();
    const float r = sh[0];
    __syncthreads();
    return r;
}

__device__ __forceinline__ double block_sum_d(double v, double* sh) {
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, off));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        double s = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) s = __dadd_rn(s, __shfl_xor_sync(0xFFFFFFFFu, s, off));
        if (threadIdx.x == 0) sh[0] = s;
    }
    __syncthreads();
    const double r = sh[0];
    __syncthreads();
    return r;
}

long long grid_cap(long long n, int threads, long long cap) {
    long long b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    return b > cap ? cap : b;
}

}  // namespace

// ------------------------------------------------------------ preprocessing
__global__ void dp_preprocess_kernel(const uint8_t* __restrict__ frames, int B, int S, int N, int H, int W, int top,
                                     int left, int oh, int ow, const float* __restrict__ mean,
                                     const float* __restrict__ stdv, float eps, float* __restrict__ out,
                                     unsigned int* __restrict__ amax, int Fr, long long run_stride) {
    pdl_wait();     // the previous step may still read these buffers
    pdl_trigger();
    const int i = blockIdx.y;            // input frame (b, s, c)
    const int c = i % N, bs = i / N;
    const int o = c * (B * S) + bs;      // camera-major output frame
    const uint8_t* src = frames + (long long)i * H * W * 3;
    float* dst = out + (long long)o * oh * ow * 3;
    float mu[3], den[3];
    #pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        mu[ch] = mean[c * 3 + ch];
        den[ch] = __fadd_rn(stdv[c * 3 + ch], eps);
    }
    float bmax = 0.0f;
    const int npx = oh * ow;
    for (int px = blockIdx.x * blockDim.x + threadIdx.x; px < npx; px += gridDim.x * blockDim.x) {
        const int y = px / ow, x = px - y * ow;
        const uint8_t* s = src + ((long long)(y + top) * W + left + x) * 3;
        #pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            const float v = __fdiv_rn(__fsub_rn(__fdiv_rn(i2f_small(s[ch]), 255.0f), mu[ch]), den[ch]);
            dst[3 * px + ch] = v;
            bmax = fmaxf(bmax, fabsf(v));
        }
    }
    __shared__ float sh[32];
    bmax = block_max_256(bmax, sh);
    if (threadIdx.x == 0 && amax) atomicMax(&amax[(long long)(o / Fr) * run_stride + o % Fr], __float_as_uint(bmax));
}

cudaError_t dp_preprocess(const uint8_t* frames, int B, int S, int N, int H, int W, int top, int left, int oh, int ow,
                          const float* mean, const float* stdv, float eps, float* out, unsigned int* amax, int Fr,
                          long long run_stride, cudaStream_t st) {
    if (B <= 0 || S <= 0 || N <= 0 || oh <= 0 || ow <= 0 || top < 0 || left < 0 || top + oh > H || left + ow > W ||
        (long long)B * S * N > 65535 || Fr <= 0)
        return cudaErrorInvalidValue;
    const long long bx = grid_cap((long long)oh * ow, 256, 64);
    const cudaError_t e = launch_k(dp_preprocess_kernel, dim3((unsigned)bx, (unsigned)(B * S * N)), 256, 0, st, frames,
                                   B, S, N, H, W, top, left, oh, ow, mean, stdv, eps, out, amax, Fr, run_stride);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------------- GroupNorm
// Block = one (group, sample). Per channel: shift K = its first pixel, S1 =
// sum(x - K), S2 = sum((x - K)^2) in double over pixel slices, then the slices
// in order; per group: mean = sum(S1 + np*K)/n, ss = sum(S2 + 2dk*S1 +
// np*dk^2) (dk = K - mean) as block reductions, inv = 1/sqrt(ss/n + eps);
// A = inv*scale, B = bias - mean*inv*scale (the reference's formulas,
// src/hal/common/conv.cpp:236-301). The sums are regrouped for parallelism;
// in double that moves A and B by far less than a float ulp.
__global__ void __launch_bounds__(256)
gn_affine_kernel(const float* __restrict__ x, int npx, int C, long long ld, int groups, float eps,
                 const float* __restrict__ scale, const float* __restrict__ bias, float* __restrict__ A,
                 float* __restrict__ B) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    extern __shared__ double gsm[];
    __shared__ double red[32];
    const int g = blockIdx.x, f = blockIdx.y;
    const int gc = C / groups, c0 = g * gc;
    const int nsl = gc >= 256 ? 1 : 256 / gc;       // pixel slices per channel
    double* p1 = gsm;                                // [nsl][gc]
    double* p2 = gsm + (size_t)nsl * gc;
    const float* xf = x + (long long)f * npx * ld + c0;
    for (int it = threadIdx.x; it < gc * nsl; it += blockDim.x) {
        const int cl = it % gc, sl = it / gc;
        const double K = (double)xf[cl];
        double s1 = 0.0, s2 = 0.0;
        int p = sl;
        // eight pixels' loads in flight before their adds (the same order of
        // additions as one pixel at a time)
        for (; p + 7 * nsl < npx; p += 8 * nsl) {
            float v[8];
            #pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = xf[(long long)(p + u * nsl) * ld + cl];
            #pragma unroll
            for (int u = 0; u < 8; ++u) {
                const double d = __dsub_rn((double)v[u], K);
                s1 = __dadd_rn(s1, d);
                s2 = __fma_rn(d, d, s2);
            }
        }
        for (; p < npx; p += nsl) {
            const double d = __dsub_rn((double)xf[(long long)p * ld + cl], K);
            s1 = __dadd_rn(s1, d);
            s2 = __fma_rn(d, d, s2);
        }
        p1[it] = s1;
        p2[it] = s2;
    }
    __syncthreads();
    const double np = (double)npx, n = np * gc;
    double t1 = 0.0;
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        double s1 = p1[cl], s2 = p2[cl];
        for (int sl = 1; sl < nsl; ++sl) {
            s1 = __dadd_rn(s1, p1[sl * gc + cl]);
            s2 = __dadd_rn(s2, p2[sl * gc + cl]);
        }
        p1[cl] = s1;
        p2[cl] = s2;
        t1 = __dadd_rn(t1, __fma_rn(np, (double)xf[cl], s1));
    }
    const double mean = __ddiv_rn(block_sum_d(t1, red), n);
    double t2 = 0.0;
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        const double dk = __dsub_rn((double)xf[cl], mean);
        const double t = __fma_rn(__dmul_rn(2.0, dk), p1[cl], p2[cl]);
        t2 = __dadd_rn(t2, __fma_rn(__dmul_rn(np, dk), dk, t));
    }
    const double ss = block_sum_d(t2, red);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, n), (double)eps)));
    const double mi = __dmul_rn(mean, inv);
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        const int c = c0 + cl;
        A[(long long)f * C + c] = (float)__dmul_rn(inv, (double)scale[c]);
        B[(long long)f * C + c] = (float)__fma_rn(-mi, (double)scale[c], (double)bias[c]);
    }
}

cudaError_t gn_affine(const float* x, int F, int npx, int C, long long ld, int groups, float eps, const float* scale,
                      const float* bias, float* A, float* B, cudaStream_t st) {
    if (F <= 0 || npx <= 0 || C <= 0 || groups <= 0 || C % groups || ld < C || F > 65535) return cudaErrorInvalidValue;
    const int gc = C / groups;
    const int nsl = gc >= 256 ? 1 : 256 / gc;
    const size_t smem = (size_t)2 * nsl * gc * sizeof(double);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(gn_affine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    const cudaError_t e = launch_k(gn_affine_kernel, dim3((unsigned)groups, (unsigned)F), 256, smem, st, x, npx, C, ld,
                                   groups, eps, scale, bias, A, B);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void __launch_bounds__(256)
gn_apply_kernel(const float* __restrict__ x, const float* __restrict__ A, const float* __restrict__ B,
                float* __restrict__ out, int npx, int C, long long ld, int epi, const float* __restrict__ res,
                unsigned int* __restrict__ amax) {
    pdl_wait();     // A / B and x come from earlier kernels in the stream
    pdl_trigger();
    const int f = blockIdx.y;
    const long long base = (long long)f * npx * ld;
    const float* Af = A + (long long)f * C;
    const float* Bf = B + (long long)f * C;
    const long long total = (long long)npx * C;
    float bmax = 0.0f;
    for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
        const int p = static_cast<int>(e / C), c = static_cast<int>(e - (long long)p * C);
        const long long i = base + (long long)p * ld + c;
        float v = __fmaf_rn(x[i], Af[c], Bf[c]);
        if (epi & kGnMish) v = mish_lanes(v);
        if (epi & kGnAdd) {
            v = __fadd_rn(v, res[i]);
            if (epi & kGnRelu) v = v > 0.0f ? v : 0.0f;        // relu(c + identity), resnet block tail
        } else if (epi & kGnRelu) {
            v = v < 0.0f ? 0.0f : v;                           // groupnorm(..., fuse_relu)
        }
        out[i] = v;
        bmax = fmaxf(bmax, fabsf(v));
    }
    if (amax) {
        __shared__ float sh[32];
        bmax = block_max_256(bmax, sh);
        if (threadIdx.x == 0) atomicMax(&amax[f], __float_as_uint(bmax));
    }
}

cudaError_t gn_apply(const float* x, const float* A, const float* B, float* out, int F, int npx, int C, long long ld,
                     int epi, const float* res, unsigned int* amax, cudaStream_t st) {
    if (F <= 0 || npx <= 0 || C <= 0 || ld < C || F > 65535 || ((epi & kGnAdd) && !res)) return cudaErrorInvalidValue;
    const long long bx = grid_cap((long long)npx * C, 256, (148 * 8 + F - 1) / F);
    const cudaError_t e = launch_k(gn_apply_kernel, dim3((unsigned)bx, (unsigned)F), 256, 0, st, x, A, B, out, npx, C,
                                   ld, epi, res, amax);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------ 1D im2col
// fp32 im2col rows of F samples (fp32 U-Net layers): colf [F*Tout][k*C], row
// (f, ot) = the k input rows ot*stride - pad + kt (zero outside [0, T))
// (src/hal/common/conv.cpp:334-347).
__global__ void im2col1d_f32_kernel(const float* __restrict__ x, int T, int C, long long ldx, int k, int stride,
                                    int pad, int Tout, float* __restrict__ colf, long long total) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long K = (long long)k * C;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / K;
        const int e = static_cast<int>(i - r * K);
        const int f = static_cast<int>(r / Tout), ot = static_cast<int>(r - (long long)f * Tout);
        const int kt = e / C, c = e - kt * C;
        const int t = ot * stride - pad + kt;
        colf[i] = (t >= 0 && t < T) ? x[((long long)f * T + t) * ldx + c] : 0.0f;
    }
}

cudaError_t im2col1d_f32x(const float* x, int F, int T, int C, long long ldx, int k, int stride, int pad, int Tout,
                          float* colf, cudaStream_t st) {
    if (F <= 0 || T <= 0 || C <= 0 || ldx < C || k <= 0 || stride <= 0 || pad < 0 || Tout <= 0) return cudaErrorInvalidValue;
    const long long total = (long long)F * Tout * k * C;
    const cudaError_t e = launch_k(im2col1d_f32_kernel, (unsigned)grid_cap(total, 256, 148 * 8), 256, 0, st, x, T, C,
                                   ldx, k, stride, pad, Tout, colf, total);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------ conv_transpose1d
// Per output (sample, ot, co): bias, then x[t][ci] * W[ci][kt][co] for kt from
// k-1 down to 0, ci in order, zero inputs skipped (src/hal/common/conv.cpp:349-395).
// That order is kept: every output is one fma chain, advanced tap slot by tap
// slot (the j-th valid kt of the output, descending), and inside a slot over
// ci. CTA = CO output channels x all Tout time steps x SB samples; a thread
// owns ST samples x OTP time steps x 4 channels. Chains of one time step share
// their tap and input row, so per ci a thread loads one float4 of weights and
// ST x values and issues ST x 4 fmas per time step. ci advances in chunks of
// kCtCi whose W [kCtCi][k][CO] and x [SB][T][kCtCi] values stream through a
// cp.async ring of kCtStages chunks. Optional per-row absmax (atomicMax).
constexpr int kCtCi = 32, kCtMaxK = 4, kCtStages = 4, kCtThreads = 256;
constexpr int kCtXs = kCtCi + 4;   // x row stride in shared memory: 16-byte rows, distinct banks per row

__host__ __device__ constexpr size_t convt_stage_floats(int k, int xrows, int co) {
    return (size_t)kCtCi * k * co + (size_t)xrows * kCtXs;
}

template <int ST, int OTP, int CO>
__global__ void __launch_bounds__(kCtThreads)
conv_transpose1d_tiled_kernel(const float* __restrict__ x, const float* __restrict__ W,
                              const float* __restrict__ bias, float* __restrict__ out, int F, int T, int Cin,
                              int Cout, int k, int stride, int pad, int Tout, int SB, int slots,
                              unsigned int* __restrict__ rowmax) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    extern __shared__ __align__(16) float ct_smem[];
    constexpr int NQ = CO / 4;                     // 4-channel groups per CTA
    const int n_otg = Tout / OTP;                  // thread groups over time steps
    const int cq = threadIdx.x % NQ;
    const int otg = (threadIdx.x / NQ) % n_otg;
    const int sg = (threadIdx.x / NQ) / n_otg;     // sample group
    const int co0 = blockIdx.x * CO, f0 = blockIdx.y * SB;
    const int sb = min(SB, F - f0);
    const int co = co0 + 4 * cq;
    const int xrows = SB * T;
    const size_t stage_fl = convt_stage_floats(k, xrows, CO);
    const int nchunk = (Cin + kCtCi - 1) / kCtCi;
    const int iters = slots * nchunk;              // (slot, chunk) in chain order
    const bool thread_live = sg * ST < sb;
    float acc[OTP][ST][4];
    #pragma unroll
    for (int jo = 0; jo < OTP; ++jo)
        #pragma unroll
        for (int si = 0; si < ST; ++si)
            #pragma unroll
            for (int u = 0; u < 4; ++u) acc[jo][si][u] = (bias && co + u < Cout) ? bias[co + u] : 0.0f;
    auto issue = [&](int it, int stg) {
        const int c = it % nchunk;
        float* sW = ct_smem + (size_t)stg * stage_fl;
        float* sx = sW + (size_t)kCtCi * k * CO;
        const int ci0 = c * kCtCi;
        for (int e = threadIdx.x; e < kCtCi * k * NQ; e += blockDim.x) {
            const int q = e % NQ, r = e / NQ, kt = r % k, ci = ci0 + r / k;
            const bool ok = ci < Cin;
            cp_async16(sW + (size_t)r * CO + 4 * q, W + ((long long)(ok ? ci : 0) * k + kt) * Cout + co0 + 4 * q,
                       ok ? 16 : 0);
        }
        for (int e = threadIdx.x; e < xrows * (kCtCi / 4); e += blockDim.x) {
            const int row = e / (kCtCi / 4), q = e - row * (kCtCi / 4), ci = ci0 + 4 * q;
            const int s_ = row / T, t = row - s_ * T;
            const bool ok = ci < Cin && s_ < sb;
            cp_async16(sx + (size_t)row * kCtXs + 4 * q,
                       x + ((long long)(ok ? f0 + s_ : 0) * T + t) * Cin + (ok ? ci : 0), ok ? 16 : 0);
        }
    };
    for (int s0 = 0; s0 < kCtStages - 1; ++s0) {
        if (s0 < iters) issue(s0, s0);
        cp_async_commit();
    }
    int cur_slot = -1;
    int kt_i[OTP], t_i[OTP];
    for (int it = 0; it < iters; ++it) {
        const int j = it / nchunk, c = it - j * nchunk;
        if (j != cur_slot) {      // this slot's tap and input step per time step (-1: none)
            cur_slot = j;
            #pragma unroll
            for (int jo = 0; jo < OTP; ++jo) {
                const int ot = otg * OTP + jo;
                kt_i[jo] = -1;
                t_i[jo] = 0;
                int seen = 0;
                for (int kt = k - 1; kt >= 0; --kt) {
                    const int num = ot + pad - kt;
                    if (num < 0 || num % stride) continue;
                    const int t = num / stride;
                    if (t >= T) continue;
                    if (seen++ == j) { kt_i[jo] = kt; t_i[jo] = t; break; }
                }
            }
        }
        asm volatile("cp.async.wait_group %0;" :: "n"(kCtStages - 2) : "memory");
        __syncthreads();
        // refill the stage the previous iteration read (every thread is past it)
        if (it + kCtStages - 1 < iters) issue(it + kCtStages - 1, (it + kCtStages - 1) % kCtStages);
        cp_async_commit();
        if (!thread_live) continue;
        const float* sW = ct_smem + (size_t)(it % kCtStages) * stage_fl;
        const float* sx = sW + (size_t)kCtCi * k * CO;
        const int cmax = min(kCtCi, Cin - c * kCtCi);
        #pragma unroll
        for (int jo = 0; jo < OTP; ++jo) {
            if (kt_i[jo] < 0) continue;
            const float* wrow = sW + (size_t)kt_i[jo] * CO + 4 * cq;
            const float* xrow = sx + (size_t)(sg * ST * T + t_i[jo]) * kCtXs;
            for (int ci = 0; ci < cmax; ++ci) {
                const float4 w4 = *reinterpret_cast<const float4*>(wrow + (size_t)ci * k * CO);
                #pragma unroll
                for (int si = 0; si < ST; ++si) {
                    const float v = xrow[(size_t)si * T * kCtXs + ci];
                    if (v == 0.0f) continue;
                    acc[jo][si][0] = __fmaf_rn(v, w4.x, acc[jo][si][0]);
                    acc[jo][si][1] = __fmaf_rn(v, w4.y, acc[jo][si][1]);
                    acc[jo][si][2] = __fmaf_rn(v, w4.z, acc[jo][si][2]);
                    acc[jo][si][3] = __fmaf_rn(v, w4.w, acc[jo][si][3]);
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    #pragma unroll
    for (int jo = 0; jo < OTP; ++jo) {
        const int ot = otg * OTP + jo;
        #pragma unroll
        for (int si = 0; si < ST; ++si) {
            const int sl = sg * ST + si;
            const bool live = sl < sb;
            const long long orow = (long long)(f0 + sl) * Tout + ot;
            float m = 0.0f;
            if (live) {
                #pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (co + u < Cout) {
                        out[orow * Cout + co + u] = acc[jo][si][u];
                        m = fmaxf(m, fabsf(acc[jo][si][u]));
                    }
            }
            if (rowmax) {
                // the CO channels of this row sit in NQ consecutive lanes; every
                // lane of the warp takes part in the shuffles
                #pragma unroll
                for (int off = NQ / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
                if (cq == 0 && live) atomicMax(&rowmax[orow], __float_as_uint(m));
            }
        }
    }
}

template <int ST, int OTP, int CO>
cudaError_t launch_convt(const float* x, const float* W, const float* bias, float* out, int F, int T, int Cin,
                         int Cout, int k, int stride, int pad, int Tout, unsigned int* rowmax, cudaStream_t st) {
    const int slots = (k + stride - 1) / stride;
    const int per_group = (CO / 4) * (Tout / OTP);          // threads per sample group
    const int groups = kCtThreads / per_group;
    int SB = groups * ST;
    if (SB > F) SB = F;
    // whole warps (the row-absmax shuffles take every lane); extra threads own no chain
    const int threads = (per_group * ((SB + ST - 1) / ST) + 31) & ~31;
    const size_t smem = sizeof(float) * kCtStages * convt_stage_floats(k, SB * T, CO);
    if (groups < 1 || smem > 200 * 1024 || Cout % CO) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(conv_transpose1d_tiled_kernel<ST, OTP, CO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        attr = true;
    }
    return launch_k(conv_transpose1d_tiled_kernel<ST, OTP, CO>,
                    dim3((unsigned)(Cout / CO), (unsigned)((F + SB - 1) / SB)), (unsigned)threads, smem, st, x, W,
                    bias, out, F, T, Cin, Cout, k, stride, pad, Tout, SB, slots, rowmax);
}

// Few samples (batch 1): CTA = 8 output channels x 16 thread rows, a thread
// owns OPT chains of one sample, ci in chunks of 128 through the same kind of
// cp.async ring: more CTAs and threads per output than the tiled kernel above,
// which is what a lone sample's latency needs. Same per-output order.
constexpr int kChCo = 8, kChCi = 128, kChRows = 16, kChMaxK = 4, kChStages = 4;
constexpr int kChXs = kChCi + 4;   // x row stride in shared memory: 16-byte rows, distinct banks per row

__host__ __device__ constexpr size_t convt_chain_stage_floats(int k, int T) {
    return (size_t)kChCi * k * kChCo + (size_t)T * kChXs;
}

template <int OPT>
__global__ void __launch_bounds__(128)
conv_transpose1d_chain_kernel(const float* __restrict__ x, const float* __restrict__ W,
                              const float* __restrict__ bias, float* __restrict__ out, int T, int Cin, int Cout,
                              int k, int stride, int pad, int Tout, int slots, unsigned int* __restrict__ rowmax) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    extern __shared__ __align__(16) float ct_smem[];
    const int tx = threadIdx.x & (kChCo - 1), ty = threadIdx.x / kChCo;
    const int co0 = blockIdx.x * kChCo, f = blockIdx.y;
    const int co = co0 + tx;
    const float* xf = x + (long long)f * T * Cin;
    const size_t stage_fl = convt_chain_stage_floats(k, T);
    const int nchunk = (Cin + kChCi - 1) / kChCi;
    const int iters = slots * nchunk;           // (slot, chunk) in chain order
    float acc[OPT];
    int ot[OPT];
    #pragma unroll
    for (int i = 0; i < OPT; ++i) {
        ot[i] = ty + kChRows * i;
        acc[i] = (bias && co < Cout) ? bias[co] : 0.0f;
    }
    // cp.async of chunk c (ci block) into ring stage s: W rows (ci, kt) of 8
    // floats (two 16-byte pieces) and x rows t of kChCi floats; zero past Cin
    auto issue = [&](int it, int stg) {
        const int c = it % nchunk;
        float* sW = ct_smem + (size_t)stg * stage_fl;
        float* sx = sW + (size_t)kChCi * k * kChCo;
        const int ci0 = c * kChCi;
        for (int e = threadIdx.x; e < kChCi * k * 2; e += blockDim.x) {
            const int half = e & 1, r = e >> 1, kt = r % k, ci = ci0 + r / k;
            const bool ok = ci < Cin;
            cp_async16(sW + (size_t)r * kChCo + half * 4,
                       W + ((long long)(ok ? ci : 0) * k + kt) * Cout + co0 + half * 4, ok ? 16 : 0);
        }
        for (int e = threadIdx.x; e < T * (kChCi / 4); e += blockDim.x) {
            const int t = e / (kChCi / 4), q = e - t * (kChCi / 4), ci = ci0 + 4 * q;
            const bool ok = ci < Cin;
            cp_async16(sx + (size_t)t * kChXs + 4 * q, xf + (long long)t * Cin + (ok ? ci : 0), ok ? 16 : 0);
        }
    };
    for (int s0 = 0; s0 < kChStages - 1; ++s0) {
        if (s0 < iters) issue(s0, s0);
        cp_async_commit();
    }
    int cur_slot = -1;
    int kt_i[OPT], t_i[OPT];
    for (int it = 0; it < iters; ++it) {
        const int j = it / nchunk, c = it - j * nchunk;
        if (j != cur_slot) {      // this slot's tap and input row per output (-1: none)
            cur_slot = j;
            #pragma unroll
            for (int i = 0; i < OPT; ++i) {
                kt_i[i] = -1;
                t_i[i] = 0;
                if (ot[i] >= Tout) continue;
                int seen = 0;
                for (int kt = k - 1; kt >= 0; --kt) {
                    const int num = ot[i] + pad - kt;
                    if (num < 0 || num % stride) continue;
                    const int t = num / stride;
                    if (t >= T) continue;
                    if (seen++ == j) { kt_i[i] = kt; t_i[i] = t; break; }
                }
            }
        }
        asm volatile("cp.async.wait_group %0;" :: "n"(kChStages - 2) : "memory");
        __syncthreads();
        // refill the stage the previous iteration read (every thread is past it)
        if (it + kChStages - 1 < iters) issue(it + kChStages - 1, (it + kChStages - 1) % kChStages);
        cp_async_commit();
        const float* sW = ct_smem + (size_t)(it % kChStages) * stage_fl;
        const float* sx = sW + (size_t)kChCi * k * kChCo;
        const int cmax = min(kChCi, Cin - c * kChCi);
        #pragma unroll
        for (int i = 0; i < OPT; ++i) {
            if (kt_i[i] < 0) continue;
            const float* xr = sx + (size_t)t_i[i] * kChXs;
            const float* wr = sW + (size_t)kt_i[i] * kChCo + tx;
            // eight steps' operands are loaded before their fmas, so the chain
            // runs at the fma latency rather than the shared-memory latency
            int ci = 0;
            for (; ci + 8 <= cmax; ci += 8) {
                float xv[8], wv[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    xv[u] = xr[ci + u];
                    wv[u] = wr[(size_t)(ci + u) * k * kChCo];
                }
                #pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (xv[u] != 0.0f) acc[i] = __fmaf_rn(xv[u], wv[u], acc[i]);
            }
            for (; ci < cmax; ++ci) {
                const float v = xr[ci];
                if (v == 0.0f) continue;
                acc[i] = __fmaf_rn(v, wr[(size_t)ci * k * kChCo], acc[i]);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    #pragma unroll
    for (int i = 0; i < OPT; ++i) {
        const bool valid = ot[i] < Tout && co < Cout;
        if (valid) out[((long long)f * Tout + ot[i]) * Cout + co] = acc[i];
        if (rowmax) {
            // the 8 channels of this row sit in 8 consecutive lanes; every lane
            // of the warp takes part in the shuffles
            float m = valid ? fabsf(acc[i]) : 0.0f;
            #pragma unroll
            for (int off = 4; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
            if (tx == 0 && ot[i] < Tout) atomicMax(&rowmax[f * Tout + ot[i]], __float_as_uint(m));
        }
    }
}

template <int OPT>
cudaError_t launch_convt_chain(const float* x, const float* W, const float* bias, float* out, int F, int T, int Cin,
                         int Cout, int k, int stride, int pad, int Tout, unsigned int* rowmax, cudaStream_t st) {
    const int slots = (k + stride - 1) / stride;
    const size_t smem = sizeof(float) * kChStages * convt_chain_stage_floats(k, T);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(conv_transpose1d_chain_kernel<OPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024);
        attr = true;
    }
    return launch_k(conv_transpose1d_chain_kernel<OPT>, dim3((unsigned)(Cout / kChCo), (unsigned)F), 128, smem, st,
                    x, W, bias, out, T, Cin, Cout, k, stride, pad, Tout, slots, rowmax);
}

// 64 steps of one output's chain: acc = fma(x[u], w[u * wstep], acc) for u
// ascending, skipping x == 0 (the reference's skip) when SKIP. The next eight
// steps' operands are loaded before the current eight fmas, so the chain runs
// at the fma latency. Without zeros in x, SKIP = false gives the same bits.
template <bool SKIP, int WS>      // WS: the weight stride when known at compile time (else 0: wstep_rt)
__device__ __forceinline__ float convt_chain64(const float* xr, const float* wr, int wstep_rt, float acc) {
    const int wstep = WS ? WS : wstep_rt;      // a constant stride makes every load offset an immediate
    float xa[8], wa[8], xb[8], wb[8];
    auto ld = [&](float* xv, float* wv, int u0) {
        const float4 p = *reinterpret_cast<const float4*>(xr + u0);
        const float4 q = *reinterpret_cast<const float4*>(xr + u0 + 4);
        xv[0] = p.x; xv[1] = p.y; xv[2] = p.z; xv[3] = p.w;
        xv[4] = q.x; xv[5] = q.y; xv[6] = q.z; xv[7] = q.w;
        #pragma unroll
        for (int u = 0; u < 8; ++u) wv[u] = wr[(u0 + u) * wstep];
    };
    auto fm = [&](const float* xv, const float* wv) {
        #pragma unroll
        for (int u = 0; u < 8; ++u)
            if (!SKIP || xv[u] != 0.0f) acc = __fmaf_rn(xv[u], wv[u], acc);
    };
    ld(xa, wa, 0);
    #pragma unroll
    for (int u0 = 0; u0 < 64; u0 += 16) {
        ld(xb, wb, u0 + 8);
        fm(xa, wa);
        if (u0 + 16 < 64) ld(xa, wa, u0 + 16);
        fm(xb, wb);
    }
    return acc;
}

// OR of v over the `n` threads that meet at named barrier `id` (whole warps)
__device__ __forceinline__ bool bar_or(int id, int n, bool v) {
    int r;
    asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.s32 p, %1, 0;\n\t"
                 "bar.red.or.pred q, %2, %3, p;\n\tselp.s32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"(v ? 1 : 0), "r"(id), "r"(n) : "memory");
    return r != 0;
}

// Few samples with the CTA's whole weight slice resident: the chain kernel's
// CTA shape (8 output channels x 16 thread rows of one sample, OPT chains per
// thread, same per-output order) with W[0:Cin][0:k][co0:co0+8] in shared
// memory. The slice arrives as TMA tile loads of kRsBox (ci, tap) rows, one
// mbarrier each, all issued before the wait on the previous kernel (weights
// are load-time constants), so the first slot's chain starts on the first
// chunk and every later slot reads only shared memory: the weights cross HBM
// once per launch instead of once per slot.
constexpr int kRsBox = 256;        // (ci, tap) rows per TMA chunk (the box height)
constexpr int kRsMaxChunks = 64;

__host__ __device__ constexpr size_t convt_rs_w_bytes(int nchunks, int box) { return (size_t)nchunks * box * kChCo * 4; }

template <int OPT, int KS>       // KS: the tap count when fixed at compile time (the U-Net's 4), else 0
__global__ void __launch_bounds__(128)
conv_transpose1d_resident_kernel(const __grid_constant__ CUtensorMap tw, const float* __restrict__ x,
                                 const float* __restrict__ bias, float* __restrict__ out, int T, int Cin, int Cout,
                                 int k_rt, int stride, int pad, int Tout, int slots, int box, int nchunks,
                                 unsigned int* __restrict__ rowmax) {
    const int k = KS ? KS : k_rt;
    // Pointers are offsets into the __shared__ array (never integer casts), so
    // the compiler keeps them in the shared window: LDS, not generic loads.
    extern __shared__ __align__(16) float rs_smem[];
    float* sW = rs_smem + ((128u - (smem_u32(rs_smem) & 127u)) & 127u) / 4;    // 128-byte aligned TMA target
    float* sx = sW + convt_rs_w_bytes(nchunks, box) / 4;                      // [T][Cin + 4]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sx + (size_t)T * (Cin + 4));  // [nchunks]
    const int xs = Cin + 4;
    const int tx = threadIdx.x & (kChCo - 1), ty = threadIdx.x / kChCo;
    const int co0 = blockIdx.x * kChCo, f = blockIdx.y;
    const int co = co0 + tx;
    if (threadIdx.x == 0) {
        for (int c = 0; c < nchunks; ++c) mbar_init(&bars[c], 1);
        fence_mbar_init();
        tma_prefetch_desc(&tw);
        for (int c = 0; c < nchunks; ++c) {
            mbar_arrive_expect_tx(&bars[c], static_cast<uint32_t>(box * kChCo * 4));
            tma_load_2d(sW + (size_t)c * box * kChCo, &tw, &bars[c], co0, c * box);
        }
    }
    pdl_wait();     // x comes from the previous kernel in the stream
    pdl_trigger();
    const float* xf = x + (long long)f * T * Cin;
    bool zero = false;
    for (int e = threadIdx.x; e < T * (Cin / 4); e += blockDim.x) {
        const int t = e / (Cin / 4), q = e - t * (Cin / 4);
        const float4 v = *reinterpret_cast<const float4*>(xf + (long long)t * Cin + 4 * q);
        zero |= v.x == 0.0f || v.y == 0.0f || v.z == 0.0f || v.w == 0.0f;
        *reinterpret_cast<float4*>(sx + (size_t)t * xs + 4 * q) = v;
    }
    // x staged, barriers initialized; does any input need the zero skip?
    const bool any_zero = __syncthreads_or(zero) != 0;
    float acc[OPT];
    int ot[OPT];
    #pragma unroll
    for (int i = 0; i < OPT; ++i) {
        ot[i] = ty + kChRows * i;
        acc[i] = (bias && co < Cout) ? bias[co] : 0.0f;
    }
    int ready = 0;       // chunks this thread has seen arrive
    bool ok = true;
    for (int j = 0; j < slots && ok; ++j) {
        int kt_i[OPT], t_i[OPT];
        #pragma unroll
        for (int i = 0; i < OPT; ++i) {      // this slot's tap and input row per output (-1: none)
            kt_i[i] = -1;
            t_i[i] = 0;
            if (ot[i] >= Tout) continue;
            int seen = 0;
            for (int kt = k - 1; kt >= 0; --kt) {
                const int num = ot[i] + pad - kt;
                if (num < 0 || num % stride) continue;
                const int t = num / stride;
                if (t >= T) continue;
                if (seen++ == j) { kt_i[i] = kt; t_i[i] = t; break; }
            }
        }
        for (int ci0 = 0; ci0 < Cin && ok; ci0 += 64) {
            const int cn = min(64, Cin - ci0);
            // every (ci, tap) row of this block of 64 input channels has landed
            const int need = ((ci0 + cn) * k - 1) / box + 1;
            while (ready < need) {
                if (!mbar_wait(&bars[ready], 0)) { ok = false; break; }
                ++ready;
            }
            if (!ok) break;
            #pragma unroll
            for (int i = 0; i < OPT; ++i) {
                if (kt_i[i] < 0) continue;
                const float* xr = sx + (size_t)t_i[i] * xs + ci0;
                const float* wr = sW + ((size_t)ci0 * k + kt_i[i]) * kChCo + tx;
                if (cn == 64) {
                    acc[i] = any_zero ? convt_chain64<true, KS * kChCo>(xr, wr, k * kChCo, acc[i])
                                      : convt_chain64<false, KS * kChCo>(xr, wr, k * kChCo, acc[i]);
                } else {
                    for (int u = 0; u < cn; ++u) {
                        const float v = xr[u];
                        if (v == 0.0f) continue;
                        acc[i] = __fmaf_rn(v, wr[(size_t)u * k * kChCo], acc[i]);
                    }
                }
            }
        }
    }
    // no copy may still be landing when the CTA leaves: after a timeout the
    // rest are waited for once more, under one more bounded interval
    while (ok && ready < nchunks) {
        if (!mbar_wait(&bars[ready], 0)) ok = false;
        else ++ready;
    }
    if (!ok) {
        const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
        for (int c = ready; c < nchunks; ++c) mbar_wait_until(&bars[c], 0, deadline);
        return;
    }
    #pragma unroll
    for (int i = 0; i < OPT; ++i) {
        const bool valid = ot[i] < Tout && co < Cout;
        if (valid) out[((long long)f * Tout + ot[i]) * Cout + co] = acc[i];
        if (rowmax) {
            // the 8 channels of this row sit in 8 consecutive lanes; every lane
            // of the warp takes part in the shuffles
            float m = valid ? fabsf(acc[i]) : 0.0f;
            #pragma unroll
            for (int off = 4; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
            if (tx == 0 && ot[i] < Tout) atomicMax(&rowmax[f * Tout + ot[i]], __float_as_uint(m));
        }
    }
}

// fp32 [rows][cols] map with a {8, box_rows} box, no swizzle (the resident
// transposed conv's weight chunks: 32-byte rows packed in shared memory)
static bool make_tmap_f32_box8(CUtensorMap* map, const float* base, int rows, int cols, int box_rows) {
    auto fn = get_encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (cols & 3) || rows <= 0 || cols < kChCo) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 4};
    const cuuint32_t boxd[2] = {static_cast<cuuint32_t>(kChCo), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, boxd, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr size_t kRsMaxSmem = 220 * 1024;

static size_t convt_rs_smem(int T, int Cin, int k, int* box, int* nchunks) {
    const int rows = Cin * k;
    *box = rows < kRsBox ? rows : kRsBox;
    *nchunks = (rows + *box - 1) / *box;
    return 128 + convt_rs_w_bytes(*nchunks, *box) + (size_t)T * (Cin + 4) * 4 + kRsMaxChunks * 8;
}

// cudaErrorNotSupported: the shape is not for this kernel (the caller takes another)
template <int OPT>
cudaError_t launch_convt_resident(const float* x, const float* W, const float* bias, float* out, int F, int T,
                                  int Cin, int Cout, int k, int stride, int pad, int Tout, unsigned int* rowmax,
                                  cudaStream_t st) {
    int box = 0, nchunks = 0;
    const size_t smem = convt_rs_smem(T, Cin, k, &box, &nchunks);
    if (smem > kRsMaxSmem || nchunks > kRsMaxChunks || Cin % 4 || Cout % kChCo) return cudaErrorNotSupported;
    CUtensorMap tw;
    if (!make_tmap_f32_box8(&tw, W, Cin * k, Cout, box)) return cudaErrorNotSupported;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(conv_transpose1d_resident_kernel<OPT, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kRsMaxSmem);
        cudaFuncSetAttribute(conv_transpose1d_resident_kernel<OPT, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kRsMaxSmem);
        attr = true;
    }
    const int slots = (k + stride - 1) / stride;
    const dim3 grid((unsigned)(Cout / kChCo), (unsigned)F);
    if (k == 4)
        return launch_k(conv_transpose1d_resident_kernel<OPT, 4>, grid, 128, smem, st, tw, x, bias, out, T, Cin, Cout, k,
                        stride, pad, Tout, slots, box, nchunks, rowmax);
    return launch_k(conv_transpose1d_resident_kernel<OPT, 0>, grid, 128, smem, st, tw, x, bias, out, T, Cin, Cout, k,
                    stride, pad, Tout, slots, box, nchunks, rowmax);
}

// Several samples: CTA = 8 output channels x all Tout time steps x SB
// samples; a consumer thread owns one (channel, time step) of kBtSpt samples,
// their chains interleaved. x of the CTA's samples stays in shared memory; the
// weights stream from the transposed copy Wt [Cout][k][Cin] (ci contiguous)
// through a ring of TMA stages of ci_st input channels x `stride` taps x 8
// channels (128-byte swizzle: a warp's float4 reads of 8 rows hit 8 distinct
// bank groups), loaded by a producer warp that starts before the wait on the
// previous kernel. Pass p streams the taps [k - (p+1)*stride, k - p*stride):
// an output has at most one tap in such a window (the one of its residue mod
// stride), so the passes in order visit each output's taps in descending order
// and ci ascending within a tap - the reference's per-output order - and every
// weight is read once per CTA (the tiled kernel reads all k taps per slot).
// Eight 8 KB stages in flight per CTA: enough bytes to cover the TMA latency
// at the rate the chains consume them (four left the consumers waiting).
constexpr int kBtCo = 8, kBtBoxCi = 32, kBtStageCi = 128, kBtStages = 8, kBtSpt = 2, kBtMaxConsumers = 512;

__host__ __device__ constexpr int convt_bt_stage_bytes(int ci_st, int stride) {
    return (ci_st / kBtBoxCi) * kBtCo * stride * 128;
}

// One ring stage of a consumer's kBtSpt chains: nbox boxes of 32 input
// channels, the weight row `wrow` of each box (128-byte swizzled rows) against
// the samples' x rows (xr, sample stride `ss`). SKIP: the reference's zero skip.
template <bool SKIP>
__device__ __forceinline__ void convt_bt_stage(const uint8_t* wst, int sw, int box_bytes, int nbox, const float* xr,
                                               int ss, float (&acc)[kBtSpt]) {
    #pragma unroll 1
    for (int b = 0; b < nbox; ++b) {
        const uint8_t* wb = wst + b * box_bytes;
        const float* xb = xr + b * kBtBoxCi;
        #pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 w4 = *reinterpret_cast<const float4*>(wb + ((j ^ sw) << 4));
            #pragma unroll
            for (int i = 0; i < kBtSpt; ++i) {
                const float4 x4 = *reinterpret_cast<const float4*>(xb + i * ss + 4 * j);
                if (!SKIP || x4.x != 0.0f) acc[i] = __fmaf_rn(x4.x, w4.x, acc[i]);
                if (!SKIP || x4.y != 0.0f) acc[i] = __fmaf_rn(x4.y, w4.y, acc[i]);
                if (!SKIP || x4.z != 0.0f) acc[i] = __fmaf_rn(x4.z, w4.z, acc[i]);
                if (!SKIP || x4.w != 0.0f) acc[i] = __fmaf_rn(x4.w, w4.w, acc[i]);
            }
        }
    }
}

__global__ void __launch_bounds__(kBtMaxConsumers + 32)
conv_transpose1d_batched_kernel(const __grid_constant__ CUtensorMap twt, const float* __restrict__ x,
                                const float* __restrict__ bias, float* __restrict__ out, int F, int T, int Cin,
                                int Cout, int k, int stride, int pad, int Tout, int SB, int ci_st,
                                unsigned int* __restrict__ rowmax) {
    extern __shared__ __align__(16) uint8_t bt_smem[];
    uint8_t* ring = bt_smem + ((1024u - (smem_u32(bt_smem) & 1023u)) & 1023u);   // 128-byte swizzle: 1 KB aligned
    const int nbox = ci_st / kBtBoxCi;
    const int box_bytes = kBtCo * stride * 128;
    const int stage_bytes = nbox * box_bytes;
    const int xs = Cin + 4;                                          // 16-byte rows, distinct banks per row
    float* sx = reinterpret_cast<float*>(ring + (size_t)kBtStages * stage_bytes);     // [SB][T][xs]
    uint64_t* full = reinterpret_cast<uint64_t*>(sx + (size_t)SB * T * xs);
    uint64_t* empty = full + kBtStages;
    const int NC = kBtCo * Tout * (SB / kBtSpt);                     // consumer threads (whole warps)
    const int co0 = blockIdx.x * kBtCo, f0 = blockIdx.y * SB;
    const int nci = Cin / ci_st;
    const int G = ((k + stride - 1) / stride) * nci;                 // stages, pass-major
    if (threadIdx.x == 0) {
        for (int s = 0; s < kBtStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NC / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x >= NC) {
        // producer: weights are load-time constants, so no wait on the previous kernel
        if (threadIdx.x == NC) {
            tma_prefetch_desc(&twt);
            int issued = 0;
            for (int g = 0; g < G; ++g) {
                const int s = g % kBtStages;
                if (g >= kBtStages && !mbar_wait(&empty[s], ((g / kBtStages) - 1) & 1)) break;
                const int p = g / nci, c = g - p * nci;
                mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(stage_bytes));
                for (int b = 0; b < nbox; ++b)
                    tma_load_3d(ring + (size_t)s * stage_bytes + (size_t)b * box_bytes, &twt, &full[s],
                                c * ci_st + b * kBtBoxCi, k - (p + 1) * stride, co0);
                issued = g + 1;
            }
            // the copies still in flight (at most the last kBtStages) land before
            // this thread, and so the CTA, leaves, even if the consumers gave up
            const uint64_t deadline = globaltimer_ns() + kWaitLimitNs;
            for (int g = issued > kBtStages ? issued - kBtStages : 0; g < issued; ++g)
                mbar_wait_until(&full[g % kBtStages], (g / kBtStages) & 1, deadline);
        }
        return;
    }
    pdl_wait();     // x comes from the previous kernel in the stream
    pdl_trigger();
    const int c4 = Cin / 4;
    bool zero = false;
    for (int e = threadIdx.x; e < SB * T * c4; e += NC) {
        const int row = e / c4, q = e - row * c4;                   // row = sample * T + t
        float4 v = make_float4(1.0f, 1.0f, 1.0f, 1.0f);            // samples past F: no zeros to skip
        if (f0 + row / T < F) {
            v = *reinterpret_cast<const float4*>(x + ((long long)f0 * T + row) * Cin + 4 * q);
            zero |= v.x == 0.0f || v.y == 0.0f || v.z == 0.0f || v.w == 0.0f;
        }
        *reinterpret_cast<float4*>(sx + (size_t)row * xs + 4 * q) = v;
    }
    // consumers only: x staged; without zeros in it the skip changes nothing
    const bool any_zero = bar_or(1, NC, zero);
    const int ot = threadIdx.x % Tout;
    const int col = (threadIdx.x / Tout) % kBtCo;
    const int sg = threadIdx.x / (Tout * kBtCo);
    const int co = co0 + col;
    float acc[kBtSpt];
    #pragma unroll
    for (int i = 0; i < kBtSpt; ++i) acc[i] = bias ? bias[co] : 0.0f;
    int cur_p = -1, kt = -1, t = 0, wrow = 0;
    bool ok = true;
    for (int g = 0; g < G; ++g) {
        const int s = g % kBtStages;
        const int p = g / nci, c = g - p * nci;
        if (p != cur_p) {      // this pass's tap of this output (-1: none)
            cur_p = p;
            const int kt_lo = k - (p + 1) * stride;
            const int num_lo = ot + pad - kt_lo;
            kt = kt_lo + ((num_lo % stride) + stride) % stride;
            const int num = ot + pad - kt;
            t = num >= 0 ? num / stride : -1;
            if (kt < 0 || kt >= k || t < 0 || t >= T) kt = -1;
            wrow = col * stride + (kt - kt_lo);
        }
        if (!mbar_wait(&full[s], (g / kBtStages) & 1)) { ok = false; break; }
        if (kt >= 0) {
            const uint8_t* wst = ring + (size_t)s * stage_bytes + wrow * 128;
            const float* xr = sx + ((size_t)sg * kBtSpt * T + t) * xs + c * ci_st;
            if (any_zero) convt_bt_stage<true>(wst, wrow & 7, box_bytes, nbox, xr, T * xs, acc);
            else convt_bt_stage<false>(wst, wrow & 7, box_bytes, nbox, xr, T * xs, acc);
        }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) return;
    #pragma unroll
    for (int i = 0; i < kBtSpt; ++i) {
        const int sl = sg * kBtSpt + i;
        const bool live = f0 + sl < F;
        const long long orow = (long long)(f0 + sl) * Tout + ot;
        if (live) out[orow * Cout + co] = acc[i];
        if (rowmax) {
            // lane ^ Tout, ^ 2 Tout, ... hold this time step's other channels
            // of the CTA (Tout divides 32); every lane takes part
            float m = live ? fabsf(acc[i]) : 0.0f;
            for (int off = Tout; off < 32; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
            if ((threadIdx.x & 31) < Tout && live) atomicMax(&rowmax[orow], __float_as_uint(m));
        }
    }
}

// Wt [Cout][k][Cin] as a 3D map {Cin, k, Cout}, box {32, stride, 8}, 128-byte swizzle
static bool make_tmap_convt_wt(CUtensorMap* map, const float* Wt, int Cin, int k, int Cout, int stride) {
    auto fn = get_encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(Wt) & 15) || Cin % kBtBoxCi) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(Cin), static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(Cout)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(Cin) * 4, static_cast<cuuint64_t>(k) * Cin * 4};
    const cuuint32_t boxd[3] = {static_cast<cuuint32_t>(kBtBoxCi), static_cast<cuuint32_t>(stride),
                                static_cast<cuuint32_t>(kBtCo)};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(Wt), dims, strides, boxd, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static size_t convt_bt_smem(int SB, int T, int Cin, int ci_st, int stride) {
    return 1024 + (size_t)kBtStages * convt_bt_stage_bytes(ci_st, stride) + (size_t)SB * T * (Cin + 4) * 4 +
           2 * kBtStages * 8;
}

// cudaErrorNotSupported: the shape is not for this kernel (the caller takes another)
cudaError_t launch_convt_batched(const float* x, const float* Wt, const float* bias, float* out, int F, int T,
                                 int Cin, int Cout, int k, int stride, int pad, int Tout, unsigned int* rowmax,
                                 cudaStream_t st) {
    const bool tout_ok = Tout == 4 || Tout == 8 || Tout == 16 || Tout == 32;
    const int ci_st = Cin <= kBtStageCi ? Cin : kBtStageCi;
    if (!Wt || !tout_ok || Cin % kBtBoxCi || Cin % ci_st || Cout % kBtCo || stride > 32 || k > 256)
        return cudaErrorNotSupported;
    // samples per CTA: the fewest waves of CTAs (a CTA's time hardly depends on
    // its sample count: more samples are more threads), then the most CTAs
    const int groups_max = kBtMaxConsumers / (kBtCo * Tout);
    const long long co_blocks = Cout / kBtCo;
    const size_t limit = 220 * 1024;
    int SB = 0;
    long long best_waves = 0, best_grid = 0;
    for (int sb = kBtSpt; sb <= kBtSpt * groups_max; sb += kBtSpt) {
        const size_t sm = convt_bt_smem(sb, T, Cin, ci_st, stride);
        if (sm > limit) break;
        const long long grid = co_blocks * ((F + sb - 1) / sb);
        const long long per_sm = (long long)(228 * 1024) / (long long)(sm + 1024);
        const long long waves = (grid + 148 * per_sm - 1) / (148 * per_sm);
        if (!SB || waves < best_waves || (waves == best_waves && grid > best_grid)) {
            SB = sb;
            best_waves = waves;
            best_grid = grid;
        }
        if (sb >= F) break;
    }
    if (!SB) return cudaErrorNotSupported;
    const size_t smem = convt_bt_smem(SB, T, Cin, ci_st, stride);
    if ((F + SB - 1) / SB > 65535) return cudaErrorNotSupported;
    CUtensorMap twt;
    if (!make_tmap_convt_wt(&twt, Wt, Cin, k, Cout, stride)) return cudaErrorNotSupported;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(conv_transpose1d_batched_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)limit);
        attr = true;
    }
    const int threads = kBtCo * Tout * (SB / kBtSpt) + 32;
    return launch_k(conv_transpose1d_batched_kernel, dim3((unsigned)co_blocks, (unsigned)((F + SB - 1) / SB)),
                    (unsigned)threads, smem, st, twt, x, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, SB, ci_st,
                    rowmax);
}

cudaError_t conv_transpose1d_f(const float* x, const float* W, const float* Wt, const float* bias, float* out, int F,
                               int T, int Cin, int Cout, int k, int stride, int pad, unsigned int* rowmax,
                               cudaStream_t st) {
    const int Tout = (T - 1) * stride - 2 * pad + k;
    // 16-byte cp.async rows; time steps spread over at most 256 / 8 thread groups x 4 per thread
    if (F <= 0 || T <= 0 || Cin <= 0 || Cout <= 0 || k <= 0 || k > kCtMaxK || stride <= 0 || pad < 0 || Tout <= 0 ||
        Tout > 4 * (kCtThreads / 8) || T > 64 || Cin % 4 || Cout % 8 || F > 65535 ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W)) & 15))
        return cudaErrorInvalidValue;
    const int OTP = Tout <= 32 ? 1 : Tout <= 64 ? 2 : 4;
    if (Tout % OTP) return cudaErrorInvalidValue;
    if (F < 4 && Tout <= 4 * kChRows && Cout % kChCo == 0) {
        // a lone sample (or two, three): one sample per CTA row, one chain per
        // thread; the weight slice resident in shared memory where it fits
        cudaError_t e2;
        if (Tout <= kChRows) e2 = launch_convt_resident<1>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        else if (Tout <= 2 * kChRows) e2 = launch_convt_resident<2>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        else e2 = launch_convt_resident<4>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        if (e2 != cudaErrorNotSupported) {
            if (e2 != cudaSuccess) return e2;
            return cudaGetLastError();
        }
        if (Tout <= kChRows) e2 = launch_convt_chain<1>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        else if (Tout <= 2 * kChRows) e2 = launch_convt_chain<2>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        else e2 = launch_convt_chain<4>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        if (e2 != cudaSuccess) return e2;
        return cudaGetLastError();
    }
    if (Wt) {
        const cudaError_t e2 = launch_convt_batched(x, Wt, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
        if (e2 != cudaErrorNotSupported) {
            if (e2 != cudaSuccess) return e2;
            return cudaGetLastError();
        }
    }
    // many samples: 32 channels x 4 samples per CTA tile (weights reused across
    // the samples); otherwise 8 channels per CTA
    const bool wide = F >= 4 && Cout % 32 == 0;
    cudaError_t e;
    if (OTP == 1) e = wide ? launch_convt<4, 1, 32>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st)
                           : launch_convt<1, 1, 8>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
    else if (OTP == 2) e = wide ? launch_convt<4, 2, 32>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st)
                                : launch_convt<1, 2, 8>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
    else e = wide ? launch_convt<4, 4, 32>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st)
                  : launch_convt<1, 4, 8>(x, W, bias, out, F, T, Cin, Cout, k, stride, pad, Tout, rowmax, st);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// --------------------------------------------------- U-Net GroupNorm + Mish
// Block = one (group, sample) of x [F][T][C]: the group's statistics exactly
// as gn_affine_kernel (per channel over the T time steps, then the group), then
// v = mish(fma(x, A, B)) and the epilogue: FiLM fma(sc, v, bi) (film_scale) or
// v + film (bias only), or + res; out may alias x. rowmax (optional): atomicMax
// of each time step's |out| over this group's channels (the next conv's row
// quantization reads it).
__global__ void __launch_bounds__(256)
unet_gn_kernel(const float* x, int T, int C, int groups, float eps, const float* __restrict__ scale,
               const float* __restrict__ bias, int epi, const float* __restrict__ film, long long ld_film,
               const float* res, float* out, unsigned int* __restrict__ rowmax, int piece) {
    pdl_wait();     // x comes from the GEMM before
    pdl_trigger();
    extern __shared__ float ug_smem[];
    __shared__ double red[32];
    const int g = blockIdx.x, f = blockIdx.y;
    const int gc = C / groups, c0 = g * gc;
    float* sx = ug_smem;                                            // [T][gc]: the group's tile
    float* sA = ug_smem + (size_t)T * gc;                           // [gc]
    float* sB = sA + gc;                                            // [gc]
    unsigned int* srm = reinterpret_cast<unsigned int*>(sB + gc);   // [T]
    const float* xf = x + (long long)f * T * C + c0;
    // the tile in one sweep (all loads in flight), statistics from shared memory
    if ((gc & 3) == 0 && (C & 3) == 0 && (c0 & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int g4 = gc >> 2;
        for (int e = threadIdx.x; e < T * g4; e += blockDim.x) {
            const int p = e / g4, q = e - p * g4;
            *reinterpret_cast<float4*>(sx + (size_t)p * gc + 4 * q) =
                *reinterpret_cast<const float4*>(xf + (long long)p * C + 4 * q);
        }
    } else {
        for (int e = threadIdx.x; e < T * gc; e += blockDim.x) {
            const int p = e / gc, cl = e - p * gc;
            sx[e] = xf[(long long)p * C + cl];
        }
    }
    for (int p = threadIdx.x; p < T; p += blockDim.x) srm[p] = 0u;
    // the first epilogue pass's FiLM / residual operands and this thread's
    // first channel's scale and shift, loaded now so their latency overlaps
    // the statistics
    const int e_lo = blockIdx.z * piece, e_hi = min(T * gc, e_lo + piece);
    float pre_a = 0.0f, pre_b = 0.0f;
    const float sc0 = threadIdx.x < gc ? scale[c0 + threadIdx.x] : 0.0f;
    const float bi0 = threadIdx.x < gc ? bias[c0 + threadIdx.x] : 0.0f;
    {
        const int e = e_lo + threadIdx.x;
        if (e < e_hi) {
            const int p = e / gc, c = c0 + (e - p * gc);
            if (epi == kUgFilmScale) {
                pre_a = film[(long long)f * ld_film + c];
                pre_b = film[(long long)f * ld_film + C + c];
            } else if (epi == kUgFilmBias) {
                pre_a = film[(long long)f * ld_film + c];
            } else if (epi == kUgRes) {
                pre_a = res[((long long)f * T + p) * C + c];
            }
        }
    }
    __syncthreads();
    const double np = (double)T, n = np * gc;
    // per channel: shifted sums over the T steps (first step as the shift)
    double t1 = 0.0;
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        const double K = (double)sx[cl];
        double s1 = 0.0;
        for (int p = 0; p < T; ++p) s1 = __dadd_rn(s1, __dsub_rn((double)sx[(size_t)p * gc + cl], K));
        t1 = __dadd_rn(t1, __fma_rn(np, K, s1));
    }
    const double mean = __ddiv_rn(block_sum_d(t1, red), n);
    double t2 = 0.0;
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        const double K = (double)sx[cl];
        double s1 = 0.0, s2 = 0.0;
        for (int p = 0; p < T; ++p) {
            const double d = __dsub_rn((double)sx[(size_t)p * gc + cl], K);
            s1 = __dadd_rn(s1, d);
            s2 = __fma_rn(d, d, s2);
        }
        const double dk = __dsub_rn(K, mean);
        const double t = __fma_rn(__dmul_rn(2.0, dk), s1, s2);
        t2 = __dadd_rn(t2, __fma_rn(__dmul_rn(np, dk), dk, t));
    }
    const double ss = block_sum_d(t2, red);
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, n), (double)eps)));
    const double mi = __dmul_rn(mean, inv);
    for (int cl = threadIdx.x; cl < gc; cl += blockDim.x) {
        const float scv = cl == (int)threadIdx.x ? sc0 : scale[c0 + cl];
        const float biv = cl == (int)threadIdx.x ? bi0 : bias[c0 + cl];
        sA[cl] = (float)__dmul_rn(inv, (double)scv);
        sB[cl] = (float)__fma_rn(-mi, (double)scv, (double)biv);
    }
    __syncthreads();
    const float* ff = film ? film + (long long)f * ld_film : nullptr;
    // a warp's 32 consecutive elements share a time step when gc % 32 == 0:
    // one shared-memory atomic per warp then, else one per element
    const bool warp_rows = (gc & 31) == 0;
    // this CTA's piece of the (group, sample): elements [e_lo, e_hi) in whole
    // 256-element passes (every CTA of it computed the same statistics)
    for (int e0 = e_lo; e0 < e_hi; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        float m = 0.0f;
        int p = 0;
        if (e < e_hi) {
            p = e / gc;
            const int cl = e - p * gc, c = c0 + cl;
            const long long i = ((long long)f * T + p) * C + c;
            const bool first = e0 == e_lo;
            float v = mish_lanes(__fmaf_rn(sx[e], sA[cl], sB[cl]));
            if (epi == kUgFilmScale) v = __fmaf_rn(first ? pre_a : ff[c], v, first ? pre_b : ff[C + c]);
            else if (epi == kUgFilmBias) v = __fadd_rn(v, first ? pre_a : ff[c]);
            else if (epi == kUgRes) v = __fadd_rn(v, first ? pre_a : res[i]);
            out[i] = v;
            m = fabsf(v);
            if (rowmax && !warp_rows) atomicMax(&srm[p], __float_as_uint(m));
        }
        if (rowmax && warp_rows) {   // every lane takes part (blockDim, piece and T*gc are multiples of 32)
            m = warp_max_f(m);
            if ((threadIdx.x & 31) == 0 && e < e_hi) atomicMax(&srm[p], __float_as_uint(m));
        }
    }
    if (rowmax) {
        __syncthreads();
        for (int p = threadIdx.x; p < T; p += blockDim.x)
            if (srm[p]) atomicMax(&rowmax[f * T + p], srm[p]);
    }
}

cudaError_t unet_gn(const float* x, int F, int T, int C, int groups, float eps, const float* scale,
                    const float* bias, int epi, const float* film, long long ld_film, const float* res, float* out,
                    unsigned int* rowmax, cudaStream_t st) {
    if (F <= 0 || T <= 0 || C <= 0 || groups <= 0 || C % groups || F > 65535 ||
        ((epi == kUgFilmScale || epi == kUgFilmBias) && !film) || (epi == kUgRes && !res))
        return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * ((size_t)T * (C / groups) + 2 * (size_t)(C / groups) + T);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(unet_gn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    // With out apart from x, each (group, sample) spreads its elementwise
    // epilogue (Mish and the rest) over up to `pieces` CTAs of one 256-element
    // pass or more, each recomputing the group's statistics from the whole
    // tile, until the grid is about two CTAs per SM. In place (out == x) a
    // piece's writes could reach another CTA's tile before it is read: one CTA.
    const int n = T * (C / groups);
    int pieces = 1;
    if (out != x) {
        const long long gf = (long long)groups * F;
        pieces = (n + 255) / 256;
        const long long cap = (2LL * 148 + gf - 1) / gf;
        if (pieces > cap) pieces = (int)cap;
        if (pieces > 64) pieces = 64;
        if (pieces < 1) pieces = 1;
    }
    const int piece = ((n + pieces - 1) / pieces + 255) / 256 * 256;
    pieces = (n + piece - 1) / piece;
    const cudaError_t e = launch_k(unet_gn_kernel, dim3((unsigned)groups, (unsigned)F, (unsigned)pieces), 256, smem, st,
                                   x, T, C, groups, eps, scale, bias, epi, film, ld_film, res, out, rowmax, piece);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------- 1D im2col + row quantization
// Thread = 4 output bytes of one im2col row (sample f, time ot). The row's
// absmax is the max of its taps' per-time-step absmax (rowmax [F][T], float
// bits; zero taps add nothing), so every thread forms its row scale from at
// most k values and quantizes its 4 elements independently: the same int8
// codes and scale as quantize_act_i8 of the fp32 im2col row. rowmax may be null
// for narrow rows (k*C <= 64): the thread then scans the row itself.
__global__ void __launch_bounds__(256)
im2col1d_q8w_kernel(const float* __restrict__ x, int T, int C, int k, int stride, int pad, int Tout,
                    const unsigned int* __restrict__ rowmax, int8_t* __restrict__ q, long long ldq,
                    float* __restrict__ scale, long long rows, int vec4) {
    pdl_wait();     // x and rowmax come from earlier kernels in the stream
    pdl_trigger();
    const long long g4n = ldq >> 2, total = rows * g4n;
    const int K = k * C;
    for (long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x; tid < total;
         tid += (long long)gridDim.x * blockDim.x) {
        const long long r = tid / g4n;
        const int g4 = static_cast<int>(tid - r * g4n);
        const int f = static_cast<int>(r / Tout), ot = static_cast<int>(r - (long long)f * Tout);
        const float* xf = x + (long long)f * T * C;
        float m = 0.0f;
        if (rowmax) {
            unsigned int mb = 0u;
            for (int kt = 0; kt < k; ++kt) {
                const int t = ot * stride - pad + kt;
                if (t >= 0 && t < T) mb = max(mb, rowmax[f * T + t]);
            }
            m = __uint_as_float(mb);
        } else {
            for (int e = 0; e < K; ++e) {
                const int kt = e / C, t = ot * stride - pad + kt;
                if (t >= 0 && t < T) m = fmaxf(m, fabsf(xf[(long long)t * C + (e - kt * C)]));
            }
        }
        const float s = nn_row_scale(m), inv = __fdiv_rn(1.0f, s);
        if (g4 == 0) scale[r] = s;
        int8_t b[4];
        if (vec4) {   // C % 4 == 0: the 4 elements are 4 channels of one tap
            const int e = 4 * g4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e < K) {
                const int kt = e / C, t = ot * stride - pad + kt;
                if (t >= 0 && t < T) v = *reinterpret_cast<const float4*>(xf + (long long)t * C + (e - kt * C));
            }
            const bool in = e < K;
            b[0] = in ? nn_q8(v.x, inv) : 0;
            b[1] = in ? nn_q8(v.y, inv) : 0;
            b[2] = in ? nn_q8(v.z, inv) : 0;
            b[3] = in ? nn_q8(v.w, inv) : 0;
        } else {
            #pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = 4 * g4 + u;
                float v = 0.0f;
                if (e < K) {
                    const int kt = e / C, t = ot * stride - pad + kt;
                    if (t >= 0 && t < T) v = xf[(long long)t * C + (e - kt * C)];
                }
                b[u] = e < K ? nn_q8(v, inv) : 0;
            }
        }
        *reinterpret_cast<char4*>(q + r * ldq + 4 * g4) = make_char4(b[0], b[1], b[2], b[3]);
    }
}

cudaError_t im2col1d_q8w(const float* x, int F, int T, int C, int k, int stride, int pad, int Tout,
                         const unsigned int* rowmax, int8_t* q, long long ldq, float* scale, cudaStream_t st) {
    if (F <= 0 || T <= 0 || C <= 0 || k <= 0 || stride <= 0 || pad < 0 || Tout <= 0 || ldq < (long long)k * C ||
        (ldq & 15) || (reinterpret_cast<uintptr_t>(q) & 15) || (!rowmax && (long long)k * C > 64))
        return cudaErrorInvalidValue;
    const long long rows = (long long)F * Tout;
    const int vec4 = (C % 4 == 0) && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const cudaError_t e = launch_k(im2col1d_q8w_kernel, (unsigned)grid_cap(rows * (ldq >> 2), 256, 148 * 8), 256, 0,
                                   st, x, T, C, k, stride, pad, Tout, rowmax, q, ldq, scale, rows, vec4);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// cat [F*T][C1 + C2] = [a | b] per row, with the row's absmax (float bits) into
// rowmax. Row blockIdx.x, piece blockIdx.y: the pieces stride the row's
// elements (float4 units when vec4), so a short U-Net row of 4096 channels is
// one load per thread over several CTAs instead of a serial loop in one. With
// more than one piece the partial maxima meet by atomicMax (absmax >= 0, so the
// float bits order as unsigned), which needs the slots zeroed before the
// launch; max is order-free, so the result is the same as one pass.
__global__ void __launch_bounds__(256)
concat_rows_kernel(const float* __restrict__ a, int C1, const float* __restrict__ b, int C2, float* __restrict__ cat,
                   unsigned int* __restrict__ rowmax, int vec4) {
    pdl_wait();     // inputs come from earlier kernels in the stream
    pdl_trigger();
    __shared__ float sh[32];
    const long long r = blockIdx.x;
    const int Cc = C1 + C2;
    const int first = blockIdx.y * blockDim.x + threadIdx.x, step = gridDim.y * blockDim.x;
    float m = 0.0f;
    if (vec4) {
        const int n1 = C1 >> 2, n = Cc >> 2;
        const float4* a4 = reinterpret_cast<const float4*>(a + r * C1);
        const float4* b4 = reinterpret_cast<const float4*>(b + r * C2);
        float4* c4 = reinterpret_cast<float4*>(cat + r * Cc);
        for (int c = first; c < n; c += step) {
            const float4 v = c < n1 ? a4[c] : b4[c - n1];
            c4[c] = v;
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    } else {
        for (int c = first; c < Cc; c += step) {
            const float v = c < C1 ? a[r * C1 + c] : b[r * C2 + (c - C1)];
            cat[r * Cc + c] = v;
            m = fmaxf(m, fabsf(v));
        }
    }
    m = block_max_256(m, sh);
    if (threadIdx.x == 0 && rowmax) {
        if (gridDim.y == 1) rowmax[r] = __float_as_uint(m);
        else atomicMax(rowmax + r, __float_as_uint(m));
    }
}

// --------------------------------------------------- cond encoder input
// gm = mish([stepfeat | gcond]) per step and query. Mish's 8-lane body covers
// the first CD - CD % 8 elements (mish_lanes, exact); the last CD % 8 are the
// reference's scalar libm tail, whose values arrive precomputed in tail
// [B][CD % 8] (evaluated with the host's libm, see DpPolicy::forward).
__global__ void dp_cond_input_kernel(const float* __restrict__ stepfeat, int n_steps, int D,
                                     const float* __restrict__ gcond, const float* __restrict__ tail, int B, int CD,
                                     float* __restrict__ gm) {
    pdl_wait();     // gcond comes from the encoders of this step
    pdl_trigger();
    const long long total = (long long)n_steps * B * CD;
    const int nt = CD % 8, lanes_end = CD - nt;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / CD;
        const int j = static_cast<int>(i - r * CD);
        const int step = static_cast<int>(r / B), b = static_cast<int>(r - (long long)step * B);
        if (j < lanes_end) {
            const float v = j < D ? stepfeat[(long long)step * D + j] : gcond[(long long)b * (CD - D) + (j - D)];
            gm[i] = mish_lanes(v);
        } else {
            gm[i] = tail[(long long)b * nt + (j - lanes_end)];
        }
    }
}

cudaError_t dp_cond_input(const float* stepfeat, int n_steps, int D, const float* gcond, const float* tail, int B,
                          int CD, float* gm, cudaStream_t st) {
    if (n_steps <= 0 || D <= 0 || B <= 0 || CD <= D || CD - CD % 8 < D || (CD % 8 && !tail))
        return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(dp_cond_input_kernel, (unsigned)grid_cap((long long)n_steps * B * CD, 256, 148 * 4),
                                   256, 0, st, stepfeat, n_steps, D, gcond, tail, B, CD, gm);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// The scalar tail of the reference's Mish over the conditioning vector (the
// last cond_dim % 8 entries its 8-lane loop leaves, src/hal/common/eltwise.cpp:244-248),
// with the host library's float functions restated: tail[b][i] =
// mish(gcond[b][G - n + i]).
__global__ void dp_mish_tail_kernel(const float* __restrict__ gcond, int G, int n, int B, float* __restrict__ tail) {
    pdl_wait();     // gcond comes from the previous kernel
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * n) return;
    const int b = i / n, j = i - b * n;
    tail[i] = lf_mish(gcond[(long long)b * G + (G - n) + j]);
}

cudaError_t dp_mish_tail(const float* gcond, int G, int n, int B, float* tail, cudaStream_t st) {
    if (n <= 0 || n > G || B <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(dp_mish_tail_kernel, (unsigned)((B * n + 127) / 128), 128, 0, st, gcond, G, n, B, tail);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------- step prologue
__global__ void dp_prologue_kernel(unsigned int* __restrict__ zero, int n_zero, const float* __restrict__ state, int B,
                                   int S, int sd, const float* __restrict__ smin, const float* __restrict__ smax,
                                   float eps, float* __restrict__ gcond, int per_step, const float* __restrict__ noise,
                                   long long noise_stride, int HA, float* __restrict__ sample) {
    pdl_wait();     // the previous step may still read these buffers
    pdl_trigger();
    const long long tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = tid; i < n_zero; i += stride) zero[i] = 0u;
    // 2 (state - min) / d - 1, d = max - min (eps when 0): diffusion_model.cpp:203-207
    for (long long i = tid; i < (long long)B * S * sd; i += stride) {
        const int j = static_cast<int>(i % sd);
        const long long bs = i / sd;
        const int s = static_cast<int>(bs % S), b = static_cast<int>(bs / S);
        const float den = __fsub_rn(smax[j], smin[j]);
        const float d = den == 0.0f ? eps : den;
        const float t = __fsub_rn(state[i], smin[j]);
        gcond[(long long)b * S * per_step + (long long)s * per_step + j] =
            __fsub_rn(__fdiv_rn(__fadd_rn(t, t), d), 1.0f);
    }
    for (long long i = tid; i < (long long)B * HA; i += stride) {
        const long long b = i / HA;
        sample[i] = noise[b * noise_stride + (i - b * HA)];
    }
}

cudaError_t dp_prologue(unsigned int* zero, int n_zero, const float* state, int B, int S, int sd, const float* smin,
                        const float* smax, float eps, float* gcond, int per_step, const float* noise,
                        long long noise_stride, int HA, float* sample, cudaStream_t st) {
    if (B <= 0 || S <= 0 || sd <= 0 || HA <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(dp_prologue_kernel, 32, 256, 0, st, zero, n_zero, state, B, S, sd, smin, smax, eps,
                                   gcond, per_step, noise, noise_stride, HA, sample);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------- reverse step
__global__ void dp_sched_step_kernel(float* __restrict__ sample, const float* __restrict__ eps,
                                     const float* __restrict__ noise, long long noise_stride, int HA, long long n,
                                     DdStepConsts c) {
    pdl_wait();     // eps comes from the U-Net's last kernel
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const double s = (double)sample[i], e = (double)eps[i];
        double x0 = __ddiv_rn(__fma_rn(-c.sqrt_bp, e, s), c.sqrt_ap);
        if (c.clip) {
            x0 = (c.lo < x0) ? x0 : c.lo;    // std::max(lo, x0)
            x0 = (x0 < c.hi) ? x0 : c.hi;    // std::min(hi, .)
        }
        double v;
        if (!c.ddpm) {
            v = __fma_rn(x0, c.a, __dmul_rn(c.b, e));
        } else {
            v = __fma_rn(x0, c.a, __dmul_rn(c.b, s));
            if (noise) {
                const long long b = i / HA;
                v = __fma_rn(c.var, (double)noise[b * noise_stride + (i - b * HA)], v);
            }
        }
        sample[i] = __double2float_rn(v);
    }
}

cudaError_t dp_sched_step(float* sample, const float* eps, const float* noise, long long noise_stride, int B, int HA,
                          const DdStepConsts& c, cudaStream_t st) {
    if (B <= 0 || HA <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)B * HA;
    const cudaError_t e = launch_k(dp_sched_step_kernel, (unsigned)grid_cap(n, 256, 148), 256, 0, st, sample, eps,
                                   noise, noise_stride, HA, n, c);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------------ actions
__global__ void dp_actions_kernel(const float* __restrict__ sample, int B, int horizon, int A, int start, int n_act,
                                  const float* __restrict__ amin, const float* __restrict__ amax, float eps,
                                  float* __restrict__ actions) {
    pdl_wait();     // sample comes from the last reverse step
    pdl_trigger();
    const long long total = (long long)B * n_act * A;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int a = static_cast<int>(i % A);
        const long long bt = i / A;
        const int t = static_cast<int>(bt % n_act), b = static_cast<int>(bt / n_act);
        const float s = sample[((long long)b * horizon + start + t) * A + a];
        if (amin) {
            const float den = __fsub_rn(amax[a], amin[a]);
            const float d = den == 0.0f ? eps : den;
            actions[i] = __fmaf_rn(__fmul_rn(__fadd_rn(s, 1.0f), 0.5f), d, amin[a]);
        } else {
            actions[i] = s;
        }
    }
}

cudaError_t dp_actions(const float* sample, int B, int horizon, int A, int start, int n_act, const float* amin,
                       const float* amax, float eps, float* actions, cudaStream_t st) {
    if (B <= 0 || A <= 0 || n_act <= 0 || start < 0 || start + n_act > horizon) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(dp_actions_kernel, (unsigned)grid_cap((long long)B * n_act * A, 256, 64), 256, 0,
                                   st, sample, B, horizon, A, start, n_act, amin, amax, eps, actions);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------- spatial softmax
// Per (frame, channel): max shift, then exp / sum / expected (x, y) in pixel
// order with the coordinate products fused (src/hal/common/conv.cpp:397-422),
// exp the host library's (libm_expf).
__global__ void spatial_softmax_f_kernel(const float* __restrict__ x, const float* __restrict__ grid,
                                         float* __restrict__ out, int F, int npx, int C) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)F * C) return;
    const int f = static_cast<int>(i / C), c = static_cast<int>(i - (long long)f * C);
    const float* xf = x + (long long)f * npx * C;
    float m = -INFINITY;
    for (int p = 0; p < npx; ++p) {
        const float v = xf[(long long)p * C + c];
        if (v > m) m = v;
    }
    float sum = 0.0f, ex = 0.0f, ey = 0.0f;
    for (int p = 0; p < npx; ++p) {
        const float e = libm_expf(__fsub_rn(xf[(long long)p * C + c], m));
        sum = __fadd_rn(sum, e);
        ex = __fmaf_rn(e, grid[2 * p], ex);
        ey = __fmaf_rn(e, grid[2 * p + 1], ey);
    }
    const float inv = __fdiv_rn(1.0f, sum);
    out[(long long)f * 2 * C + 2 * c] = __fmul_rn(ex, inv);
    out[(long long)f * 2 * C + 2 * c + 1] = __fmul_rn(ey, inv);
}

cudaError_t concat_channels(const float* a, int C1, const float* b, int C2, float* cat, int F, int T,
                            unsigned int* rowmax, cudaStream_t st) {
    if (F <= 0 || T <= 0 || C1 <= 0 || C2 <= 0 || (long long)F * T > 2147483647LL) return cudaErrorInvalidValue;
    const int vec4 = ((C1 | C2) & 3) == 0 && ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) |
                                                reinterpret_cast<uintptr_t>(cat)) & 15) == 0;
    const int units = vec4 ? (C1 + C2) / 4 : C1 + C2;
    const int pieces = (units + 255) / 256 < 65535 ? (units + 255) / 256 : 65535;
    const cudaError_t e = launch_k(concat_rows_kernel, dim3((unsigned)(F * T), (unsigned)pieces), 256, 0, st, a, C1, b,
                                   C2, cat, rowmax, vec4);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t spatial_softmax_f(const float* x, const float* grid, float* out, int F, int npx, int C, cudaStream_t st) {
    if (F <= 0 || npx <= 0 || C <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(spatial_softmax_f_kernel, (unsigned)(((long long)F * C + 127) / 128), 128, 0, st, x,
                                   grid, out, F, npx, C);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void relu_rows_kernel(float* __restrict__ x, int M, int N, long long ld) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const long long total = (long long)M * N;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / N;
        float* p = x + r * ld + (i - r * N);
        const float v = *p;
        *p = v < 0.0f ? 0.0f : v;   // tcpu::relu (src/hal/common/eltwise.cpp:209-215)
    }
}

cudaError_t relu_rows(float* x, int M, int N, long long ld, cudaStream_t st) {
    if (M <= 0 || N <= 0 || ld < N) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(relu_rows_kernel, (unsigned)grid_cap((long long)M * N, 256, 148), 256, 0, st, x, M,
                                   N, ld);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace vsb
