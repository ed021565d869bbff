// Octo kernels around the shared GEMM / LayerNorm / attention / conv ones:
// the SmallStem input, the T5 language tower's embedding, bias and attention,
// the block-causal token sequence and its mask, and the diffusion head's
// elementwise steps. Every formula is the reference's, operation for
// operation, with the contractions its -ffp-contract=fast build makes (read
// from the compiled reference): the policy's actions then equal the
// reference's bit for bit wherever the layers before them do.
#include "sm100.cuh"
#include "launch.cuh"
#include "octo.h"

#include <cfloat>

namespace vsb {

// --------------------------------------------------------------- stem input
__global__ void octo_stem_input_kernel(const uint8_t* __restrict__ img, long long npx, float* __restrict__ out,
                                       unsigned int* __restrict__ amax) {
    pdl_wait();
    pdl_trigger();
    __shared__ float sh[8];
    const int f = blockIdx.y;
    const uint8_t* src = img + (long long)f * npx * 3;
    float* dst = out + (long long)f * npx * 6;
    float m = 0.0f;
    for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < npx; p += (long long)gridDim.x * blockDim.x) {
        float v[6];
        #pragma unroll
        for (int c = 0; c < 3; ++c) {
            v[c] = __fsub_rn(__fdiv_rn(static_cast<float>(src[p * 3 + c]), 127.5f), 1.0f);
            m = fmaxf(m, fabsf(v[c]));
            v[3 + c] = -1.0f;
        }
        m = fmaxf(m, 1.0f);
        float2* d2 = reinterpret_cast<float2*>(dst + p * 6);
        d2[0] = make_float2(v[0], v[1]);
        d2[1] = make_float2(v[2], v[3]);
        d2[2] = make_float2(v[4], v[5]);
    }
    m = block_max_256(m, sh);
    if (threadIdx.x == 0 && amax) atomicMax(amax + f, __float_as_uint(m));
}

cudaError_t octo_stem_input(const uint8_t* img, int F, long long npx, float* out, unsigned int* amax,
                            cudaStream_t st) {
    if (F <= 0 || npx <= 0 || F > 65535) return cudaErrorInvalidValue;
    const unsigned bx = (unsigned)grid_cap(npx, 256, 64);
    const cudaError_t e = launch_k(octo_stem_input_kernel, dim3(bx, F), 256, 0, st, img, npx, out, amax);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// --------------------------------------------------------------------- T5
__global__ void t5_embed_kernel(const int* __restrict__ ids, int n, const float* __restrict__ emb, int vocab, int D,
                                int pad_id, const float* __restrict__ rel, const int* __restrict__ bucket, int NH,
                                float* __restrict__ x, float* __restrict__ bias) {
    pdl_wait();
    pdl_trigger();
    const long long nx = (long long)n * D, nb = (long long)NH * n * n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nx + nb;
         i += (long long)gridDim.x * blockDim.x) {
        if (i < nx) {
            const int t = static_cast<int>(i / D), c = static_cast<int>(i - (long long)t * D);
            const int id = ids[t];
            x[i] = (id >= 0 && id < vocab) ? emb[(long long)id * D + c] : 0.0f;
        } else {
            const long long r = i - nx;
            const int h = static_cast<int>(r / ((long long)n * n));
            const int ij = static_cast<int>(r - (long long)h * n * n);
            const int qi = ij / n, kj = ij - qi * n;
            bias[r] = ids[kj] != pad_id ? rel[(long long)bucket[kj - qi + n - 1] * NH + h] : -FLT_MAX;
        }
    }
}

cudaError_t t5_embed(const int* ids, int n, const float* emb, int vocab, int D, int pad_id, const float* rel,
                     const int* bucket, int NH, float* x, float* bias, cudaStream_t st) {
    if (n <= 0 || D <= 0 || NH <= 0 || vocab <= 0) return cudaErrorInvalidValue;
    const long long total = (long long)n * D + (long long)NH * n * n;
    const cudaError_t e = launch_k(t5_embed_kernel, (unsigned)grid_cap(total, 256, 148 * 4), 256, 0, st, ids, n,
                                   emb, vocab, D, pad_id, rel, bucket, NH, x, bias);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// simd_dot (src/hal/avx2/simd.h:12-40) of n values over one warp, n % 8 == 0:
// lane 8j + l carries the reference's chain j, lane l; 32-wide steps, then
// 8-wide steps into chain 0; (c0 + c1) + (c2 + c3); hsum8. All lanes return it.
__device__ __forceinline__ float warp_simd_dot(const float* __restrict__ a, const float* __restrict__ b, int n) {
    const int lane = threadIdx.x & 31;
    float acc = 0.0f;
    const int n32 = n & ~31;
    for (int k = 0; k < n32; k += 32) acc = __fmaf_rn(a[k + lane], b[k + lane], acc);
    for (int k = n32; k + 8 <= n; k += 8)
        if (lane < 8) acc = __fmaf_rn(a[k + lane], b[k + lane], acc);
    const float a1 = __shfl_down_sync(0xFFFFFFFFu, acc, 8);
    const float a2 = __shfl_down_sync(0xFFFFFFFFu, acc, 16);
    const float a3 = __shfl_down_sync(0xFFFFFFFFu, acc, 24);
    acc = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
    float l[8];
    #pragma unroll
    for (int i = 0; i < 8; ++i) l[i] = __shfl_sync(0xFFFFFFFFu, acc, i);
    return __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                     __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
}

constexpr int kT5MaxSeq = 256;

// one warp per (head, query): scores in shared memory, then the reference's
// serial softmax sum and in-order axpy over the keys
__global__ void t5_attention_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                                    const float* __restrict__ V, const float* __restrict__ bias, int n, int NH,
                                    int hd, float scale, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float sc[4][kT5MaxSeq];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 4 + w;   // h * n + t1
    if (row >= NH * n) return;
    const int h = row / n, t1 = row - h * n;
    const int D = NH * hd;
    const float NINF = __int_as_float(0xff800000);
    const float* q = Q + (long long)t1 * D + h * hd;
    const float* brow = bias + ((long long)h * n + t1) * n;
    float* s = sc[w];
    float mx = NINF;
    for (int t2 = 0; t2 < n; ++t2) {
        float v;
        if (brow[t2] == -FLT_MAX) {
            v = NINF;
        } else {
            const float dot = warp_simd_dot(q, K + (long long)t2 * D + h * hd, hd);
            v = __fmaf_rn(dot, scale, brow[t2]);
        }
        if (lane == 0) s[t2] = v;
        mx = v > mx ? v : mx;
    }
    __syncwarp();
    float sum = 0.0f;
    if (mx == NINF) {
        for (int t2 = lane; t2 < n; t2 += 32) s[t2] = 1.0f;
        sum = static_cast<float>(n);
    } else {
        for (int t2 = lane; t2 < n; t2 += 32) s[t2] = s[t2] == NINF ? 0.0f : libm_expf(__fsub_rn(s[t2], mx));
        __syncwarp();
        for (int t2 = 0; t2 < n; ++t2) sum = __fadd_rn(sum, s[t2]);
    }
    __syncwarp();
    const float inv = __fdiv_rn(1.0f, sum);
    float* o = out + (long long)t1 * D + h * hd;
    for (int d = lane; d < hd; d += 32) {
        float acc = 0.0f;
        for (int t2 = 0; t2 < n; ++t2) {
            const float p = s[t2];
            if (p == 0.0f) continue;
            acc = __fmaf_rn(__fmul_rn(p, inv), V[(long long)t2 * D + h * hd + d], acc);
        }
        o[d] = acc;
    }
}

cudaError_t t5_attention(const float* Q, const float* K, const float* V, const float* bias, int n, int NH, int hd,
                         float scale, float* out, cudaStream_t st) {
    if (n <= 0 || n > kT5MaxSeq || NH <= 0 || hd <= 0 || hd % 8) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(t5_attention_kernel, (unsigned)((NH * n + 3) / 4), 128, 0, st, Q, K, V, bias, n,
                                   NH, hd, scale, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------ token sequence
__global__ void octo_assemble_kernel(OctoSeq s, const float* __restrict__ task, const float* __restrict__ pos_task,
                                     const float* __restrict__ prim,
                                     const float* __restrict__ pos_prim, const float* __restrict__ wrist,
                                     const float* __restrict__ pos_wrist, const float* __restrict__ pos_readout,
                                     float* __restrict__ x) {
    pdl_wait();
    pdl_trigger();
    const int total = s.total(), per = s.P + s.Wr + s.n_task + s.R;
    const int d4 = s.d / 4;
    const long long n = (long long)s.B * total * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / d4;
        const int c = static_cast<int>(i - row * d4) * 4;
        const int b = static_cast<int>(row / total), tok = static_cast<int>(row - (long long)b * total);
        auto add = [](float4 a, float4 p) {
            return make_float4(__fadd_rn(a.x, p.x), __fadd_rn(a.y, p.y), __fadd_rn(a.z, p.z), __fadd_rn(a.w, p.w));
        };
        // task token k: its projection + pos_task[k] (the same values in both places)
        auto task_tok = [&](int k) {
            return add(*reinterpret_cast<const float4*>(task + ((long long)b * s.n_task + k) * s.d + c),
                       *reinterpret_cast<const float4*>(pos_task + (long long)k * s.d + c));
        };
        float4 v;
        if (tok < s.n_task) {
            v = task_tok(tok);
        } else {
            const int t = (tok - s.n_task) / per, j = (tok - s.n_task) - t * per;
            if (j < s.P) {
                const float4 a = *reinterpret_cast<const float4*>(prim + (((long long)b * s.wnd + t) * s.P + j) * s.d + c);
                v = add(a, *reinterpret_cast<const float4*>(pos_prim + ((long long)t * s.P + j) * s.d + c));
            } else if (j < s.P + s.Wr) {
                const int jw = j - s.P;
                if (wrist) {
                    const float4 a =
                        *reinterpret_cast<const float4*>(wrist + (((long long)b * s.wnd + t) * s.Wr + jw) * s.d + c);
                    v = add(a, *reinterpret_cast<const float4*>(pos_wrist + ((long long)t * s.Wr + jw) * s.d + c));
                } else {
                    v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            } else if (j < s.P + s.Wr + s.n_task) {
                v = task_tok(j - s.P - s.Wr);
            } else {
                v = *reinterpret_cast<const float4*>(pos_readout +
                                                     ((long long)t * s.R + (j - s.P - s.Wr - s.n_task)) * s.d + c);
            }
        }
        *reinterpret_cast<float4*>(x + row * s.d + c) = v;
    }
}

cudaError_t octo_assemble(const OctoSeq& s, const float* task, const float* pos_task, const float* prim,
                          const float* pos_prim, const float* wrist, const float* pos_wrist, const float* pos_readout,
                          float* x, cudaStream_t st) {
    if (s.B <= 0 || s.wnd <= 0 || s.d % 4) return cudaErrorInvalidValue;
    const long long n = (long long)s.B * s.total() * (s.d / 4);
    const cudaError_t e = launch_k(octo_assemble_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, s, task,
                                   pos_task, prim, pos_prim, wrist, pos_wrist, pos_readout, x);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// groups: 0 task prefix (timestep -1), 1 primary, 2 wrist, 3 repeated task, 4 readout
__device__ __forceinline__ void octo_token(const OctoSeq& s, int tok, int& g, int& t) {
    if (tok < s.n_task) {
        g = 0;
        t = -1;
        return;
    }
    const int per = s.P + s.Wr + s.n_task + s.R;
    t = (tok - s.n_task) / per;
    const int j = (tok - s.n_task) - t * per;
    g = j < s.P ? 1 : j < s.P + s.Wr ? 2 : j < s.P + s.Wr + s.n_task ? 3 : 4;
}

__global__ void octo_mask_kernel(OctoSeq s, const uint8_t* __restrict__ tmask, int wrist, float* __restrict__ mask) {
    pdl_wait();
    pdl_trigger();
    const int total = s.total();
    const long long tt = (long long)total * total;
    const long long n = (long long)s.B * tt;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int b = static_cast<int>(i / tt);
        const long long r = i - (long long)b * tt;
        const int qi = static_cast<int>(r / total), kj = static_cast<int>(r - (long long)qi * total);
        int gi, ti, gj, tj;
        octo_token(s, qi, gi, ti);
        octo_token(s, kj, gj, tj);
        bool keep;
        if (gi == 0) keep = gj == 0;                 // task -> task only
        else if (gj == 0) keep = true;               // everyone -> task
        else if (gj <= 3) keep = tj <= ti;           // -> observations, causal over steps
        else keep = gi == 4 && tj <= ti;             // readout -> readouts, causal
        // keys of padded steps: primary and wrist observations are blocked
        const uint8_t* tm = tmask + (long long)b * s.wnd;
        const bool pad_ok = gj == 1 ? tm[tj] != 0 : gj == 2 ? (wrist && tm[tj] != 0) : true;
        mask[i] = (keep && pad_ok) ? 0.0f : -FLT_MAX;
    }
}

cudaError_t octo_mask(const OctoSeq& s, const uint8_t* tmask, bool wrist, float* mask, cudaStream_t st) {
    if (s.B <= 0 || s.wnd <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)s.B * s.total() * s.total();
    const cudaError_t e = launch_k(octo_mask_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, s, tmask,
                                   wrist ? 1 : 0, mask);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void gather_rows_kernel(const float* __restrict__ src, const int* __restrict__ slot, int n_rows,
                                   long long n, float* __restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const long long total = (long long)n_rows * n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int b = static_cast<int>(i / n);
        dst[i] = src[(long long)slot[b] * n + (i - (long long)b * n)];
    }
}

cudaError_t gather_rows(const float* src, const int* slot, int n_rows, long long n, float* dst, cudaStream_t st) {
    if (n_rows <= 0 || n <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(gather_rows_kernel, (unsigned)grid_cap((long long)n_rows * n, 256, 148 * 4), 256,
                                   0, st, src, slot, n_rows, n, dst);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------- head
__global__ void silu_exact_kernel(float* __restrict__ x, long long n) {
    pdl_wait();
    pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        x[i] = __fdiv_rn(v, __fadd_rn(1.0f, libm_expf(-v)));
    }
}

// ------------------------------------------- activation + row quantization
// One CTA per row: v = act(x) (kAct* kinds of lm_ops, or kActSiluLibm for
// silu with the C library's expf), staged in shared memory, optionally written
// back, then quantize_act_i8 of the row (the scale and codes of quantize_rows):
// the activation and the next W8A8 layer's input quantization in one pass.
__device__ __forceinline__ float act_any(int kind, float v) {
    return kind == kActSiluLibm ? __fdiv_rn(v, __fadd_rn(1.0f, libm_expf(-v))) : act_eval(kind, v, 0.0f, false);
}

__global__ void __launch_bounds__(256) act_rows_q_kernel(int kind, float* __restrict__ x, int K, int keep,
                                                          int8_t* __restrict__ q, long long ldq,
                                                          float* __restrict__ scale) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float arow[];
    __shared__ float red[8];
    const long long row = blockIdx.x;
    float* xr = x + row * K;
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += 256) {
        const float v = act_any(kind, xr[k]);
        arow[k] = v;
        m = fmaxf(m, fabsf(v));
        if (keep) xr[k] = v;
    }
    m = block_max_256(m, red);
    const float sc = row_scale(m), inv = __fdiv_rn(1.0f, sc);
    int8_t* qr = q + row * ldq;
    for (long long k = threadIdx.x; k < ldq; k += 256) qr[k] = k < K ? q8(arow[k], inv) : 0;
    if (threadIdx.x == 0) scale[row] = sc;
}

cudaError_t act_rows_q(int kind, float* x, int M, int K, bool keep, int8_t* q, long long ldq, float* scale,
                       cudaStream_t st) {
    if (M <= 0 || K <= 0 || ldq < K || K > 12288) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * (size_t)K;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(act_rows_q_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    const cudaError_t e = launch_k(act_rows_q_kernel, (unsigned)M, 256, smem, st, kind, x, K, keep ? 1 : 0, q, ldq,
                                   scale);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------- head step tail
// One CTA (32 warps) per query: silu(h) -> eps = out_proj(.) with the exact
// fp32 dense_linear order per output (mm_block4 for outputs in whole blocks
// of 4, simd_dot for the rest; src/hal/avx2/gemm.cpp:33-122) -> the DDPM
// update of x -> the next step's score-net input row [cond | emb | x] and its
// int8 quantization. With x0 (the initial noise) instead of h: only the
// first input row (and sample = x0).
__device__ __forceinline__ float warp_dense_out(const float* __restrict__ xr, const float* __restrict__ wr, int K,
                                                bool block4) {
    const int lane = threadIdx.x & 31;
    float acc = 0.0f;
    int kend;
    if (block4) {
        const int K16 = K & ~15;
        if (lane < 16)
            for (int k = 0; k < K16; k += 16) acc = __fmaf_rn(xr[k + lane], wr[k + lane], acc);
        kend = K16;
        if (K - K16 >= 8) {
            if (lane < 8) acc = __fmaf_rn(xr[K16 + lane], wr[K16 + lane], acc);
            kend = K16 + 8;
        }
        acc = __fadd_rn(acc, __shfl_down_sync(0xFFFFFFFFu, acc, 8));
    } else {
        const int K32 = K & ~31;
        for (int k = 0; k < K32; k += 32) acc = __fmaf_rn(xr[k + lane], wr[k + lane], acc);
        kend = K32;
        for (; kend + 8 <= K; kend += 8)
            if (lane < 8) acc = __fmaf_rn(xr[kend + lane], wr[kend + lane], acc);
        const float a1 = __shfl_down_sync(0xFFFFFFFFu, acc, 8);
        const float a2 = __shfl_down_sync(0xFFFFFFFFu, acc, 16);
        const float a3 = __shfl_down_sync(0xFFFFFFFFu, acc, 24);
        acc = __fadd_rn(__fadd_rn(acc, a1), __fadd_rn(a2, a3));
    }
    float l[8];
    #pragma unroll
    for (int i = 0; i < 8; ++i) l[i] = __shfl_sync(0xFFFFFFFFu, acc, i);
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[1], l[5])),
                          __fadd_rn(__fadd_rn(l[2], l[6]), __fadd_rn(l[3], l[7])));
    if (block4)
        for (int k = kend; k < K; ++k) sum = __fmaf_rn(xr[k], wr[k], sum);
    else
        for (int k = kend; k < K; ++k) sum = __fadd_rn(sum, __fmul_rn(xr[k], wr[k]));
    return sum;
}

__global__ void __launch_bounds__(1024) octo_head_tail_kernel(OctoHeadTail a) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float hsm[];
    float* hs = hsm;                  // [H] silu(h)
    float* xs = hs + a.H;             // [FL] updated sample
    float* in = xs + a.FL;            // [IN] next input row
    __shared__ float red[32];
    const int b = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int IN = a.TD + a.E + a.FL;
    float* xb = a.sample + (long long)b * a.FL;
    if (a.h) {
        const float* hb = a.h + (long long)b * a.H;
        for (int k = tid; k < a.H; k += blockDim.x) hs[k] = __fdiv_rn(hb[k], __fadd_rn(1.0f, libm_expf(-hb[k])));
        __syncthreads();
        const int nb4 = a.FL - a.FL % 4;
        for (int n = warp; n < a.FL; n += blockDim.x >> 5) {
            float e = warp_dense_out(hs, a.W + (long long)n * a.H, a.H, n < nb4);
            e = a.bias ? __fadd_rn(e, a.bias[n]) : e;
            if (lane == 0) {
                const float zv = a.z ? a.z[(long long)b * a.z_stride + n] : 0.0f;
                const float v = __fmaf_rn(__fmaf_rn(-a.a2, e, xb[n]), a.a1, __fmul_rn(a.sb, zv));
                xs[n] = v < -a.max_action ? -a.max_action : v > a.max_action ? a.max_action : v;
            }
        }
        __syncthreads();
        for (int n = tid; n < a.FL; n += blockDim.x) xb[n] = xs[n];
    } else {
        for (int n = tid; n < a.FL; n += blockDim.x) {
            xs[n] = a.x0[(long long)b * a.FL + n];
            xb[n] = xs[n];
        }
        __syncthreads();
    }
    if (!a.cond_next) return;
    float m = 0.0f;
    for (int c = tid; c < IN; c += blockDim.x) {
        const float v = c < a.TD ? a.cond_next[c] : c < a.TD + a.E ? a.emb[(long long)b * a.E + (c - a.TD)]
                                                                   : xs[c - a.TD - a.E];
        in[c] = v;
        m = fmaxf(m, fabsf(v));
        if (a.in_f32) a.in_f32[(long long)b * IN + c] = v;
    }
    if (!a.q) return;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    #pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, off));
    const float sc = row_scale(m), inv = __fdiv_rn(1.0f, sc);
    int8_t* qr = a.q + (long long)b * a.ldq;
    for (long long c = tid; c < a.ldq; c += blockDim.x) qr[c] = c < IN ? q8(in[c], inv) : 0;
    if (tid == 0) a.qscale[b] = sc;
}

cudaError_t octo_head_tail(const OctoHeadTail& a, cudaStream_t st) {
    if (a.B <= 0 || a.FL <= 0 || (!a.h && !a.x0) || (a.h && (!a.W || a.H <= 0))) return cudaErrorInvalidValue;
    const size_t smem = sizeof(float) * ((size_t)a.H + a.FL + a.TD + a.E + a.FL);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(octo_head_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    const cudaError_t e = launch_k(octo_head_tail_kernel, (unsigned)a.B, 1024, smem, st, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t silu_exact(float* x, long long n, cudaStream_t st) {
    if (n <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(silu_exact_kernel, (unsigned)grid_cap(n, 256, 148 * 4), 256, 0, st, x, n);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void octo_head_input_kernel(const float* __restrict__ cond_t, int TD, const float* __restrict__ emb, int E,
                                       const float* __restrict__ x, int FL, int B, float* __restrict__ in) {
    pdl_wait();
    pdl_trigger();
    const int IN = TD + E + FL;
    const long long n = (long long)B * IN;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int b = static_cast<int>(i / IN), c = static_cast<int>(i - (long long)b * IN);
        in[i] = c < TD ? cond_t[c] : c < TD + E ? emb[(long long)b * E + (c - TD)] : x[(long long)b * FL + (c - TD - E)];
    }
}

cudaError_t octo_head_input(const float* cond_t, int TD, const float* emb, int E, const float* x, int FL, int B,
                            float* in, cudaStream_t st) {
    if (B <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)B * (TD + E + FL);
    const cudaError_t e = launch_k(octo_head_input_kernel, (unsigned)grid_cap(n, 256, 148 * 2), 256, 0, st, cond_t,
                                   TD, emb, E, x, FL, B, in);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void octo_ddpm_step_kernel(float* __restrict__ x, const float* __restrict__ eps,
                                      const float* __restrict__ z, long long z_stride, int B, int FL, float a1,
                                      float a2, float sb, float max_action) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * FL) return;
    const int b = i / FL, k = i - b * FL;
    const float zv = z ? z[(long long)b * z_stride + k] : 0.0f;
    const float v = __fmaf_rn(__fmaf_rn(-a2, eps[i], x[i]), a1, __fmul_rn(sb, zv));
    x[i] = v < -max_action ? -max_action : v > max_action ? max_action : v;
}

cudaError_t octo_ddpm_step(float* x, const float* eps, const float* z, long long z_stride, int B, int FL, float a1,
                           float a2, float sb, float max_action, cudaStream_t st) {
    if (B <= 0 || FL <= 0) return cudaErrorInvalidValue;
    const int n = B * FL;
    const cudaError_t e = launch_k(octo_ddpm_step_kernel, (unsigned)((n + 255) / 256), 256, 0, st, x, eps, z,
                                   z_stride, B, FL, a1, a2, sb, max_action);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void octo_actions_kernel(const float* __restrict__ x, int n, int A, const float* __restrict__ mean,
                                    const float* __restrict__ stdv, const float* __restrict__ mask, int unnormalize,
                                    float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int a = i % A;
    const float v = x[i];
    out[i] = (unnormalize && mask[a] > 0.0f) ? __fmaf_rn(v, stdv[a], mean[a]) : v;
}

cudaError_t octo_actions(const float* x, int B, int FL, int A, const float* mean, const float* stdv,
                         const float* mask, bool unnormalize, float* out, cudaStream_t st) {
    if (B <= 0 || FL <= 0 || A <= 0 || FL % A) return cudaErrorInvalidValue;
    const int n = B * FL;
    const cudaError_t e = launch_k(octo_actions_kernel, (unsigned)((n + 255) / 256), 256, 0, st, x, n, A, mean, stdv,
                                   mask, unnormalize ? 1 : 0, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace vsb
