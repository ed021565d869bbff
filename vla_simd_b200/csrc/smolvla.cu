// SmolVLA kernels around the shared GEMM / LayerNorm / RMSNorm / attention
// ones: the C ABI's resize-with-pad, SigLIP's patch extraction, position add
// and pixel shuffle, the prefix sequence and its masks / positions, RoPE from
// a host-computed table, the SwiGLU gate (with the next layer's row
// quantization), the action expert's K/V scatter and the flow-matching
// update. Every formula is the reference's, with the contractions its
// -ffp-contract=fast build makes (read from the compiled reference).
#include "sm100.cuh"
#include "launch.cuh"
#include "smolvla.h"

#include <cfloat>

namespace vsb {

// ------------------------------------------------------------ resize + pad
// src/preprocess/image.cpp:12-51: bilinear over the source in double, the
// resized image at the bottom-right of an S x S canvas of -1, CHW, [-1, 1].
__global__ void smolvla_resize_kernel(const uint8_t* __restrict__ src, int F, int h, int w, SmolvlaResize g,
                                      float* __restrict__ dst) {
    pdl_wait();
    pdl_trigger();
    const int S = g.S;
    const long long per = (long long)3 * S * S;
    const long long n = (long long)F * per;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int f = static_cast<int>(i / per);
        const long long r = i - (long long)f * per;
        const int c = static_cast<int>(r / ((long long)S * S));
        const int yx = static_cast<int>(r - (long long)c * S * S);
        const int y = yx / S, x = yx - y * S;
        const int oy = y - g.pad_h, ox = x - g.pad_w;
        float out = -1.0f;
        if (oy >= 0 && ox >= 0) {
            const uint8_t* s = src + (long long)f * h * w * 3;
            const double fy = __fma_rn(static_cast<double>(oy) + 0.5, g.sy, -0.5);
            int y0 = static_cast<int>(floor(fy));
            const double dy = fy - y0;
            const int y1 = min(y0 + 1, h - 1);
            y0 = max(y0, 0);
            const double fx = __fma_rn(static_cast<double>(ox) + 0.5, g.sx, -0.5);
            int x0 = static_cast<int>(floor(fx));
            const double dx = fx - x0;
            const int x1 = min(x0 + 1, w - 1);
            x0 = max(x0, 0);
            const double p00 = s[((long long)y0 * w + x0) * 3 + c], p01 = s[((long long)y0 * w + x1) * 3 + c];
            const double p10 = s[((long long)y1 * w + x0) * 3 + c], p11 = s[((long long)y1 * w + x1) * 3 + c];
            const double row0 = __fma_rn(p00, 1.0 - dx, __dmul_rn(p01, dx));
            const double row1 = __fma_rn(p10, 1.0 - dx, __dmul_rn(p11, dx));
            const double v = __fma_rn(row0, 1.0 - dy, __dmul_rn(row1, dy));
            out = static_cast<float>(__fma_rn(__ddiv_rn(v, 255.0), 2.0, -1.0));
        }
        dst[i] = out;
    }
}

cudaError_t smolvla_resize(const uint8_t* src, int F, int h, int w, const SmolvlaResize& g, float* dst,
                           cudaStream_t st) {
    if (F <= 0 || h <= 0 || w <= 0 || g.S <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)F * 3 * g.S * g.S;
    const cudaError_t e = launch_k(smolvla_resize_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, src, F, h,
                                   w, g, dst);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------- patches, shuffle
// extract_patches (src/hal/common/conv.cpp:179-190): patch (ph, pw) -> row of
// (ic, kh, kw) values.
__global__ void smolvla_patches_kernel(const float* __restrict__ pix, int F, int S, int P, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int grid = S / P, pd = 3 * P * P;
    const long long n = (long long)F * grid * grid * pd;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / pd;
        const int e = static_cast<int>(i - row * pd);
        const int f = static_cast<int>(row / (grid * grid));
        const int p = static_cast<int>(row - (long long)f * grid * grid);
        const int ph = p / grid, pw = p - ph * grid;
        const int ic = e / (P * P), k = e - ic * P * P, kh = k / P, kw = k - kh * P;
        out[i] = pix[(((long long)f * 3 + ic) * S + (ph * P + kh)) * S + (pw * P + kw)];
    }
}

cudaError_t smolvla_patches(const float* pix, int F, int S, int P, float* out, cudaStream_t st) {
    if (F <= 0 || P <= 0 || S % P) return cudaErrorInvalidValue;
    const long long n = (long long)F * 3 * S * S;
    const cudaError_t e = launch_k(smolvla_patches_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, pix, F, S,
                                   P, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void add_rows_mod_kernel(float* __restrict__ x, long long M, int H, const float* __restrict__ add, int R) {
    pdl_wait();
    pdl_trigger();
    const long long n = M * H;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / H;
        const int c = static_cast<int>(i - r * H);
        x[i] = __fadd_rn(x[i], add[(r % R) * H + c]);
    }
}

cudaError_t add_rows_mod(float* x, long long M, int H, const float* add, int R, cudaStream_t st) {
    if (M <= 0 || H <= 0 || R <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(add_rows_mod_kernel, (unsigned)grid_cap(M * H, 256, 148 * 8), 256, 0, st, x, M, H,
                                   add, R);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// SigLIP connector pixel shuffle (src/models/smolvla/siglip_vision.cpp:191-203):
// token (h2, w2) = concat over (dh, dw) of patch (h2*sf + dh, w2*sf + dw).
__global__ void pixel_shuffle_kernel(const float* __restrict__ h, int F, int side, int sf, int H,
                                     float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int g2 = side / sf, SD = H * sf * sf;
    const long long n = (long long)F * g2 * g2 * SD;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long tok = i / SD;
        const int e = static_cast<int>(i - tok * SD);
        const int f = static_cast<int>(tok / (g2 * g2));
        const int t = static_cast<int>(tok - (long long)f * g2 * g2);
        const int h2 = t / g2, w2 = t - h2 * g2;
        const int blk = e / H, c = e - blk * H;
        const int dh = blk / sf, dw = blk - dh * sf;
        const int src = (h2 * sf + dh) * side + (w2 * sf + dw);
        out[i] = h[((long long)f * side * side + src) * H + c];
    }
}

cudaError_t pixel_shuffle(const float* h, int F, int side, int sf, int H, float* out, cudaStream_t st) {
    if (F <= 0 || sf <= 0 || side % sf) return cudaErrorInvalidValue;
    const long long n = (long long)F * side * side * H;
    const cudaError_t e = launch_k(pixel_shuffle_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, h, F, side,
                                   sf, H, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// dst[b][r][c] = src[b][r][c] for r < rows, c < cols (batch / row strides in floats)
__global__ void copy_rows_kernel(const float* __restrict__ src, long long src_bs, long long src_ld, float* __restrict__ dst,
                                 long long dst_bs, long long dst_ld, int B, int rows, int cols) {
    pdl_wait();
    pdl_trigger();
    const long long n = (long long)B * rows * cols;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long br = i / cols;
        const int c = static_cast<int>(i - br * cols);
        const int b = static_cast<int>(br / rows), r = static_cast<int>(br - (long long)b * rows);
        dst[b * dst_bs + r * dst_ld + c] = src[b * src_bs + r * src_ld + c];
    }
}

cudaError_t copy_rows(const float* src, long long src_bs, long long src_ld, float* dst, long long dst_bs,
                      long long dst_ld, int B, int rows, int cols, cudaStream_t st) {
    if (B <= 0 || rows <= 0 || cols <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)B * rows * cols;
    const cudaError_t e = launch_k(copy_rows_kernel, (unsigned)grid_cap(n, 256, 148 * 4), 256, 0, st, src, src_bs,
                                   src_ld, dst, dst_bs, dst_ld, B, rows, cols);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------ prefix
// SmolvlaModel::predict_normalized (src/models/smolvla/smolvla_model.cpp:180-196):
// [image tokens * sqrt(H) | bf16 token embeddings * sqrt(H) | state row].
__global__ void smolvla_prefix_kernel(SmolvlaPrefix p, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int np = p.n_img + p.n_lang + 1;
    const long long n = (long long)p.B * np * p.D;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / p.D;
        const int c = static_cast<int>(i - row * p.D);
        const int b = static_cast<int>(row / np), j = static_cast<int>(row - (long long)b * np);
        float v;
        if (j < p.n_img) {
            v = __fmul_rn(p.img[((long long)b * p.n_img + j) * p.D + c], p.sq);
        } else if (j < p.n_img + p.n_lang) {
            const int id = p.tokens[(long long)b * p.n_lang + (j - p.n_img)];
            const uint16_t e = p.emb[(long long)id * p.D + c];
            v = __fmul_rn(__uint_as_float(static_cast<unsigned int>(e) << 16), p.sq);
        } else {
            v = p.state_row[(long long)b * p.D + c];
        }
        out[i] = v;
    }
}

cudaError_t smolvla_prefix(const SmolvlaPrefix& p, float* out, cudaStream_t st) {
    if (p.B <= 0 || p.D <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)p.B * (p.n_img + p.n_lang + 1) * p.D;
    const cudaError_t e = launch_k(smolvla_prefix_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, p, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// state (raw - mean) / (std + eps) into [B][msd] (zeros past real_state_dim)
__global__ void smolvla_state_kernel(const float* __restrict__ raw, int B, int sd, int msd, const float* __restrict__ mean,
                                     const float* __restrict__ stdv, float eps, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * msd) return;
    const int b = i / msd, k = i - b * msd;
    out[i] = k < sd ? __fdiv_rn(__fsub_rn(raw[b * sd + k], mean[k]), __fadd_rn(stdv[k], eps)) : 0.0f;
}

cudaError_t smolvla_state(const float* raw, int B, int sd, int msd, const float* mean, const float* stdv, float eps,
                          float* out, cudaStream_t st) {
    if (B <= 0 || sd <= 0 || msd < sd) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(smolvla_state_kernel, (unsigned)((B * msd + 255) / 256), 256, 0, st, raw, B, sd,
                                   msd, mean, stdv, eps, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Prefix-LM mask, positions and the denoise masks (smolvla_model.cpp:198-225):
// pad = lang_mask for language tokens, 1 otherwise; att = 1 only for the state
// token; pmask[i][j] = att(j) <= att(i) && pad[i] && pad[j]; pos = cumsum(pad) - 1;
// dmask[i][j < np] = pad[j], dmask[i][np + j] = j <= i; pos_full[i] =
// sum(pad) + i; the cross-attention mask is dmask's prefix columns and the
// rebased positions pos_full - min(pos_full) (action_expert.cpp:356-363).
__global__ void smolvla_masks_kernel(const int* __restrict__ lang_mask, SmolvlaMaskArgs a) {
    pdl_wait();
    pdl_trigger();
    const int np = a.n_img + a.n_lang + 1, SK = np + a.C;
    const int b = blockIdx.y;
    const int* lm = lang_mask + (long long)b * a.n_lang;
    auto pad = [&](int j) { return (j < a.n_img || j >= a.n_img + a.n_lang) ? 1 : (lm[j - a.n_img] != 0 ? 1 : 0); };
    const long long n_pm = (long long)np * np, n_dm = (long long)a.C * SK;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_pm + n_dm;
         i += (long long)gridDim.x * blockDim.x) {
        if (i < n_pm) {
            const int qi = static_cast<int>(i / np), kj = static_cast<int>(i - (long long)qi * np);
            const int att_i = qi >= np - 1, att_j = kj >= np - 1;
            a.pmask[(long long)b * n_pm + i] = (att_j <= att_i && pad(qi) && pad(kj)) ? 0.0f : -FLT_MAX;
        } else {
            const long long r = i - n_pm;
            const int qi = static_cast<int>(r / SK), kj = static_cast<int>(r - (long long)qi * SK);
            const float v = kj < np ? (pad(kj) ? 0.0f : -FLT_MAX) : (kj - np <= qi ? 0.0f : -FLT_MAX);
            a.dmask[(long long)b * n_dm + r] = v;
            if (kj < np) a.cmask[((long long)b * a.C + qi) * np + kj] = v;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        int c = 0;
        for (int j = 0; j < np; ++j) {
            c += pad(j);
            a.pos[(long long)b * np + j] = c - 1;
        }
        for (int i = 0; i < a.C; ++i) {
            a.pos_full[(long long)b * a.C + i] = c + i;
            a.pos_rebased[(long long)b * a.C + i] = i;   // pos_full - min(pos_full)
        }
    }
}

cudaError_t smolvla_masks(const int* lang_mask, const SmolvlaMaskArgs& a, cudaStream_t st) {
    if (a.B <= 0 || a.C <= 0 || a.B > 65535) return cudaErrorInvalidValue;
    const int np = a.n_img + a.n_lang + 1;
    const long long n = (long long)np * np + (long long)a.C * (np + a.C);
    const cudaError_t e = launch_k(smolvla_masks_kernel, dim3((unsigned)grid_cap(n, 256, 64), a.B), 256, 0, st,
                                   lang_mask, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------------ RoPE
// rope_neox (src/hal/common/norms.cpp:31-61) with the per-position cos / sin
// of the reference's double recurrence precomputed on the host (table
// [max_pos + 1][half][2]); the rotation in double with the reference build's
// contractions: v[i] = fma(x0, c, -(x1*s)), v[i+half] = fma(x0, s, x1*c).
__global__ void rope_table_kernel(float* __restrict__ x, long long ld, long long rows, int n_heads, int hd,
                                  const int* __restrict__ pos, const double* __restrict__ table, int max_pos,
                                  int rows_per_pos_group, int* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const int half = hd / 2;
    const long long n = rows * n_heads * half;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / (n_heads * half);
        const int r = static_cast<int>(i - row * n_heads * half);
        const int hh = r / half, k = r - hh * half;
        const int p = pos[row / rows_per_pos_group * rows_per_pos_group + row % rows_per_pos_group];
        if (p < 0 || p > max_pos) {
            if (status) atomicExch(status, 1);
            continue;
        }
        const double c = table[((long long)p * half + k) * 2], s = table[((long long)p * half + k) * 2 + 1];
        float* v = x + row * ld + (long long)hh * hd;
        const double x0 = v[k], x1 = v[k + half];
        v[k] = static_cast<float>(__fma_rn(x0, c, -__dmul_rn(x1, s)));
        v[k + half] = static_cast<float>(__fma_rn(x0, s, __dmul_rn(x1, c)));
    }
}

cudaError_t rope_table(float* x, long long ld, long long rows, int n_heads, int hd, const int* pos,
                       const double* table, int max_pos, int* status, cudaStream_t st) {
    if (rows <= 0 || n_heads <= 0 || hd <= 0 || hd % 2) return cudaErrorInvalidValue;
    const long long n = rows * n_heads * (hd / 2);
    const cudaError_t e = launch_k(rope_table_kernel, (unsigned)grid_cap(n, 256, 148 * 8), 256, 0, st, x, ld, rows,
                                   n_heads, hd, pos, table, max_pos, 1, status);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// The expert's suffix K / V of B queries: kv [B*C][2KV] (k | v) -> KVf
// [B][SK][2KV] rows n_prefix.., the K half rotated by pos_full [B][C].
__global__ void kv_scatter_rope_kernel(const float* __restrict__ kv, int B, int C, int KV, int hd,
                                       const int* __restrict__ pos, const double* __restrict__ table, int max_pos,
                                       float* __restrict__ KVf, int n_prefix, int* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    const int SK = n_prefix + C, half = hd / 2, nh = KV / hd;
    const long long n = (long long)B * C * KV;   // K pairs: nh*half per row; V: KV per row
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long row = i / KV;
        const int e = static_cast<int>(i - row * KV);
        const int b = static_cast<int>(row / C), c = static_cast<int>(row - (long long)b * C);
        const float* src = kv + row * 2 * KV;
        float* dst = KVf + ((long long)b * SK + n_prefix + c) * 2 * KV;
        dst[KV + e] = src[KV + e];   // V
        if (e < nh * half) {
            const int hh = e / half, k = e - hh * half;
            const int p = pos[row];
            if (p < 0 || p > max_pos) {
                if (status) atomicExch(status, 1);
                continue;
            }
            const double cs = table[((long long)p * half + k) * 2], sn = table[((long long)p * half + k) * 2 + 1];
            const double x0 = src[hh * hd + k], x1 = src[hh * hd + k + half];
            dst[hh * hd + k] = static_cast<float>(__fma_rn(x0, cs, -__dmul_rn(x1, sn)));
            dst[hh * hd + k + half] = static_cast<float>(__fma_rn(x0, sn, __dmul_rn(x1, cs)));
        }
    }
}

cudaError_t kv_scatter_rope(const float* kv, int B, int C, int KV, int hd, const int* pos, const double* table,
                            int max_pos, float* KVf, int n_prefix, int* status, cudaStream_t st) {
    if (B <= 0 || C <= 0 || KV <= 0 || hd <= 0 || hd % 2 || KV % hd) return cudaErrorInvalidValue;
    const long long n = (long long)B * C * KV;
    const cudaError_t e = launch_k(kv_scatter_rope_kernel, (unsigned)grid_cap(n, 256, 148 * 4), 256, 0, st, kv, B, C,
                                   KV, hd, pos, table, max_pos, KVf, n_prefix, status);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ---------------------------------------------------------------- SwiGLU
// silu_gate (src/hal/common/eltwise.cpp:24-57, its SIMD body) of gu [M][2F]
// (gate | up) -> out [M][F] (when set) and the row's int8 quantization (when q is set).
__global__ void __launch_bounds__(256) silu_gate_rows_kernel(const float* __restrict__ gu, int F,
                                                              float* __restrict__ out, int8_t* __restrict__ q,
                                                              long long ldq, float* __restrict__ scale) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float grow[];
    __shared__ float red[8];
    const long long row = blockIdx.x;
    const float* g = gu + row * 2 * F;
    float m = 0.0f;
    for (int k = threadIdx.x; k < F; k += 256) {
        const float v = act_eval(kActSiluGate, g[k], g[F + k], false);
        if (q) grow[k] = v;
        if (out) out[row * F + k] = v;
        m = fmaxf(m, fabsf(v));
    }
    if (!q) return;
    m = block_max_256(m, red);
    const float sc = row_scale(m), inv = __fdiv_rn(1.0f, sc);
    int8_t* qr = q + row * ldq;
    for (long long k = threadIdx.x; k < ldq; k += 256) qr[k] = k < F ? q8(grow[k], inv) : 0;
    if (threadIdx.x == 0) scale[row] = sc;
}

cudaError_t silu_gate_rows(const float* gu, int M, int F, float* out, int8_t* q, long long ldq, float* scale,
                           cudaStream_t st) {
    if (M <= 0 || F <= 0 || (q && ldq < F) || F > 12288) return cudaErrorInvalidValue;
    const size_t smem = q ? sizeof(float) * (size_t)F : 0;
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        const cudaError_t e = cudaFuncSetAttribute(silu_gate_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)smem);
        if (e != cudaSuccess) return e;
        configured = smem;
    }
    const cudaError_t e = launch_k(silu_gate_rows_kernel, (unsigned)M, 256, smem, st, gu, F, out, q, ldq, scale);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// ------------------------------------------------------------ flow step
// action_time = [action_emb | time_emb] per row (action_expert.cpp:197-203)
__global__ void concat_time_kernel(const float* __restrict__ aemb, const float* __restrict__ te, long long M, int EH,
                                   float* __restrict__ at) {
    pdl_wait();
    pdl_trigger();
    const long long n = M * 2 * EH;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / (2 * EH);
        const int c = static_cast<int>(i - r * 2 * EH);
        at[i] = c < EH ? aemb[r * EH + c] : te[c - EH];
    }
}

cudaError_t concat_time(const float* aemb, const float* te, long long M, int EH, float* at, cudaStream_t st) {
    if (M <= 0 || EH <= 0) return cudaErrorInvalidValue;
    const cudaError_t e = launch_k(concat_time_kernel, (unsigned)grid_cap(M * 2 * EH, 256, 148 * 4), 256, 0, st, aemb,
                                   te, M, EH, at);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// The real-time-chunking guidance and the Euler step (action_expert.cpp:372-386):
// v -= gw * ((prev - (x - time*v)) * w[r]) as fma(-d, gw, v) with x - time*v =
// fma(-time, v, x); then x = fma(dt, v, x).
__global__ void flow_update_kernel(float* __restrict__ x, float* __restrict__ v, int B, int C, int MAD,
                                   const float* __restrict__ prev, const float* __restrict__ w, float time,
                                   const float* __restrict__ gw_ptr, float dt) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * C * MAD) return;
    float vt = v[i];
    const float xi = x[i];
    if (prev) {
        const float gw = *gw_ptr;
        const int b = i / (C * MAD), r = (i / MAD) % C;
        const float d = __fmul_rn(__fsub_rn(prev[i], __fmaf_rn(-time, vt, xi)), w[b * C + r]);
        vt = __fmaf_rn(-d, gw, vt);
        v[i] = vt;
    }
    x[i] = __fmaf_rn(dt, vt, xi);
}

cudaError_t flow_update(float* x, float* v, int B, int C, int MAD, const float* prev, const float* w, float time,
                        const float* gw, float dt, cudaStream_t st) {
    if (B <= 0 || C <= 0 || MAD <= 0 || (prev && (!w || !gw))) return cudaErrorInvalidValue;
    const int n = B * C * MAD;
    const cudaError_t e = launch_k(flow_update_kernel, (unsigned)((n + 255) / 256), 256, 0, st, x, v, B, C, MAD, prev,
                                   w, time, gw, dt);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// actions [B][C][A] = fma(x[b][c][a], std[a] + eps, mean[a]) for a < A of each
// [MAD]-wide row (smolvla_model.cpp:284-287), or x itself when !unnormalize;
// guide [B][C][MAD] = (prev - mean) / (std + eps) for rows < n_prev (zeros
// elsewhere) is the matching normalization of the RTC prefix.
__global__ void smolvla_actions_kernel(const float* __restrict__ x, int B, int C, int MAD, int A,
                                       const float* __restrict__ mean, const float* __restrict__ stdv, float eps,
                                       int unnormalize, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * C * A) return;
    const int a = i % A, rc = i / A;
    const float v = x[(long long)rc * MAD + a];
    out[i] = unnormalize ? __fmaf_rn(__fadd_rn(stdv[a], eps), v, mean[a]) : v;
}

cudaError_t smolvla_actions(const float* x, int B, int C, int MAD, int A, const float* mean, const float* stdv,
                            float eps, bool unnormalize, float* out, cudaStream_t st) {
    if (B <= 0 || C <= 0 || A <= 0 || A > MAD) return cudaErrorInvalidValue;
    const int n = B * C * A;
    const cudaError_t e = launch_k(smolvla_actions_kernel, (unsigned)((n + 255) / 256), 256, 0, st, x, B, C, MAD, A,
                                   mean, stdv, eps, unnormalize ? 1 : 0, out);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

__global__ void smolvla_guide_kernel(const float* __restrict__ prev, int B, int C, int MAD, int A, int n_prev,
                                     const float* __restrict__ mean, const float* __restrict__ stdv, float eps,
                                     float* __restrict__ guide) {
    pdl_wait();
    pdl_trigger();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * C * MAD) return;
    const int b = i / (C * MAD), r = (i / MAD) % C, j = i % MAD;
    float v = 0.0f;
    if (r < n_prev && j < A)
        v = __fdiv_rn(__fsub_rn(prev[((long long)b * n_prev + r) * A + j], mean[j]), __fadd_rn(stdv[j], eps));
    guide[i] = v;
}

cudaError_t smolvla_guide(const float* prev, int B, int C, int MAD, int A, int n_prev, const float* mean,
                          const float* stdv, float eps, float* guide, cudaStream_t st) {
    if (B <= 0 || C <= 0 || n_prev < 0 || n_prev > C) return cudaErrorInvalidValue;
    const int n = B * C * MAD;
    const cudaError_t e = launch_k(smolvla_guide_kernel, (unsigned)((n + 255) / 256), 256, 0, st, prev, B, C, MAD, A,
                                   n_prev, mean, stdv, eps, guide);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace vsb
