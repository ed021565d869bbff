// Host-side interface of the Diffusion Policy kernels (dp.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vsb {

// GroupNorm apply epilogues (bit flags, applied in this order after x*A + B):
enum : int {
    kGnMish = 1,   // v = mish(v)                     (DPConvBlock, src/models/diffusion/unet1d.cpp:185-191)
    kGnAdd = 2,    // v = v + res                     (residual of a block)
    kGnRelu = 4,   // v = v > 0 ? v : 0               (ResNet GroupNorm blocks)
};

// Observation frames in query order (b, s, c) [B*S*N][H][W][3] uint8 ->
// normalized, center-cropped fp32 NHWC in camera-major order:
// out frame o = c*(B*S) + b*S + s, [oh][ow][3]; per output frame absmax (float
// bits) into amax[(o / Fr) * run_stride + o % Fr] (the slots of the encoder
// run of Fr frames that reads it). mean/stdv [N][3] (DiffusionModel::preprocess,
// src/models/diffusion/diffusion_model.cpp:165-188).
cudaError_t dp_preprocess(const uint8_t* frames, int B, int S, int N, int H, int W, int top, int left, int oh, int ow,
                          const float* mean, const float* stdv, float eps, float* out, unsigned int* amax, int Fr,
                          long long run_stride, cudaStream_t st);

// GroupNorm statistics over F samples of x [F][npx][ld] (C channels):
// A[f][c] = inv*scale[c], B[f][c] = bias[c] - mean*inv*scale[c] per group
// (src/hal/common/conv.cpp:227-309; double accumulation).
cudaError_t gn_affine(const float* x, int F, int npx, int C, long long ld, int groups, float eps, const float* scale,
                      const float* bias, float* A, float* B, cudaStream_t st);

// out = epi(fma(x, A, B)) over F samples of [npx][C] (row stride ld for x,
// res and out); optional per-sample absmax of out into amax[f].
cudaError_t gn_apply(const float* x, const float* A, const float* B, float* out, int F, int npx, int C, long long ld,
                     int epi, const float* res, unsigned int* amax, cudaStream_t st);

// fp32 1D im2col of F samples x [F][T][ldx] (C channels) -> colf [F*Tout][k*C]
// (src/hal/common/conv.cpp:334-347), for the fp32 U-Net layers.
cudaError_t im2col1d_f32x(const float* x, int F, int T, int C, long long ldx, int k, int stride, int pad, int Tout,
                          float* colf, cudaStream_t st);

// cat [F][T][C1 + C2] = [a [F][T][C1] | b [F][T][C2]] per time step, with each
// row's absmax (float bits) into rowmax [F*T] when given. Rows longer than 256
// units (float4 units when C1, C2 and the pointers allow) are split over CTAs
// that meet by atomicMax: rowmax must be zero before the launch.
cudaError_t concat_channels(const float* a, int C1, const float* b, int C2, float* cat, int F, int T,
                            unsigned int* rowmax, cudaStream_t st);

// conv_transpose1d of F samples (x [F][T][Cin], W [Cin][k][Cout]) -> out [F][Tout][Cout],
// the reference's per-output accumulation order (src/hal/common/conv.cpp:349-395);
// optional per-row absmax of the output (atomicMax into rowmax [F*Tout], zeroed by the caller).
// Wt (optional): the same weights as [Cout][k][Cin], which the several-sample
// kernel streams. cudaErrorInvalidValue: a shape no kernel here takes.
cudaError_t conv_transpose1d_f(const float* x, const float* W, const float* Wt, const float* bias, float* out, int F,
                               int T, int Cin, int Cout, int k, int stride, int pad, unsigned int* rowmax,
                               cudaStream_t st);

// U-Net GroupNorm -> Mish -> epilogue over x [F][T][C] (out may alias x):
// kUgMish nothing more, kUgFilmScale fma(film[f][c], v, film[f][C + c]),
// kUgFilmBias v + film[f][c], kUgRes v + res (DPConvBlock + FiLM / residual,
// src/models/diffusion/unet1d.cpp:185-215). rowmax (optional, zeroed by the
// caller): per-time-step absmax of out (atomicMax, float bits).
enum : int { kUgMish = 0, kUgFilmScale = 1, kUgFilmBias = 2, kUgRes = 3 };
cudaError_t unet_gn(const float* x, int F, int T, int C, int groups, float eps, const float* scale,
                    const float* bias, int epi, const float* film, long long ld_film, const float* res, float* out,
                    unsigned int* rowmax, cudaStream_t st);

// Per-row int8 quantization of the 1D im2col of x [F][T][C] -> q [F*Tout][ldq],
// scale [F*Tout], from the per-time-step absmax rowmax [F][T] (null: rows of at
// most 64 values, scanned directly). The same codes and scales as quantize_act_i8
// of the fp32 im2col rows.
cudaError_t im2col1d_q8w(const float* x, int F, int T, int C, int k, int stride, int pad, int Tout,
                         const unsigned int* rowmax, int8_t* q, long long ldq, float* scale, cudaStream_t st);

// gm[(i*B + b)][CD] = mish([stepfeat[i] (D) | gcond[b] (CD - D)]) for i < n_steps:
// the cond encoder input of every denoising step (src/models/diffusion/unet1d.cpp:234-249).
// The last CD % 8 elements of each row are taken from tail [B][CD % 8]
// (mish's scalar libm tail, computed by the caller).
// tail[b][i] = the reference's scalar Mish of gcond[b][G - n + i] (the host
// library's expf / log1pf / tanhf restated), b < B, i < n.
cudaError_t dp_mish_tail(const float* gcond, int G, int n, int B, float* tail, cudaStream_t st);
cudaError_t dp_cond_input(const float* stepfeat, int n_steps, int D, const float* gcond, const float* tail, int B,
                          int CD, float* gm, cudaStream_t st);

// Step prologue: zero `n_zero` absmax slots, write the MIN_MAX-normalized state
// of every (b, s) into gcond [B][S*per_step] at column s*per_step, and copy the
// noise prior (noise [B][noise_stride] from offset 0, horizon*A values) into sample.
cudaError_t dp_prologue(unsigned int* zero, int n_zero, const float* state, int B, int S, int sd, const float* smin,
                        const float* smax, float eps, float* gcond, int per_step, const float* noise,
                        long long noise_stride, int HA, float* sample, cudaStream_t st);

// One reverse step in place on sample [n] from eps [n] (DPNoiseScheduler::step,
// src/models/diffusion/scheduler.cpp:76-117): DDIM when ddpm == 0, else DDPM
// with noise (stride between samples noise_stride, may be null).
struct DdStepConsts {
    double sqrt_ap, sqrt_bp;      // sqrt(alpha_bar_t), sqrt(1 - alpha_bar_t)
    double a, b;                  // DDIM: sqrt(alpha_bar_prev), sqrt(1 - alpha_bar_prev); DDPM: c0, c1
    double var;                   // DDPM noise scale (0 when t == 0)
    int ddpm, clip;
    double lo, hi;
};
cudaError_t dp_sched_step(float* sample, const float* eps, const float* noise, long long noise_stride, int B, int HA,
                          const DdStepConsts& c, cudaStream_t st);

// actions [B][n_act][A] = sample [B][horizon][A] rows start..start+n_act, MIN_MAX
// unnormalized when amin/amax are given (diffusion_model.cpp:258-271).
cudaError_t dp_actions(const float* sample, int B, int horizon, int A, int start, int n_act, const float* amin,
                       const float* amax, float eps, float* actions, cudaStream_t st);

// Spatial soft-argmax of F maps x [F][npx][C] with grid [npx][2] -> out [F][2C]
// (src/hal/common/conv.cpp:397-422).
cudaError_t spatial_softmax_f(const float* x, const float* grid, float* out, int F, int npx, int C, cudaStream_t st);

// v = max(v, 0) over rows [M] of N values with row stride ld.
cudaError_t relu_rows(float* x, int M, int N, long long ld, cudaStream_t st);

}  // namespace vsb
