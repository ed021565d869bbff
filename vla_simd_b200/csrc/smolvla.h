// Host-side interface of the SmolVLA kernels (smolvla.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vsb {

// resize_with_pad geometry (src/preprocess/image.cpp:12-25), computed on the host
// in double exactly as the reference does.
struct SmolvlaResize {
    int S = 0, pad_w = 0, pad_h = 0;
    double sx = 0, sy = 0;
};
// F frames [F][h][w][3] uint8 -> [F][3][S][S] fp32 in [-1, 1].
cudaError_t smolvla_resize(const uint8_t* src, int F, int h, int w, const SmolvlaResize& g, float* dst,
                           cudaStream_t st);

// F images [F][3][S][S] -> patch rows [F * (S/P)^2][3*P*P] (src/hal/common/conv.cpp:179-190).
cudaError_t smolvla_patches(const float* pix, int F, int S, int P, float* out, cudaStream_t st);

// x[r][c] += add[r % R][c] over M rows of H values (the position embedding of every view).
cudaError_t add_rows_mod(float* x, long long M, int H, const float* add, int R, cudaStream_t st);

// h [F][side*side][H] -> [F * (side/sf)^2][H*sf*sf] (the SigLIP connector's pixel shuffle).
cudaError_t pixel_shuffle(const float* h, int F, int side, int sf, int H, float* out, cudaStream_t st);

// dst[b][r][c] = src[b][r][c] for r < rows, c < cols (batch and row strides in floats).
cudaError_t copy_rows(const float* src, long long src_bs, long long src_ld, float* dst, long long dst_bs,
                      long long dst_ld, int B, int rows, int cols, cudaStream_t st);

struct SmolvlaPrefix {
    int B = 0, n_img = 0, n_lang = 0, D = 0;
    float sq = 0;                       // sqrt(D) in float
    const float* img = nullptr;         // [B][n_img][D]
    const uint16_t* emb = nullptr;      // [vocab][D] bf16
    const int* tokens = nullptr;        // [B][n_lang]
    const float* state_row = nullptr;   // [B][D]
};
// prefix [B][n_img + n_lang + 1][D] (smolvla_model.cpp:180-196).
cudaError_t smolvla_prefix(const SmolvlaPrefix& p, float* out, cudaStream_t st);

// normalized state [B][msd]: (raw - mean) / (std + eps), zeros past sd.
cudaError_t smolvla_state(const float* raw, int B, int sd, int msd, const float* mean, const float* stdv, float eps,
                          float* out, cudaStream_t st);

struct SmolvlaMaskArgs {
    int B = 0, n_img = 0, n_lang = 0, C = 0;
    float* pmask = nullptr;      // [B][np][np]
    float* dmask = nullptr;      // [B][C][np + C]
    float* cmask = nullptr;      // [B][C][np]
    int* pos = nullptr;          // [B][np]
    int* pos_full = nullptr;     // [B][C]
    int* pos_rebased = nullptr;  // [B][C]
};
// The prefix-LM mask, positions and the expert's masks from lang_mask [B][n_lang].
cudaError_t smolvla_masks(const int* lang_mask, const SmolvlaMaskArgs& a, cudaStream_t st);

// NeoX RoPE in place on `rows` rows of x (row stride ld) with positions pos[row]
// and the table [max_pos + 1][hd/2][cos, sin]; a position outside the table
// sets *status and leaves its values.
cudaError_t rope_table(float* x, long long ld, long long rows, int n_heads, int hd, const int* pos,
                       const double* table, int max_pos, int* status, cudaStream_t st);

// kv [B*C][2KV] (k | v) -> KVf [B][n_prefix + C][2KV] rows n_prefix.., K rotated by pos [B*C].
cudaError_t kv_scatter_rope(const float* kv, int B, int C, int KV, int hd, const int* pos, const double* table,
                            int max_pos, float* KVf, int n_prefix, int* status, cudaStream_t st);

// SwiGLU gate of gu [M][2F] (gate | up): out [M][F] when set, and the rows'
// int8 quantization (q [M][ldq], scale [M]) when q is set.
cudaError_t silu_gate_rows(const float* gu, int M, int F, float* out, int8_t* q, long long ldq, float* scale,
                           cudaStream_t st);

// at [M][2EH] = [aemb [M][EH] | te [EH]]
cudaError_t concat_time(const float* aemb, const float* te, long long M, int EH, float* at, cudaStream_t st);

// RTC guidance (prev = the normalized guide [B][C][MAD], w [B][C], gw the
// step's guidance weight in device memory; all null without guidance) and the
// Euler step x += dt * v.
cudaError_t flow_update(float* x, float* v, int B, int C, int MAD, const float* prev, const float* w, float time,
                        const float* gw, float dt, cudaStream_t st);

// actions [B][C][A] from x [B][C][MAD], unnormalized with fma(x, std + eps, mean).
cudaError_t smolvla_actions(const float* x, int B, int C, int MAD, int A, const float* mean, const float* stdv,
                            float eps, bool unnormalize, float* out, cudaStream_t st);

// the normalized RTC guide [B][C][MAD] from prev [B][n_prev][A] (rows >= n_prev zero).
cudaError_t smolvla_guide(const float* prev, int B, int C, int MAD, int A, int n_prev, const float* mean,
                          const float* stdv, float eps, float* guide, cudaStream_t st);

}  // namespace vsb
