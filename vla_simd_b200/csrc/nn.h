// Host-side interface of the non-GEMM kernels (nn.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vsb {

// out = LayerNorm(x) (may alias x). Optional fused per-row int8 outputs for the
// next GEMM: q1/s1 quantize (out + addend) (or out when addend is null), q2/s2
// quantize out. ldq = row stride of q1/q2.
cudaError_t layernorm(const float* x, float* out, const float* w, const float* b, int M, int H, float eps,
                      const float* addend, int8_t* q1, float* s1, int8_t* q2, float* s2, long long ldq,
                      cudaStream_t st);

// Multi-head attention, head_dim 64, rows of Q/K/V/O are tokens with the heads
// side by side (token-major, [seq][heads*64] with leading dimensions).
//
// Optional fused output (AttQuant): the per-row int8 quantization of O for the
// next W8A8 GEMM (quantize_rows' arithmetic over the n_q*64 columns of a row:
// absmax scale, q8, zero past them up to ldq). The attention CTAs of one query
// tile (one per head) count their arrivals in counters[tile]; the last one to
// finish quantizes the tile's rows and sets the counter back to zero, so no
// CTA waits on another and no quantizer launch follows.
struct AttQuant {
    int8_t* q = nullptr;                 // [rows][ldq]
    long long ldq = 0;
    float* scale = nullptr;              // [rows]
    unsigned int* counters = nullptr;    // zero before first use; left zero
    long long n_counters = 0;
    long long zq = 0, zs = 0;            // per-sequence strides of q (bytes) and scale (floats)
};
cudaError_t attention(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                      float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, int head_dim, float scale,
                      const float* mask, cudaStream_t st, const AttQuant* qz = nullptr);

// n independent sequences in one launch: sequence z reads Q + z*q, K + z*k,
// V + z*v, mask + z*mask and writes O + z*o (element strides, multiples of 4).
struct AttBatch {
    int n = 1;
    long long q = 0, k = 0, v = 0, o = 0, mask = 0;
};
cudaError_t attention_batched(const float* Q, long long ldq, const float* K, long long ldk, const float* V,
                              long long ldv, float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv,
                              int head_dim, float scale, const float* mask, const AttBatch& bs, cudaStream_t st,
                              const AttQuant* qz = nullptr);

// The tensor-core attention (attn_tc.cu): 3xTF32 tcgen05 MMAs for QK^T and PV,
// online softmax. Not bit-identical to the reference; attention_batched routes
// to it only when VLA_ATT_TC=1 (read once).
bool attention_tc_enabled();
cudaError_t attention_tc(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                         float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, float scale,
                         const float* mask, const AttBatch& bs, cudaStream_t st);

cudaError_t maxpool_relu(const float* x, float* out, int F, int H, int W, int C, int k, int stride, int pad,
                         int Ho, int Wo, unsigned int* amax, cudaStream_t st);

cudaError_t normalize_frames(const uint8_t* img, float* out, int F, long long npx, const float* mean,
                             const float* stdv, float eps, unsigned int* amax, cudaStream_t st);

cudaError_t linear_f32(const float* x, long long ldx, const float* W, const float* bias, float* out, long long ldo,
                       int M, int N, int K, const float* post_mul, const float* post_add, cudaStream_t st);

// First kernel of an ACT step: zero absmax slots, set the decoder state
// (init_f32, or zeros when null), copy the latent token, normalize the state.
cudaError_t act_prologue(unsigned int* zero_u32, int n_zero_u32, float* zero_f32, long long n_zero_f32,
                         const float* init_f32, float* tok0, const float* latent, int d, const float* state,
                         const float* mean, const float* stdv, float eps, float* state_n, int n, cudaStream_t st);

cudaError_t add_f32(const float* a, const float* b, float* out, long long n, cudaStream_t st);

}  // namespace vsb
