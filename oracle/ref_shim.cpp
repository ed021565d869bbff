// TEST INFRASTRUCTURE ONLY. extern "C" entry points over the reference's own
// tcpu:: ops (vla.simd src/ops/quant_ops.h, lm_ops.h, conv_ops.h), compiled
// together with the reference's unmodified sources by oracle/Makefile into
// oracle/_ref/libvla_ref.so, so tests (ctypes) can call the real CPU kernels as
// the parity oracle and bench.py can time them as the CPU baseline. Nothing in
// the library links this.
#include "ops/conv_ops.h"
#include "ops/lm_ops.h"
#include "ops/quant_ops.h"
#include "nn/linear.h"

#include <cstdint>
#include <vector>

extern "C" {

int ref_int8_gemm_available(void) { return tcpu::int8_gemm_available() ? 1 : 0; }
int ref_i8_kpad(int K) { return tcpu::i8_kpad(K); }
unsigned long long ref_packed_i8_words(int N, int K) { return tcpu::packed_i8_words(N, K); }

void ref_pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int N, int K) {
    tcpu::pack_weights_i8(W, Wq, wscale, N, K);
}
void ref_quantize_act_i8(const float* x, int8_t* xq, float* ascale, int seq, int K) {
    tcpu::quantize_act_i8(x, xq, ascale, seq, K);
}
void ref_dense_linear_i8(float* out, const float* x, const int8_t* Wq, const float* wscale, const float* bias,
                         int seq, int N, int K, int8_t* xq, float* as) {
    tcpu::dense_linear_i8(out, x, Wq, wscale, bias, seq, N, K, xq, as);
}
void ref_dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                             const float* wscale, const float* bias, int seq, int N, int K) {
    tcpu::dense_linear_i8_pre(out, xq, ascale, Wq, wscale, bias, seq, N, K);
}
void ref_dense_linear_i8_ref(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                             const float* wscale, const float* bias, int seq, int N, int K) {
    tcpu::dense_linear_i8_ref(out, xq, ascale, Wq, wscale, bias, seq, N, K);
}
void ref_conv2d_i8(float* out, const float* x, const int8_t* Wq, const float* wscale, const float* bias, int H,
                   int W, int Cin, int Cout, int k, int stride, int pad) {
    std::vector<int8_t> scratch;
    tcpu::conv2d_i8(out, x, Wq, wscale, bias, H, W, Cin, Cout, k, stride, pad, scratch);
}
void ref_layernorm(float* out, const float* x, const float* w, const float* b, int seq, int hidden, float eps) {
    tcpu::layernorm(out, x, w, b, seq, hidden, eps);
}
void ref_gqa_attention_masked(float* out, const float* Q, const float* K, const float* V, int seq_q, int seq_k,
                              int n_q, int n_kv, int head_dim, float scale, const float* mask) {
    if (mask)
        tcpu::gqa_attention_masked(out, Q, K, V, seq_q, seq_k, n_q, n_kv, head_dim, scale, mask);
    else
        tcpu::gqa_attention_dense(out, Q, K, V, seq_q, seq_k, n_q, n_kv, head_dim, scale);
}
void ref_maxpool2d_relu(float* out, const float* x, int H, int W, int C, int k, int stride, int pad) {
    tcpu::maxpool2d_relu(out, x, H, W, C, k, stride, pad);
}
void ref_relu(float* x, int n) { tcpu::relu(x, n); }

// The reference's own layer object (src/nn/linear.cpp): init with fp32 W [N][K]
// as a projection (Role::Gemm), optionally init_int8(), then forward(). Returns
// 1 when the layer runs on the int8 kernel (init_int8 accepted it), else 0.
int ref_nn_linear_forward(const float* W, const float* bias, int N, int K, const float* x, int seq, float* out,
                          int int8) {
    tcpu::nn::Linear l;
    l.init(W, bias, N, K, tcpu::nn::Linear::Role::Gemm);
    const int q = int8 && l.init_int8() ? 1 : 0;
    l.forward(out, x, seq);
    return q;
}
void ref_dense_linear(float* out, const float* x, const float* W, const float* bias, int seq, int N, int K) {
    tcpu::dense_linear(out, x, W, bias, seq, N, K);
}

// lm_ops.h norms / positional / activations
void ref_rmsnorm(float* out, const float* x, const float* w, int seq, int hidden, float eps) {
    tcpu::rmsnorm(out, x, w, seq, hidden, eps);
}
void ref_rope_neox(float* x, const int* pos, int seq, int n_heads, int head_dim, float base) {
    tcpu::rope_neox(x, pos, seq, n_heads, head_dim, base);
}
void ref_silu_gate(float* out, const float* g, const float* u, int n) { tcpu::silu_gate(out, g, u, n); }
void ref_silu(float* x, int n) { tcpu::silu(x, n); }
void ref_gelu_tanh(float* x, int n) { tcpu::gelu_tanh(x, n); }
void ref_gelu_erf(float* x, int n) { tcpu::gelu_erf(x, n); }
void ref_mish(float* x, int n) { tcpu::mish(x, n); }

// conv_ops.h 1D / diffusion-policy ops
void ref_groupnorm(float* out, const float* x, const float* scale, const float* bias, int n_pixels, int C,
                   int groups, float eps, int fuse_relu) {
    tcpu::groupnorm(out, x, scale, bias, n_pixels, C, groups, eps, fuse_relu != 0);
}
void ref_spatial_softmax(float* out, const float* x, const float* grid, int n_pixels, int C) {
    tcpu::spatial_softmax(out, x, grid, n_pixels, C);
}
void ref_im2col1d(float* col, const float* x, int T, int Cin, int k, int stride, int pad, int Tout) {
    std::vector<float> v;
    tcpu::im2col1d(v, x, T, Cin, k, stride, pad, Tout);
    for (size_t i = 0; i < (size_t)Tout * k * Cin; ++i) col[i] = v[i];
}
void ref_conv_transpose1d(float* out, const float* x, const float* W, const float* bias, int T, int Cin, int Cout,
                          int k, int stride, int pad) {
    tcpu::conv_transpose1d(out, x, W, bias, T, Cin, Cout, k, stride, pad);
}

}  // extern "C"
