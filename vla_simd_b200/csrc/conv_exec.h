// Load-time layer upload and the int8 / fp32 2D convolution dispatch shared by
// the policy runtimes (ACT's and Diffusion Policy's ResNet backbones).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>

namespace vsb {

// A dense layer in whichever representation the int8 selection picked.
struct DevLinear {
    int N = 0, K = 0;
    bool int8 = false;
    int8_t* Wq = nullptr;      // [N][ldw] int8 (int8 layers)
    long long ldw = 0;
    float* wscale = nullptr;   // [N]
    float* W = nullptr;        // [N][K] fp32 (fp32 layers)
    float* bias = nullptr;     // [N]
};

struct DevConv {
    int cin = 0, cout = 0, k = 0, stride = 1, pad = 0;
    DevLinear lin;             // N = cout, K = k*k*cin in (ky, kx, ci) order
    // stride-2 convs over <= 4 channels (the stem): lin.Wq re-indexed for the
    // space-to-depth form, [cout][64 * ceil(k/2)]
    int8_t* Wq_s2d = nullptr;
};

// Device allocation callback of the owning runtime (bytes -> pointer, nullptr on failure).
using DevAlloc = std::function<void*(size_t)>;

// Upload W [N][K] (+ bias [N], zero when null). int8 follows nn::Linear::init_int8's
// conditions (src/nn/linear.cpp:66-67): N % 16 == 0 and K <= INT_MAX / (255 * 127);
// a layer that fails them stays fp32. Quantization is pack_weights_i8's.
bool upload_linear(DevLinear& l, const float* W, const float* b, int N, int K, bool int8, const DevAlloc& alloc,
                   int* n_int8 = nullptr);

// A k x k conv over cin channels (weights [cout][k][k][cin], bias may be null).
bool make_dev_conv(DevConv& c, const float* w, const float* b, int cout, int k, int cin, int stride, int pad,
                   bool int8, const DevAlloc& alloc, int* n_int8 = nullptr);

int conv_out_size(int in, int k, int stride, int pad);

// Scratch of one conv launch sequence (int8 im2col / quantized input and its
// per-row or per-frame scales; fp32 im2col for fp32 convs).
struct ConvScratch {
    int8_t* col = nullptr;
    float* col_scale = nullptr;
    float* col_f = nullptr;
};

// Element counts conv2d_dev needs in ConvScratch for F frames of H x W.
void conv_scratch_needs(const DevConv& c, int F, int H, int W, bool explicit_im2col, size_t* col_i8, size_t* col_f,
                        size_t* rows);

// conv2d over F NHWC frames [F][H][W][cin] -> [F][Ho][Wo][cout] with the GEMM
// epilogue `mode` (gemm_i8.h) and residual `res`. int8 layers quantize their
// input per frame with the scale of amax_in[f] (float bits, the producer's
// absmax tap) and TCPU_I8_CLIP `clip` (src/hal/common/conv.cpp:444-466);
// amax_out (optional) receives the output's per-frame absmax. Routes to the
// space-to-depth stem form, the implicit-GEMM conv (stride 1, cin % 64 == 0) or
// im2col + GEMM, unless explicit_im2col forces the last.
cudaError_t conv2d_dev(const DevConv& c, const float* in, int F, int H, int W, float* out, int mode,
                       const float* res, const unsigned int* amax_in, unsigned int* amax_out, float clip,
                       bool explicit_im2col, const ConvScratch& s, cudaStream_t st);

}  // namespace vsb
