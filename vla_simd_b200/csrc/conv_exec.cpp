// Layer upload and 2D convolution dispatch (see conv_exec.h). Host code only.
#include "conv_exec.h"

#include "f32.h"
#include "gemm_i8.h"
#include "quant.h"

#include <climits>
#include <vector>

namespace vsb {

namespace {

long long round16(long long v) { return (v + 15) & ~15LL; }

#define VSB_TRY(expr)                                  \
    do {                                               \
        const cudaError_t e_ = (expr);                 \
        if (e_ != cudaSuccess) return e_;              \
    } while (0)

}  // namespace

int conv_out_size(int in, int k, int stride, int pad) {
    const long long num = (long long)in + 2LL * pad - k;
    if (in <= 0 || stride <= 0 || num < 0) return 0;
    return static_cast<int>(num / stride + 1);
}

bool upload_linear(DevLinear& l, const float* W, const float* b, int N, int K, bool int8, const DevAlloc& alloc,
                   int* n_int8) {
    l.N = N;
    l.K = K;
    l.int8 = int8 && N % 16 == 0 && K > 0 && K <= INT_MAX / (255 * 127);
    l.bias = static_cast<float*>(alloc(sizeof(float) * N));
    if (!l.bias) return false;
    if (b) cudaMemcpy(l.bias, b, sizeof(float) * N, cudaMemcpyHostToDevice);
    else cudaMemset(l.bias, 0, sizeof(float) * N);
    if (l.int8) {
        // quantized on the device, by the same per-row kernel as the op API's
        // pack (pack_weights_i8's arithmetic, src/hal/common/gemm_i8.cpp:56-89):
        // the fp32 weights go up once to a staging buffer freed right after
        l.ldw = round16(K);
        l.Wq = static_cast<int8_t*>(alloc((size_t)N * l.ldw));
        l.wscale = static_cast<float*>(alloc(sizeof(float) * N));
        if (!l.Wq || !l.wscale) return false;
        float* staging = nullptr;
        if (cudaMalloc(&staging, sizeof(float) * (size_t)N * K) != cudaSuccess) return false;
        cudaError_t e = cudaMemcpy(staging, W, sizeof(float) * (size_t)N * K, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemset(l.Wq, 0, (size_t)N * l.ldw);
        if (e == cudaSuccess) e = quantize_rows(staging, K, nullptr, 0, N, K, l.Wq, l.ldw, l.wscale, nullptr, 0,
                                                nullptr, 0);
        if (e == cudaSuccess) e = cudaStreamSynchronize(0);
        cudaFree(staging);
        if (e != cudaSuccess) return false;
        if (n_int8) ++*n_int8;
    } else {
        l.W = static_cast<float*>(alloc(sizeof(float) * (size_t)N * K));
        if (!l.W) return false;
        cudaMemcpy(l.W, W, sizeof(float) * (size_t)N * K, cudaMemcpyHostToDevice);
    }
    return true;
}

bool make_dev_conv(DevConv& c, const float* w, const float* b, int cout, int k, int cin, int stride, int pad,
                   bool int8, const DevAlloc& alloc, int* n_int8) {
    c.cin = cin; c.cout = cout; c.k = k; c.stride = stride; c.pad = pad;
    if (!upload_linear(c.lin, w, b, cout, k * k * cin, int8, alloc, n_int8)) return false;
    if (c.lin.int8 && s2d_conv_supported(cin, k, stride)) {
        // the same int8 weights (quantization is deterministic), re-indexed
        // for the space-to-depth form of the conv
        std::vector<int8_t> wq((size_t)cout * c.lin.ldw), ws2d((size_t)cout * 64 * ((k + 1) / 2));
        if (cudaMemcpy(wq.data(), c.lin.Wq, wq.size(), cudaMemcpyDeviceToHost) != cudaSuccess) return false;
        s2d_repack_weights_host(wq.data(), cout, k, cin, c.lin.ldw, ws2d.data());
        c.Wq_s2d = static_cast<int8_t*>(alloc(ws2d.size()));
        if (!c.Wq_s2d) return false;
        cudaMemcpy(c.Wq_s2d, ws2d.data(), ws2d.size(), cudaMemcpyHostToDevice);
    }
    return true;
}

void conv_scratch_needs(const DevConv& c, int F, int H, int W, bool explicit_im2col, size_t* col_i8, size_t* col_f,
                        size_t* rows) {
    const int Ho = conv_out_size(H, c.k, c.stride, c.pad), Wo = conv_out_size(W, c.k, c.stride, c.pad);
    const size_t r = (size_t)F * Ho * Wo;
    size_t ci8 = 0, cf = 0;
    if (c.lin.int8) {
        if (c.Wq_s2d && !explicit_im2col) ci8 = (size_t)F * (Ho + (c.k + 1) / 2 - 1) * Wo * 64;
        else if (!explicit_im2col && conv_i8_implicit_supported(c.cin, c.k, c.stride)) ci8 = (size_t)F * H * W * c.cin;
        else ci8 = r * (size_t)c.lin.ldw;
    } else {
        cf = r * (size_t)c.lin.K;
    }
    *col_i8 = ci8;
    *col_f = cf;
    *rows = r > (size_t)F ? r : (size_t)F;
}

cudaError_t conv2d_dev(const DevConv& c, const float* in, int F, int H, int W, float* out, int mode,
                       const float* res, const unsigned int* amax_in, unsigned int* amax_out, float clip,
                       bool explicit_im2col, const ConvScratch& s, cudaStream_t st) {
    const int Ho = conv_out_size(H, c.k, c.stride, c.pad), Wo = conv_out_size(W, c.k, c.stride, c.pad);
    const int rows = F * Ho * Wo;
    if (c.lin.int8 && c.Wq_s2d && !explicit_im2col) {
        // stride-2 conv over a few channels as a stride-1 conv of ceil(k/2) x 1
        // taps over 64 space-to-depth channels (same int32 sums as im2col)
        const int kt = (c.k + 1) / 2;
        VSB_TRY(s2d_quantize_i8(in, F, H, W, c.cin, c.k, c.pad, Ho, Wo, amax_in, clip, s.col, s.col_scale, st));
        ConvI8Args a;
        a.x = s.col;
        a.F = F;
        a.H = Ho + kt - 1;
        a.W = Wo;
        a.C = 64;
        a.k = kt;
        a.kw = 1;
        a.pad = 0;
        a.Wq = c.Wq_s2d;
        a.ldw = 64LL * kt;
        a.N = c.cout;
        a.fscale = s.col_scale;
        a.wscale = c.lin.wscale;
        a.bias = c.lin.bias;
        a.out = out;
        a.res = res;
        a.amax = amax_out;
        a.mode = mode;
        a.static_weights = true;
        return conv_i8_implicit(a, st);
    }
    if (c.lin.int8 && !explicit_im2col && conv_i8_implicit_supported(c.cin, c.k, c.stride)) {
        // stride-1 convs over >= 64 channels: quantize the input once, then the
        // tensor-core GEMM gathers the taps itself (no im2col matrix)
        VSB_TRY(quantize_frames_i8(in, F, (long long)H * W * c.cin, amax_in, clip, s.col, s.col_scale, st));
        ConvI8Args a;
        a.x = s.col;
        a.F = F;
        a.H = H;
        a.W = W;
        a.C = c.cin;
        a.k = c.k;
        a.pad = c.pad;
        a.Wq = c.lin.Wq;
        a.ldw = c.lin.ldw;
        a.N = c.cout;
        a.fscale = s.col_scale;
        a.wscale = c.lin.wscale;
        a.bias = c.lin.bias;
        a.out = out;
        a.res = res;
        a.amax = amax_out;
        a.mode = mode;
        a.static_weights = true;
        return conv_i8_implicit(a, st);
    }
    if (c.lin.int8) {
        VSB_TRY(im2col_i8(in, F, H, W, c.cin, c.k, c.stride, c.pad, Ho, Wo, c.lin.ldw, amax_in, clip, s.col,
                          s.col_scale, st));
        GemmI8Args a;
        a.A = s.col;
        a.lda = c.lin.ldw;
        a.B = c.lin.Wq;
        a.ldb = c.lin.ldw;
        a.M = rows;
        a.N = c.cout;
        a.K = c.lin.K;
        a.out = out;
        a.ldo = c.cout;
        a.ascale = s.col_scale;
        a.wscale = c.lin.wscale;
        a.bias = c.lin.bias;
        a.res = res;
        a.ldr = c.cout;
        a.mode = mode;
        a.amax = amax_out;
        a.amax_rows = Ho * Wo;
        a.static_weights = true;
        return gemm_i8(a, st);
    }
    VSB_TRY(im2col_f32(in, F, H, W, c.cin, c.k, c.stride, c.pad, Ho, Wo, s.col_f, st));
    return gemm_f32(s.col_f, c.lin.K, c.lin.W, c.lin.K, c.lin.bias, out, c.cout, res, c.cout, rows, c.cout,
                    c.lin.K, mode, amax_out, Ho * Wo, st);
}

}  // namespace vsb
