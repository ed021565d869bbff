/*
 * TEST INFRASTRUCTURE ONLY - the CPU oracle for the W8A8 path. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg use it, as the
 * checker / the timed CPU restatement; the library never links or calls it.
 *
 * A plain-C restatement of the reference's int8 algorithm (vla.simd,
 * src/hal/common/gemm_i8.cpp and src/hal/common/conv.cpp), each function citing
 * the lines it follows. Pinned against the reference itself: tests compare it
 * with oracle/_ref/libvla_ref.so (the reference's own sources, built by
 * oracle/Makefile) and with the committed fixtures in tests/golden/.
 *
 * Layouts here are row-major with explicit leading dimensions (the device
 * layout), plus the reference's panel packer for layout checks.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* gemm_i8.cpp:30  K rounded up to the 4-wide k-group */
int or_i8_kpad(int K) { return (K + 3) & ~3; }

/* gemm_i8.cpp:49-54  round to nearest even, clamp to +-127 */
static int8_t q8(float v) {
    long r = lrintf(v);
    if (r > 127) r = 127;
    if (r < -127) r = -127;
    return (int8_t)r;
}

/* gemm_i8.cpp:76 / :150 / :236  symmetric absmax scale with the FLT_MIN floor */
float or_row_scale(float amax) {
    if (!(amax > 0.0f)) return 1.0f;
    const float s = amax / 127.0f;
    return s > FLT_MIN ? s : FLT_MIN;
}

/* gemm_i8.cpp:209-244  per-row quantization: x [rows][K] -> q [rows][ldq]
 * (zero past K), scale [rows]. Also the per-output-row weight quantization of
 * pack_weights_i8 (:67-88), which is the same arithmetic. */
void or_quantize_rows(const float* x, int rows, int K, int8_t* q, long long ldq, float* scale) {
    for (int t = 0; t < rows; t++) {
        const float* xt = x + (size_t)t * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = fabsf(xt[k]);
            if (a > amax) amax = a;
        }
        const float s = or_row_scale(amax);
        const float inv = 1.0f / s;
        int8_t* qt = q + (size_t)t * ldq;
        for (int k = 0; k < K; k++) qt[k] = q8(xt[k] * inv);
        for (long long k = K; k < ldq; k++) qt[k] = 0;
        scale[t] = s;
    }
}

/* gemm_i8.cpp:56-89  the CPU panel layout [N/16][Kp/4][16][4] + int32 row sums */
void or_pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int N, int K) {
    const int Kp = or_i8_kpad(K), KG = Kp / 4;
    memset(Wq, 0, (size_t)N * Kp);
    int32_t* rowsum = (int32_t*)(Wq + (size_t)N * Kp);
    for (int n = 0; n < N; n++) {
        const float* wr = W + (size_t)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = fabsf(wr[k]);
            if (a > amax) amax = a;
        }
        const float s = or_row_scale(amax);
        wscale[n] = s;
        const float inv = 1.0f / s;
        int32_t sum = 0;
        for (int k = 0; k < K; k++) {
            const int8_t v = q8(wr[k] * inv);
            Wq[((size_t)((n / 16) * KG + k / 4) * 16 + (n % 16)) * 4 + (k % 4)] = v;
            sum += v;
        }
        rowsum[n] = sum;
    }
}

/* gemm_i8.cpp:270-277  the int32 accumulators the reference never exposes:
 * acc[m][n] = sum_k xq[m][k] * wq[n][k] */
void or_gemm_i8_acc(int32_t* acc, const int8_t* xq, long long ldx, const int8_t* wq, long long ldw,
                    int M, int N, int K) {
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            int32_t a = 0;
            const int8_t* xr = xq + (size_t)m * ldx;
            const int8_t* wr = wq + (size_t)n * ldw;
            for (int k = 0; k < K; k++) a += (int32_t)xr[k] * (int32_t)wr[k];
            acc[(size_t)m * N + n] = a;
        }
}

/* gemm_i8.cpp:262-281  dense_linear_i8_ref in row-major layout:
 * out = fma((float)acc * s_w[n], s_a[m], bias[n]) */
void or_dense_linear_i8_ref(float* out, const int8_t* xq, long long ldx, const float* ascale,
                            const int8_t* wq, long long ldw, const float* wscale, const float* bias,
                            int M, int N, int K) {
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            int32_t a = 0;
            const int8_t* xr = xq + (size_t)m * ldx;
            const int8_t* wr = wq + (size_t)n * ldw;
            for (int k = 0; k < K; k++) a += (int32_t)xr[k] * (int32_t)wr[k];
            const float prod = (float)a * wscale[n];   /* rounded before the fma */
            out[(size_t)m * N + n] = fmaf(prod, ascale[m], bias ? bias[n] : 0.0f);
        }
}

/* gemm_i8.cpp:177-207  fixed-scale quantization, fp32 clamp before rounding */
void or_quantize_span_i8(const float* x, int8_t* q, size_t n, float inv) {
    for (size_t i = 0; i < n; i++) {
        float v = x[i] * inv;
        if (v < -127.0f) v = -127.0f;
        if (v > 127.0f) v = 127.0f;
        q[i] = (int8_t)lrintf(v);
    }
}

/* conv.cpp:444-466  per-tensor scale: max(amax * clip / 127, FLT_MIN), 1 for zeros */
float or_tensor_scale(const float* x, size_t n, float clip) {
    float amax = 0.0f;
    for (size_t i = 0; i < n; i++) {
        const float a = fabsf(x[i]);
        if (a > amax) amax = a;
    }
    if (!(amax > 0.0f)) return 1.0f;
    const float s = amax * clip / 127.0f;
    return s > FLT_MIN ? s : FLT_MIN;
}

/* conv.cpp:468-526 + :108-156  conv2d_i8 on one NHWC frame: quantize the input
 * once with the per-tensor scale, int8 im2col in (ky, kx, ci) order, then the
 * W8A8 GEMM with that scale on every row. Wq [Cout][ldw] row-major. */
void or_conv2d_i8(float* out, const float* x, const int8_t* wq, long long ldw, const float* wscale,
                  const float* bias, int H, int W, int Cin, int Cout, int k, int stride, int pad, float clip,
                  int8_t* xq_scratch /* H*W*Cin */, int8_t* row_scratch /* k*k*Cin */) {
    const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
    const size_t nin = (size_t)H * W * Cin;
    const float s = or_tensor_scale(x, nin, clip);
    or_quantize_span_i8(x, xq_scratch, nin, 1.0f / s);
    const int K = k * k * Cin;
    for (int oy = 0; oy < Ho; oy++)
        for (int ox = 0; ox < Wo; ox++) {
            for (int ky = 0; ky < k; ky++)
                for (int kx = 0; kx < k; kx++) {
                    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
                    int8_t* dst = row_scratch + (size_t)(ky * k + kx) * Cin;
                    if (iy < 0 || iy >= H || ix < 0 || ix >= W) memset(dst, 0, (size_t)Cin);
                    else memcpy(dst, xq_scratch + ((size_t)iy * W + ix) * Cin, (size_t)Cin);
                }
            float* o = out + ((size_t)oy * Wo + ox) * Cout;
            for (int n = 0; n < Cout; n++) {
                int32_t a = 0;
                const int8_t* wr = wq + (size_t)n * ldw;
                for (int kk = 0; kk < K; kk++) a += (int32_t)row_scratch[kk] * (int32_t)wr[kk];
                o[n] = fmaf((float)a * wscale[n], s, bias ? bias[n] : 0.0f);
            }
        }
}
