#include "host_quant.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>

namespace vsb {

void quantize_rows_host(const float* W, int N, int K, int8_t* q, long long ldq, float* scale) {
    for (int n = 0; n < N; ++n) {
        const float* wr = W + (long long)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; ++k) amax = std::max(amax, std::fabs(wr[k]));
        // an all-zero row gets scale 1 (its int8 row is zero either way)
        const float s = amax > 0.0f ? std::max(amax / 127.0f, std::numeric_limits<float>::min()) : 1.0f;
        const float inv = 1.0f / s;
        int8_t* qr = q + (long long)n * ldq;
        std::memset(qr, 0, static_cast<size_t>(ldq));
        for (int k = 0; k < K; ++k) {
            long r = std::lrint(wr[k] * inv);   // round to nearest even
            r = std::min(127L, std::max(-127L, r));
            qr[k] = static_cast<int8_t>(r);
        }
        scale[n] = s;
    }
}

void sinusoid_pos_2d_host(int fh, int fw, int dim, float* out) {
    const int half = dim / 2;
    const float two_pi = 6.283185307179586f;
    const float eps = 1e-6f;
    std::vector<float> inv_freq(half);
    for (int c = 0; c < half; ++c) inv_freq[c] = std::pow(10000.0f, (float)(2 * (c / 2)) / (float)half);
    for (int i = 0; i < fh; ++i) {
        const float yr = (float)(i + 1) / ((float)fh + eps) * two_pi;
        for (int j = 0; j < fw; ++j) {
            const float xr = (float)(j + 1) / ((float)fw + eps) * two_pi;
            float* o = out + (long long)(i * fw + j) * dim;
            for (int c = 0; c < half; ++c) {
                const float y = yr / inv_freq[c];
                const float x = xr / inv_freq[c];
                o[c] = (c & 1) ? std::cos(y) : std::sin(y);
                o[half + c] = (c & 1) ? std::cos(x) : std::sin(x);
            }
        }
    }
}

}  // namespace vsb
