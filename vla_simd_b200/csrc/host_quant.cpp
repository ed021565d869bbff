#include "host_quant.h"

#include <cmath>
#include <vector>

namespace vsb {

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
