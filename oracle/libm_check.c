/* TEST INFRASTRUCTURE ONLY: checks the library's restatement of the host C
 * library's float functions (vla_simd_b200/csrc/libm_f32.h, compiled here as
 * host C with -ffp-contract=off) against the host C library itself, bit
 * pattern by bit pattern. A NaN result matches any NaN. */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../vla_simd_b200/csrc/libm_f32.h"

static float host_mish(float v) {
    /* the reference's scalar tail, src/hal/common/eltwise.cpp:244-248 */
    const float sp = v > 20.0f ? v : log1pf(expf(v));
    return v * tanhf(sp);
}

static float pick(int fn, float x, int restated) {
    switch (fn) {
        case 0: return restated ? lf_expf(x) : expf(x);
        case 1: return restated ? lf_log1pf(x) : log1pf(x);
        case 2: return restated ? lf_expm1f(x) : expm1f(x);
        case 3: return restated ? lf_tanhf(x) : tanhf(x);
        default: return restated ? lf_mish(x) : host_mish(x);
    }
}

/* Number of bit patterns in [start, start + count) (wrapping at 2^32) where
 * function `fn` (0 expf, 1 log1pf, 2 expm1f, 3 tanhf, 4 the Mish tail) differs
 * from the host library; *first_bad receives the first such pattern. */
uint64_t or_libm_mismatches(int fn, uint32_t start, uint64_t count, uint32_t* first_bad) {
    uint64_t bad = 0;
    for (uint64_t i = 0; i < count; ++i) {
        const uint32_t b = start + (uint32_t)i;
        float x;
        memcpy(&x, &b, 4);
        const float r = pick(fn, x, 1), h = pick(fn, x, 0);
        uint32_t rb, hb;
        memcpy(&rb, &r, 4);
        memcpy(&hb, &h, 4);
        if (rb != hb && !(r != r && h != h)) {
            if (!bad && first_bad) *first_bad = b;
            ++bad;
        }
    }
    return bad;
}

/* The restated functions themselves, for the device comparison. */
void or_libm_eval(int fn, const float* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) y[i] = pick(fn, x[i], 1);
}
