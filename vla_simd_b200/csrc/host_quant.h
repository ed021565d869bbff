// Host-side load-time helpers: weight quantization and the camera position table.
#pragma once
#include <cstdint>

namespace vsb {

// Per-row symmetric int8 quantization of W [N][K] into q [N][ldq] (zero past K)
// and scale [N]: pack_weights_i8's arithmetic (src/hal/common/gemm_i8.cpp:56-89)
// in this library's row-major device layout.
void quantize_rows_host(const float* W, int N, int K, int8_t* q, long long ldq, float* scale);

// ACT's 2D sinusoidal camera position embedding, [fh*fw][dim], the y half then
// the x half (ActTransformer::sinusoid_pos_2d, src/models/act/act_transformer.cpp:165-188).
void sinusoid_pos_2d_host(int fh, int fw, int dim, float* out);

}  // namespace vsb
