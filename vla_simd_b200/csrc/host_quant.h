// Host-side load-time helper: the camera position table. (Weights are
// quantized on the device at load: upload_linear, conv_exec.cpp.)
#pragma once
#include <cstdint>

namespace vsb {

// ACT's 2D sinusoidal camera position embedding, [fh*fw][dim], the y half then
// the x half (ActTransformer::sinusoid_pos_2d, src/models/act/act_transformer.cpp:165-188).
void sinusoid_pos_2d_host(int fh, int fw, int dim, float* out);

}  // namespace vsb
