// The library's single CUDA translation unit: every kernel file is included
// here so the device status word (sm100.cuh) has one definition and no
// relocatable-device-code link step is needed.
#include "gemm_i8.cu"
#include "quant.cu"
#include "nn.cu"
#include "attn_tc.cu"
#include "f32.cu"
#include "lm_ops.cu"
#include "dp.cu"
#include "octo.cu"
#include "smolvla.cu"
