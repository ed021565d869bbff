// Host-side interface of the W8A8 GEMM (gemm_i8.cu).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace vsb {

// Epilogue modes (bit flags). Without any flag: out = fma(acc*s_w, s_a, bias).
enum : int {
    kEpiRelu = 1,      // then v < 0 ? 0 : v            (tcpu::relu)
    kEpiAdd = 2,       // then out = res + v            (residual x += y)
    kEpiAddRelu = 4,   // then v = v + res; v > 0 ? v : 0 (ResNet block tail)
    kEpiAcc = 8,       // write the raw int32 accumulators instead
};

struct GemmI8Args {
    const int8_t* A = nullptr;   // [M][lda] quantized activations
    long long lda = 0;
    const int8_t* B = nullptr;   // [N][ldb] quantized weights (row n = output n)
    long long ldb = 0;
    int M = 0, N = 0, K = 0;
    void* out = nullptr;         // float [M][ldo] (int32 with kEpiAcc)
    long long ldo = 0;
    const float* ascale = nullptr;
    bool ascale_per_row = true;  // false: ascale[0] for every row
    const float* wscale = nullptr;
    const float* bias = nullptr;
    const float* res = nullptr;  // kEpiAdd / kEpiAddRelu operand, may alias out
    long long ldr = 0;
    unsigned int* amax = nullptr;  // optional: atomicMax of |out| bits into amax[m / amax_rows]
    int amax_rows = 1;
    int mode = 0;
    bool force_simt = false;     // route to the CUDA-core kernel (tests / odd strides)
    bool static_weights = false; // B/wscale/bias are load-time constants: the kernel may
                                 // fetch them before its predecessor in the stream ends
    // Optional split-K workspace for M <= 128 (one row tile) with a long K: K
    // is then split over independent CTAs whose int32 partial tiles are summed
    // by the last one to finish a tile (exact: integer sums). counters
    // [splitk_counters_n] must be zero when first used; every launch leaves them
    // zero again. Calls that may run at the same time need separate workspaces.
    int32_t* splitk_ws = nullptr;
    long long splitk_ws_elems = 0;
    unsigned int* splitk_counters = nullptr;
    int splitk_counters_n = 0;
    // Optional: the output as its per-row int8 quantization (quantize_rows'
    // arithmetic over the row's N values) instead of fp32, for a GEMM whose
    // only consumer is the next W8A8 GEMM: qout [M][ldq] (ldq == N), qscale
    // [M]; `out` is not written. Each CTA folds the |values| of its columns into
    // qamax [M] (float bits), the CTAs of one 128-row tile meet at a counter pair
    // in qsync [2 * row tiles], then each quantizes its columns with the row's
    // scale (a cooperative launch: the CTAs wait for one another). qamax and
    // qsync must be zero before the first use; every launch leaves them zero.
    // Calls that may run at the same time need separate qamax / qsync.
    int8_t* qout = nullptr;
    long long ldq = 0;
    float* qscale = nullptr;
    unsigned int* qamax = nullptr;
    unsigned int* qsync = nullptr;
    // Optional: A is the int8 im2col of a 1D conv input x [F][im_T][im_C],
    // computed inside the GEMM (the bytes and row scales im2col1d_q8w would
    // write: row m = output step m % im_Tout of sample m / im_Tout, K index
    // kt * im_C + c, each row quantized with the scale from its im_k input
    // rows' absmax in im_rowmax [F * im_T]). A / lda / ascale are then unused.
    // Only where gemm_i8_im2col_supported says so (else cudaErrorNotSupported).
    const float* im_x = nullptr;
    const unsigned int* im_rowmax = nullptr;
    int im_T = 0, im_C = 0, im_k = 0, im_stride = 1, im_pad = 0, im_Tout = 0;
};

// Whether gemm_i8 can compute the im2col A operand itself (GemmI8Args::im_x):
// at most 16 rows, K split across the SMs (the split-K workspace given), im_C
// a multiple of 16, K == im_k * im_C.
bool gemm_i8_im2col_supported(const GemmI8Args& a);

// Whether gemm_i8 runs a (with im_x and qout unset) as the warp-per-column
// GEMV: at most 4 rows, K a multiple of 16 and at most 2048, operands 16-byte
// aligned.
bool gemm_i8_takes_gemv(const GemmI8Args& a);

// Whether gemm_i8 can write the row-quantized output (GemmI8Args::qout) for
// this shape on this device: one wave of slab CTAs, N % 32 == 0, K <= 1024.
bool gemm_i8_rowq_supported(int M, int N, int K);

// Launch on `st`. Tensor-core path when lda/ldb/A/B are 16-byte aligned,
// otherwise the CUDA-core path (same results).
cudaError_t gemm_i8(const GemmI8Args& a, cudaStream_t st);

// Launch plan: output tile width BN (the B tensor map's box rows), the
// number of CTAs of a cluster that split K for one tile (1 = persistent
// kernel) and the depth of the shared-memory k-block ring.
struct GemmPlan {
    int bn = 128;
    int splits = 1;
    int stages = 4;
    bool global = false;   // split K over independent CTAs (needs GemmI8Args::splitk_ws)
};
GemmPlan gemm_i8_plan(int M, int N, int K);

// Pre-encoded variant for callers that keep tensor maps (box rows of tb = plan.bn).
bool make_tmap_i8_kmajor(CUtensorMap* map, const void* base, int rows, int K, long long ld, int box_rows);
cudaError_t gemm_i8_umma(const GemmI8Args& a, const CUtensorMap& ta, const CUtensorMap& tb, const GemmPlan& plan,
                         cudaStream_t st);

// Implicit-GEMM convolution, stride 1, on the same tensor-core kernels: the
// A operand is read straight from an int8 NHWC tensor by 4D TMA tile loads
// (one per filter tap and channel block; out-of-image taps read zeros), so no
// im2col matrix is written. x = int8 [F][H][W][C] quantized with the per-frame
// scales fscale[F]; weights [N][ldw] over K = k*k*C in (ky, kx, c) order;
// out = fp32 NHWC [F][Ho][Wo][N], the gemm_i8 epilogue (mode, residual of the
// same shape, absmax slot = frame). Requires C % 64 == 0. The filter is k x kw
// (kw = 0: square); weights' K order (ky, kx, c).
struct ConvI8Args {
    const int8_t* x = nullptr;
    int F = 0, H = 0, W = 0, C = 0, k = 0, pad = 0;
    int kw = 0;
    const int8_t* Wq = nullptr;
    long long ldw = 0;
    int N = 0;
    const float* fscale = nullptr;
    const float* wscale = nullptr;
    const float* bias = nullptr;
    float* out = nullptr;
    const float* res = nullptr;
    unsigned int* amax = nullptr;
    int mode = 0;
    bool static_weights = false;
};
bool conv_i8_implicit_supported(int C, int k, int stride);
cudaError_t conv_i8_implicit(const ConvI8Args& a, cudaStream_t st);

// Read and clear the device status word (0 = OK, see sm100.cuh).
int device_status_take();
// Device address of the status word on the current device (for asynchronous reads).
void* device_status_address();

}  // namespace vsb
