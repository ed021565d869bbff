// vla_cuda_dense_linear_i8_noalloc: the W8A8 linear (per-token quantization +
// tensor-core GEMM) for callers that cannot allocate device memory at all -
// for example a robot's real-time control loop, where cudaMalloc/cudaFree may
// synchronize the device and take unbounded time, or a host framework that
// owns every byte of GPU memory through its own pool and gives plugins none.
// Such a caller still passes its inputs and outputs; the quantization scratch
// that vla_cuda_dense_linear_i8 takes from the caller lives here instead, in a
// fixed array in the GPU's global memory.
//
// The array is a file-scope static __device__ variable of this translation
// unit (its own .cu file, so the library's other kernels never see it). Every
// GPU that loads the library holds it until the process exits.
#include "../../include/vla_simd_cuda.h"

#include "gemm_i8.h"
#include "quant.h"

#include <cuda_runtime.h>

#include <climits>
#include <cstdio>
#include <mutex>

namespace {

// 2 MiB: the int8 copy of the activations (rows padded to 16 bytes) plus one
// fp32 scale per row. The ACT encoder's widest input (602 tokens x 3200) fits.
constexpr long long kScratchBytes = 2LL << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;

// A __device__ variable's address belongs to a CUDA context, not to a device
// number: after cudaDeviceReset, or under a non-primary context a host
// framework made current through the driver API, the same device has a new
// address. So the cache holds, per device, the context the address was looked
// up in, and a call under any other context looks it up again.
struct Cached {
    void* ctx = nullptr;
    void* addr = nullptr;
};
Cached g_cache[kMaxDevices];

using CtxGetCurrentFn = int (*)(void**);   // cuCtxGetCurrent: CUresult (CUcontext*)

CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(f);
    });
    return fn;
}

// Device address of g_noalloc_scratch in the current context. In host code the
// array's name is only a stand-in for the device object, so the real address
// is asked of the runtime (cudaGetSymbolAddress, which also creates the
// device's primary context on first use) with the device current; this set-up
// runs on the first call per device and context and is cached. It must not
// run while `st` is being captured into a graph: the lookup is refused then.
void* scratch_address(cudaStream_t st, cudaError_t* err) {
    int dev = 0;
    *err = cudaGetDevice(&dev);
    if (*err != cudaSuccess) return nullptr;
    if (dev < 0 || dev >= kMaxDevices) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    void* ctx = nullptr;
    CtxGetCurrentFn get = ctx_get_current();
    const bool have_ctx = get && get(&ctx) == 0 && ctx;
    std::lock_guard<std::mutex> lock(g_mu);
    Cached& c = g_cache[dev];
    if (have_ctx && c.addr && c.ctx == ctx) return c.addr;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cap) == cudaSuccess && cap != cudaStreamCaptureStatusNone) {
        std::fprintf(stderr,
                     "vla_cuda_dense_linear_i8_noalloc: the first call on a device (or in a new CUDA context) "
                     "looks up the scratch array's address and cannot run inside stream capture; call it once "
                     "before capturing\n");
        *err = cudaErrorStreamCaptureUnsupported;
        return nullptr;
    }
    void* p = nullptr;
    *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    if (have_ctx) {
        c.ctx = ctx;
        c.addr = p;
    } else if (get) {
        // cudaGetSymbolAddress made the primary context current: key the cache by it
        void* now = nullptr;
        if (get(&now) == 0 && now) {
            c.ctx = now;
            c.addr = p;
        }
    }
    return p;
}

}  // namespace

extern "C" int32_t vla_cuda_dense_linear_i8_noalloc(float* out, const float* x, const int8_t* Wq,
                                                    const float* wscale, const float* bias, int32_t seq, int32_t N,
                                                    int32_t K, int64_t ldw, void* stream) {
    if (!out || !x || !Wq || !wscale || seq <= 0 || N <= 0 || K <= 0 || K > INT_MAX / (255 * 127) || ldw < K)
        return VLA_ERR_ARG;
    const long long ld = (static_cast<long long>(K) + 15) & ~15LL;
    const long long xq_bytes = ((static_cast<long long>(seq) * ld) + 255) & ~255LL;
    if (xq_bytes + 4LL * seq > kScratchBytes) {
        std::fprintf(stderr,
                     "vla_cuda_dense_linear_i8_noalloc: %d x %d activations need %lld bytes of scratch; the static "
                     "array holds %lld\n",
                     seq, K, xq_bytes + 4LL * seq, kScratchBytes);
        return VLA_ERR_SHAPE;
    }
    cudaError_t e = cudaSuccess;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned char* base = static_cast<unsigned char*>(scratch_address(st, &e));
    if (!base) return VLA_ERR_DEVICE;
    int8_t* xq = reinterpret_cast<int8_t*>(base);
    float* ascale = reinterpret_cast<float*>(base + xq_bytes);
    // every byte of xq / ascale the GEMM reads is written by the quantizer first
    e = vsb::quantize_rows(x, K, nullptr, 0, seq, K, xq, ld, ascale, nullptr, 0, nullptr, st);
    if (e != cudaSuccess) return e == cudaErrorInvalidValue ? VLA_ERR_ARG : VLA_ERR_DEVICE;
    vsb::GemmI8Args a;
    a.A = xq;
    a.lda = ld;
    a.B = Wq;
    a.ldb = ldw;
    a.M = seq;
    a.N = N;
    a.K = K;
    a.out = out;
    a.ldo = N;
    a.ascale = ascale;
    a.wscale = wscale;
    a.bias = bias;
    e = vsb::gemm_i8(a, st);
    if (e != cudaSuccess) return e == cudaErrorInvalidValue ? VLA_ERR_ARG : VLA_ERR_DEVICE;
    return VLA_OK;
}
