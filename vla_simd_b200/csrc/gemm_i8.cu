// W8A8 GEMM for sm_100a: int8 x int8 -> int32 on the 5th-generation tensor
// cores (tcgen05.mma kind::i8), accumulator in TMEM, operand tiles staged by TMA
// with the 128-byte swizzle, and the reference's delayed-scaling epilogue fused:
//
//   out[m,n] = fma((float)acc[m,n] * s_w[n], s_a[m], bias[n])      (then ReLU /
//              residual add / residual add + ReLU, optionally an absmax tap)
//
// which is, operation for operation, the epilogue of the reference's scalar
// oracle dense_linear_i8_ref (src/hal/common/gemm_i8.cpp:278) and of its AVX-VNNI
// kernel (src/hal/avx2/gemm_i8.cpp:101-104). Integer accumulation has no
// rounding, so the int32 sums equal the reference's exactly; the fp32 epilogue
// uses explicitly rounded intrinsics (__fmul_rn / __fmaf_rn) so nvcc cannot
// contract the multiply into the fma and the outputs are bit-identical.
//
// Layout (device side, this library's own): A = activations int8 [M][lda],
// B = weights int8 [N][ldb], both K-major (row-major over K); lda/ldb are
// multiples of 16 bytes (TMA stride rule). Bytes past K in a row are never read:
// the tensor maps' inner extent is K, so TMA zero-fills the k-tail.
//
// Persistent CTA = 320 threads (10 warps, specialized) looping over 128 x BN
// output tiles, accumulators double-buffered in TMEM so one tile's epilogue
// overlaps the next tile's loads and MMAs:
//   warp 0     lane 0: TMA producer (A and B k-blocks of 128 bytes, STAGES ring)
//   warp 1     TMEM allocation; lane 0: MMA issuer (4 x tcgen05.mma K=32 per
//              k-block), commits free ring slots back to the producer and
//              finally signals the epilogue
//   warps 2-9  epilogue: warp w reads TMEM lanes [32(w%4), +32) = tile rows
//              32(w%4).., the column chunks c with c % 2 == (w-2)/4, with
//              tcgen05.ld, applies the epilogue, stores fp32.
// Only the epilogue warps wait on the accumulator barrier; the producer and
// MMA warps never share a warp with a spinning waiter.
#include "sm100.cuh"
#include "launch.cuh"
#include "gemm_i8.h"

#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <cfloat>
#include <cstdio>
#include <mutex>

namespace vsb {

namespace {

constexpr int kBM = 128;          // UMMA M (one TMEM lane per tile row)
constexpr int kBK = 128;          // bytes of K per pipeline stage (one SW128 atom row)
constexpr int kUmmaK = 32;        // K per tcgen05.mma kind::i8
constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue

struct EpiParams {
    void* out;                    // float* (or int32_t* with kEpiAcc)
    long long ldo;
    const float* res;             // residual, read before out is written (may alias out)
    long long ldr;
    const float* ascale;          // per-row activation scale, index m * as_stride
    int as_stride;                // 1 = per row, 0 = one scale for every row
    const float* wscale;          // [N]
    const float* bias;            // [N] or null (then +0.0f, as the reference)
    unsigned int* amax;           // optional absmax tap (float bits), slot m / amax_rows
    int amax_rows;
    int mode;
    int M, N, K;
    int vec_ok;                   // 16-byte aligned rows: float4 stores
    int static_weights;           // B / wscale / bias never written by a kernel:
                                  // safe to read before the predecessor finishes
};

__device__ __forceinline__ float epi_value(int32_t acc, float ws, float as, float b, int mode,
                                           const float* resp) {
    float v = __fmaf_rn(__fmul_rn(__int2float_rn(acc), ws), as, b);
    if (mode & kEpiRelu) v = (v < 0.0f) ? 0.0f : v;                 // eltwise relu (eltwise.cpp:213-214)
    if (mode & kEpiAdd) v = __fadd_rn(*resp, v);                      // x[i] += y[i]
    if (mode & kEpiAddRelu) { v = __fadd_rn(v, *resp); v = v > 0.0f ? v : 0.0f; }  // resnet_backbone.cpp:293-295
    return v;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
w8a8_umma_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b,
                 const EpiParams p) {
    constexpr int kABytes = kBM * kBK;
    constexpr int kBBytes = BN * kBK;
    constexpr uint32_t kIdesc = idesc_s8s8_s32(kBM, BN);
    constexpr int kStg = 32 * 33;   // floats: one epilogue warp's 32 x 32 staging tile, padded
    constexpr int kEpiWarps = 8;

    extern __shared__ uint8_t smem_raw[];
    // SW128 tiles want 1024-byte alignment
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * kABytes;
    float* stg_all = reinterpret_cast<float*>(sB + STAGES * kBBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + kEpiWarps * kStg);
    uint64_t* empty = full + STAGES;
    uint64_t* acc_full = empty + STAGES;     // [2]: accumulator buffer ready for the epilogue
    uint64_t* acc_empty = acc_full + 2;      // [2]: epilogue done reading the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* s_consumed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_tn = (p.N + BN - 1) / BN;
    const int n_tiles = n_tn * ((p.M + kBM - 1) / kBM);
    const int nkb = (p.K + kBK - 1) / kBK;
    // weights that a predecessor kernel may still be writing: wait up front
    if (!p.static_weights) pdl_wait();

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiWarps); }
        *s_consumed = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above touched only on-chip state (and constant weights); let
    // the next kernel in the stream start its own setup.
    pdl_trigger();

    int issued = 0;
    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: tiles t = blockIdx.x, +gridDim.x, ...; one ring
            // of STAGES k-block slots shared across tiles. The weight halves of
            // the first slots go out before waiting for the predecessor kernel.
            const int pre = nkb < STAGES ? nkb : STAGES;
            {
                const int n0 = (blockIdx.x % n_tn) * BN;
                for (int kb = 0; kb < pre; ++kb) {
                    mbar_arrive_expect_tx(&full[kb], kABytes + kBBytes);
                    tma_load_2d(sB + kb * kBBytes, &tmap_b, &full[kb], kb * kBK, n0);
                }
            }
            pdl_wait();
            int it = 0;
            bool fail = false;
            for (int t = blockIdx.x; t < n_tiles && !fail; t += gridDim.x) {
                const int m0 = (t / n_tn) * kBM, n0 = (t % n_tn) * BN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (it < pre) {   // first tile's weights already in flight
                        tma_load_2d(sA + s * kABytes, &tmap_a, &full[s], kb * kBK, m0);
                    } else {
                        const int use = it / STAGES;   // > 0 unless the ring is longer than the first tile
                        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) { fail = true; break; }
                        mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
                        tma_load_2d(sA + s * kABytes, &tmap_a, &full[s], kb * kBK, m0);
                        tma_load_2d(sB + s * kBBytes, &tmap_b, &full[s], kb * kBK, n0);
                    }
                    issued = it + 1;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: tile i accumulates into TMEM buffer i % 2
            int it = 0, i = 0;
            bool fail = false;
            for (int t = blockIdx.x; t < n_tiles && !fail; t += gridDim.x, ++i) {
                const int buf = i & 1, ub = i >> 1;
                if (ub > 0 && !mbar_wait(&acc_empty[buf], (ub - 1) & 1)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * BN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1)) { fail = true; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kABytes);
                    const uint32_t b_addr = smem_u32(sB + s * kBBytes);
                    #pragma unroll
                    for (int k = 0; k < kBK / kUmmaK; ++k) {
                        umma_s8(d_tmem, sw128_kmajor_desc(a_addr + k * kUmmaK),
                                sw128_kmajor_desc(b_addr + k * kUmmaK), kIdesc, (kb | k) != 0);
                    }
                    umma_commit(&empty[s]);
                    *s_consumed = it + 1;
                }
                if (!fail) umma_commit(&acc_full[buf]);
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue (warps 2-9). Per 32-column chunk: phase A (thread = tile
        // row, as TMEM hands it out) turns the accumulators into
        // v = fma(acc*s_w, s_a, b) (or raw int32 bits) in this warp's staging
        // tile; phase B (coalesced) - lane l covers columns 4*(l%8)..+3 of rows
        // l/8 + 4i - adds the residual and stores, four whole 128-byte row
        // segments per instruction. Column scales and biases reach the lanes by
        // shuffle from one load per lane.
        const int quarter = warp & 3;   // TMEM lanes this warp may read: 32 * (warp id % 4)
        const int half = (warp - 2) >> 2;   // which column chunks: c % 2 == half
        float* stg = stg_all + (warp - 2) * kStg;
        const bool acc_mode = (p.mode & kEpiAcc) != 0;
        const int cq = (lane & 7) * 4;
        const int rq = lane >> 3;
        pdl_wait();   // activation scales / residual / output: predecessor data
        int i = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
            const int buf = i & 1;
            // warp-uniform: the tcgen05.ld and shuffles below need every lane
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[buf], (i >> 1) & 1))) break;
            tc_fence_after();
            const int m0 = (t / n_tn) * kBM, n0 = (t % n_tn) * BN;
            const int m_row = m0 + quarter * 32 + lane;
            const float as = m_row < p.M ? p.ascale[(long long)m_row * p.as_stride] : 0.0f;
            float tmax = 0.0f;
            #pragma unroll 1
            for (int c = half; c < BN / 32; c += 2) {
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, acc);
                const int ncol = n0 + c * 32 + lane;
                const float my_ws = ncol < p.N ? p.wscale[ncol] : 0.0f;
                const float my_b = (p.bias && ncol < p.N) ? p.bias[ncol] : 0.0f;
                tmem_ld_wait();
                if (n0 + c * 32 >= p.N) continue;            // warp-uniform
                #pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float ws = __shfl_sync(0xFFFFFFFFu, my_ws, j);
                    const float bj = __shfl_sync(0xFFFFFFFFu, my_b, j);
                    float v;
                    if (acc_mode) {
                        v = __int_as_float(static_cast<int32_t>(acc[j]));
                    } else {
                        v = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(acc[j])), ws), as, bj);
                        if (p.mode & kEpiRelu) v = (v < 0.0f) ? 0.0f : v;   // tcpu::relu (eltwise.cpp:213-214)
                    }
                    stg[lane * 33 + j] = v;
                }
                __syncwarp();
                const int n = n0 + c * 32 + cq;
                #pragma unroll
                for (int r8 = 0; r8 < 8; ++r8) {
                    const int r = rq + 4 * r8;
                    const int m = m0 + quarter * 32 + r;
                    if (m >= p.M || n >= p.N) continue;
                    float v[4] = {stg[r * 33 + cq], stg[r * 33 + cq + 1], stg[r * 33 + cq + 2], stg[r * 33 + cq + 3]};
                    const bool full4 = n + 4 <= p.N;
                    if (acc_mode) {
                        int32_t* o = static_cast<int32_t*>(p.out) + (long long)m * p.ldo + n;
                        #pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (n + e < p.N) o[e] = __float_as_int(v[e]);
                        continue;
                    }
                    if (p.mode & (kEpiAdd | kEpiAddRelu)) {
                        const float* rr = p.res + (long long)m * p.ldr + n;
                        float rv[4];
                        if (p.vec_ok && full4) {
                            const float4 tt = *reinterpret_cast<const float4*>(rr);
                            rv[0] = tt.x; rv[1] = tt.y; rv[2] = tt.z; rv[3] = tt.w;
                        } else {
                            #pragma unroll
                            for (int e = 0; e < 4; ++e) rv[e] = n + e < p.N ? rr[e] : 0.0f;
                        }
                        #pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (p.mode & kEpiAdd) v[e] = __fadd_rn(rv[e], v[e]);             // x[i] += y[i]
                            if (p.mode & kEpiAddRelu) {                                        // resnet_backbone.cpp:293-295
                                v[e] = __fadd_rn(v[e], rv[e]);
                                v[e] = v[e] > 0.0f ? v[e] : 0.0f;
                            }
                        }
                        if (p.amax) {
                            #pragma unroll
                            for (int e = 0; e < 4; ++e) stg[r * 33 + cq + e] = v[e];
                        }
                    }
                    float* o = static_cast<float*>(p.out) + (long long)m * p.ldo + n;
                    if (p.vec_ok && full4) {
                        *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
                    } else {
                        #pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (n + e < p.N) o[e] = v[e];
                    }
                }
                if (p.amax) {
                    // final values are back in the staging tile: per-row max, thread = row
                    __syncwarp();
                    #pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (n0 + c * 32 + j < p.N) tmax = fmaxf(tmax, fabsf(stg[lane * 33 + j]));
                }
                __syncwarp();
            }
            // this tile's TMEM buffer may be reused by the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
            if (p.amax) {
                // one atomic per warp when the warp's rows share a slot, else per row
                const bool row_ok = m_row < p.M;
                const unsigned key = row_ok ? static_cast<unsigned>(m_row / p.amax_rows) : 0xFFFFFFFFu;
                const unsigned k0 = __shfl_sync(0xFFFFFFFFu, key, 0);
                if (__all_sync(0xFFFFFFFFu, key == k0 || key == 0xFFFFFFFFu)) {
                    float wm = row_ok ? tmax : 0.0f;    // rows past M hold bias-only values
                    #pragma unroll
                    for (int off = 16; off > 0; off >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xFFFFFFFFu, wm, off));
                    if (lane == 0 && k0 != 0xFFFFFFFFu) atomicMax(&p.amax[k0], __float_as_uint(wm));
                } else if (row_ok) {
                    atomicMax(&p.amax[key], __float_as_uint(tmax));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // never leave the CTA with TMA writes still landing in its shared memory
        for (int kb = *s_consumed; kb < issued; ++kb)
            if (!mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1)) break;
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * BN);
    }
}

// ------------------------------------------------------------------ SIMT path
// Plain CUDA-core int8 GEMM (dp4a), used for operand strides TMA cannot
// describe (lda/ldb not a multiple of 16) and as an independent GPU cross-check
// of the tensor-core kernel in the tests. Same epilogue, bit for bit.
__global__ void w8a8_simt_kernel(const int8_t* __restrict__ A, long long lda,
                                 const int8_t* __restrict__ B, long long ldb, const EpiParams p) {
    pdl_wait();     // inputs come from the previous kernel in the stream
    pdl_trigger();
    const int n = blockIdx.y * blockDim.x + threadIdx.x;
    const int m = blockIdx.x;
    if (n >= p.N || m >= p.M) return;
    const int8_t* a = A + (long long)m * lda;
    const int8_t* b = B + (long long)n * ldb;
    int32_t acc = 0;
    int k = 0;
    if ((((uintptr_t)a | (uintptr_t)b) & 3) == 0) {
        for (; k + 4 <= p.K; k += 4)
            acc = __dp4a(*reinterpret_cast<const int*>(a + k), *reinterpret_cast<const int*>(b + k), acc);
    }
    for (; k < p.K; ++k) acc += static_cast<int32_t>(a[k]) * static_cast<int32_t>(b[k]);
    if (p.mode & kEpiAcc) {
        static_cast<int32_t*>(p.out)[(long long)m * p.ldo + n] = acc;
        return;
    }
    const float rv = p.res ? p.res[(long long)m * p.ldr + n] : 0.0f;
    const float v = epi_value(acc, p.wscale[n], p.ascale[(long long)m * p.as_stride],
                              p.bias ? p.bias[n] : 0.0f, p.mode, &rv);
    static_cast<float*>(p.out)[(long long)m * p.ldo + n] = v;
    if (p.amax) atomicMax(&p.amax[m / p.amax_rows], __float_as_uint(fabsf(v)));
}

// ------------------------------------------------------------- tensor maps

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

}  // namespace

bool make_tmap_i8_kmajor(CUtensorMap* map, const void* base, int rows, int K, long long ld, int box_rows) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 15) || K <= 0 || rows <= 0) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

namespace {

template <int BN, int STAGES>
constexpr size_t umma_smem_bytes() {
    return 1024 + STAGES * (kBM * kBK + BN * kBK) + 8 * 32 * 33 * 4 + (2 * STAGES + 4) * 8 + 16;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Persistent launch: at most (SMs x resident CTAs) CTAs, each looping over
// output tiles t = blockIdx.x, +gridDim.x, ...
template <int BN, int STAGES>
cudaError_t launch_umma(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& p, cudaStream_t st) {
    constexpr size_t smem = umma_smem_bytes<BN, STAGES>();
    static int per_sm = 0;
    if (!per_sm) {
        const cudaError_t e = cudaFuncSetAttribute(w8a8_umma_kernel<BN, STAGES>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        int occ = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, w8a8_umma_kernel<BN, STAGES>, kThreads, smem);
        per_sm = occ > 0 ? occ : 1;
    }
    const long long tiles = (long long)((p.N + BN - 1) / BN) * ((p.M + kBM - 1) / kBM);
    const long long cap = (long long)sm_count() * per_sm;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    const cudaError_t le_ = launch_k(w8a8_umma_kernel<BN, STAGES>, grid, kThreads, smem, st, ta, tb, p);
    if (le_ != cudaSuccess) return le_;
    return cudaGetLastError();
}

EpiParams make_epi(const GemmI8Args& a) {
    EpiParams p{};
    p.out = a.out;
    p.ldo = a.ldo;
    p.res = a.res;
    p.ldr = a.ldr;
    p.ascale = a.ascale;
    p.as_stride = a.ascale_per_row ? 1 : 0;
    p.wscale = a.wscale;
    p.bias = a.bias;
    p.amax = a.amax;
    p.amax_rows = a.amax_rows > 0 ? a.amax_rows : 1;
    p.mode = a.mode;
    p.M = a.M;
    p.N = a.N;
    p.K = a.K;
    p.static_weights = a.static_weights ? 1 : 0;
    const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out), rb = reinterpret_cast<uintptr_t>(a.res);
    p.vec_ok = !(a.mode & kEpiAcc) && (ob & 15) == 0 && (a.ldo & 3) == 0 &&
               (!a.res || ((rb & 15) == 0 && (a.ldr & 3) == 0));
    return p;
}

}  // namespace

int gemm_i8_pick_bn(int M, int N) {
    // Fill the 148 SMs: the widest N tile that still yields ~0.8 waves of CTAs,
    // else the narrowest (the 602-row transformer GEMMs, the deep conv stages).
    const int mt = (M + kBM - 1) / kBM;
    for (int bn : {128, 64, 32})
        if (N > bn / 2 && mt * ((N + bn - 1) / bn) >= 120) return bn;
    return 32;
}

cudaError_t gemm_i8_umma(const GemmI8Args& a, const CUtensorMap& ta, const CUtensorMap& tb, int bn,
                         cudaStream_t st) {
    const EpiParams p = make_epi(a);
    if (bn == 32) return launch_umma<32, 4>(ta, tb, p, st);
    if (bn == 64) return launch_umma<64, 4>(ta, tb, p, st);
    if (bn == 256) return launch_umma<256, 4>(ta, tb, p, st);
    return launch_umma<128, 3>(ta, tb, p, st);
}

cudaError_t gemm_i8(const GemmI8Args& a, cudaStream_t st) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaErrorInvalidValue;
    const bool tma_ok = ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) == 0 &&
                        (a.lda & 15) == 0 && (a.ldb & 15) == 0;
    if (!a.force_simt && tma_ok) {
        // operands TMA can describe always take the tensor-core kernel; a tensor
        // map the driver refuses is an error, never a silent detour
        const int bn = gemm_i8_pick_bn(a.M, a.N);
        CUtensorMap ta, tb;
        if (!make_tmap_i8_kmajor(&ta, a.A, a.M, a.K, a.lda, kBM) ||
            !make_tmap_i8_kmajor(&tb, a.B, a.N, a.K, a.ldb, bn))
            return cudaErrorInvalidConfiguration;
        return gemm_i8_umma(a, ta, tb, bn, st);
    }
    const EpiParams p = make_epi(a);
    if ((a.N + 127) / 128 > 65535) return cudaErrorInvalidValue;
    dim3 grid(a.M, (a.N + 127) / 128);
    {
        const cudaError_t le_ = launch_k(w8a8_simt_kernel, grid, 128, 0, st,
                                         a.A, a.lda, a.B, a.ldb, p);
        if (le_ != cudaSuccess) return le_;
    }
    return cudaGetLastError();
}

int device_status_take() {
    int h = 0;
    if (cudaMemcpyFromSymbol(&h, g_vsb_status, sizeof(int)) != cudaSuccess) return -1;
    if (h) {
        const int z = 0;
        cudaMemcpyToSymbol(g_vsb_status, &z, sizeof(int));
    }
    return h;
}

}  // namespace vsb
