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
//   warp 0     lane 0: TMA producer (A and B k-blocks of 128 bytes, `stages`-deep ring)
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
#include <atomic>
#include <cfloat>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace vsb {

namespace {

constexpr int kBM = 128;          // UMMA M (one TMEM lane per tile row)
constexpr int kBK = 128;          // bytes of K per pipeline stage (one SW128 atom row)
constexpr int kUmmaK = 32;        // K per tcgen05.mma kind::i8
constexpr int kThreads = 320;   // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kMaxGlobalSplits = 64;   // K splits over independent CTAs (workspace reduction)

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
    int m_tiles;                  // 128-row M tiles
    // Implicit convolution (conv_bw > 0). A is an int8 NHWC tensor [F][H][W][C]
    // read through a 4D tensor map; M tile mt is the output patch (frame f,
    // tile row ty, tile column tx) of conv_bh x conv_bw pixels, tile row r the
    // pixel (ty*conv_bh + r / conv_bw, tx*conv_bw + r % conv_bw). K runs over
    // (ky, kx, channel block): k-block kb = tap * conv_cb + channel block.
    // ascale is per frame.
    int conv_bw, conv_bh, conv_tx, conv_ty, conv_ho, conv_wo, conv_k, conv_pad, conv_cb;
    int conv_kw;                  // filter width (conv_k = height)
    // split K over independent CTAs (w8a8_splitk_kernel<BN, true>): partial
    // int32 tiles [tile][split][M][BN] in ws, arrivals counted per tile
    int32_t* ws;
    unsigned int* counters;
    int splitk_coop;              // GLOBAL split-K, co-resident: counters [2 * tiles], every CTA reduces rows
    // slab kernel (w8a8_slab_kernel): columns per CTA, CTAs per M tile, staging tiles per epilogue warp
    int slab_bn, slab_groups, slab_nstg;
    // slab kernel, row-quantized output (GemmI8Args::qout)
    int8_t* qout;
    long long ldq;
    float* qscale;
    unsigned int* qamax;
    unsigned int* qsync;
    // GLOBAL split-K with the A operand computed in the kernel (GemmI8Args::im_x)
    const float* im_x;
    const unsigned int* im_rowmax;
    int im_T, im_C, im_k, im_stride, im_pad, im_Tout;
};

// quantize_rows' arithmetic (src/hal/common/gemm_i8.cpp:209-244): the row
// scale s = max(amax / 127, FLT_MIN) (1 for an all-zero row) and the byte of
// q = clamp(rne(v / s)) from inv = 1 / s
__device__ __forceinline__ float rowq_scale(float amax) {
    return amax > 0.0f ? fmaxf(__fdiv_rn(amax, 127.0f), FLT_MIN) : 1.0f;
}
__device__ __forceinline__ uint32_t rowq_q8(float v, float inv) {
    float t = __fmul_rn(v, inv);
    t = t != t ? 0.0f : fminf(fmaxf(t, -127.0f), 127.0f);
    return static_cast<uint32_t>(static_cast<uint8_t>(static_cast<int8_t>(f2i_rn_small(t))));
}
__device__ __forceinline__ uint32_t rowq_pack4(float4 v, float inv) {
    return rowq_q8(v.x, inv) | (rowq_q8(v.y, inv) << 8) | (rowq_q8(v.z, inv) << 16) | (rowq_q8(v.w, inv) << 24);
}

// The A operand of a 1D conv computed in the GEMM (the im2col1d_q8w kernel's
// bytes, without its launch): the 256 epilogue threads (et 0-255, named
// barrier 2) fill this CTA's k-block stages of the 128-byte-swizzled K-major A
// ring. Row m = output step ot of sample f (m = f * Tout + ot); K index
// kt * C + c reads x[f][ot * stride - pad + kt][c] (zero outside the input),
// quantized with the row's scale from its k input rows' absmax (rowmax), kept
// in s_sc [M] (also for the epilogue). Stages are filled as the ring frees
// them (empty), each published with an async-proxy fence and one arrival on
// full (whose other arrival carries the weight tile's bytes). Rows >= M are
// left as they are: no output reads their accumulators. Returns false if a
// wait ran out (recorded in the status word).
__device__ __forceinline__ bool im2col_fill_a(const EpiParams& p, uint8_t* sA, uint64_t* full, uint64_t* empty,
                                              int stages, int kb0, int my_kb, float* s_sc, int et) {
    constexpr int kABytes = kBM * kBK;
    const int M = p.M, C = p.im_C, T = p.im_T, Tout = p.im_Tout;
    for (int m = et; m < M; m += 256) {
        const int f = m / Tout, ot = m - f * Tout;
        unsigned int mb = 0u;
        for (int kt = 0; kt < p.im_k; ++kt) {
            const int t = ot * p.im_stride - p.im_pad + kt;
            if (t >= 0 && t < T) mb = max(mb, __ldcg(p.im_rowmax + (long long)f * T + t));
        }
        s_sc[m] = rowq_scale(__uint_as_float(mb));
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    const int per_kb = M * (kBK / 16);            // 16-byte chunks of one k-block
    int i0 = 0;
    while (i0 < my_kb) {
        // the ring's first `stages` k-blocks in one sweep (every load in flight), then one at a time
        const int i1 = i0 == 0 ? min(my_kb, stages) : i0 + 1;
        if (i0 >= stages && !mbar_wait(&empty[i0 % stages], ((i0 / stages) - 1) & 1)) return false;
        const int n_items = (i1 - i0) * per_kb;
        #pragma unroll 4
        for (int it = et; it < n_items; it += 256) {
            const int di = it / per_kb, rem = it - di * per_kb;
            const int m = rem >> 3, j = rem & 7;
            const int e0 = (kb0 + i0 + di) * kBK + 16 * j;
            uint4 w = make_uint4(0u, 0u, 0u, 0u);
            if (e0 < p.K) {
                const int kt = e0 / C, c = e0 - kt * C;
                const int f = m / Tout, ot = m - f * Tout;
                const int t = ot * p.im_stride - p.im_pad + kt;
                if (t >= 0 && t < T) {
                    const float4* src = reinterpret_cast<const float4*>(p.im_x + ((long long)f * T + t) * C + c);
                    const float4 v0 = __ldcg(src), v1 = __ldcg(src + 1), v2 = __ldcg(src + 2), v3 = __ldcg(src + 3);
                    const float inv = __fdiv_rn(1.0f, s_sc[m]);
                    w = make_uint4(rowq_pack4(v0, inv), rowq_pack4(v1, inv), rowq_pack4(v2, inv), rowq_pack4(v3, inv));
                }
            }
            *reinterpret_cast<uint4*>(sA + (size_t)((i0 + di) % stages) * kABytes + m * kBK + ((j ^ (m & 7)) << 4)) = w;
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync 2, 256;" ::: "memory");
        if (et == 0)
            for (int i = i0; i < i1; ++i) mbar_arrive(&full[i % stages]);
        i0 = i1;
    }
    return true;
}

// Output row (index into out / res, and the absmax slot numerator) of tile
// row r of M tile mt; -1 where the tile row maps to no output.
__device__ __forceinline__ int out_row(const EpiParams& p, int mt, int r) {
    if (!p.conv_bw) {
        const int m = mt * kBM + r;
        return m < p.M ? m : -1;
    }
    const int per_f = p.conv_ty * p.conv_tx;
    const int f = mt / per_f, rem = mt - f * per_f;
    const int ty = rem / p.conv_tx, tx = rem - ty * p.conv_tx;
    const int ly = r / p.conv_bw, lx = r - ly * p.conv_bw;
    const int oy = ty * p.conv_bh + ly, ox = tx * p.conv_bw + lx;
    if (ly >= p.conv_bh || oy >= p.conv_ho || ox >= p.conv_wo) return -1;
    return (f * p.conv_ho + oy) * p.conv_wo + ox;
}

// activation scale of output row m
__device__ __forceinline__ float row_ascale(const EpiParams& p, int m) {
    return p.conv_bw ? p.ascale[m / (p.conv_ho * p.conv_wo)] : p.ascale[(long long)m * p.as_stride];
}

// The A operand of M tile mt, k-block kb (KBB bytes of K) -> shared memory.
template <int KBB>
__device__ __forceinline__ void load_a(const EpiParams& p, const CUtensorMap* ta, void* dst, uint64_t* bar, int mt,
                                       int kb) {
    if (!p.conv_bw) {
        tma_load_2d(dst, ta, bar, kb * KBB, mt * kBM);
        return;
    }
    const int per_f = p.conv_ty * p.conv_tx;
    const int f = mt / per_f, rem = mt - f * per_f;
    const int ty = rem / p.conv_tx, tx = rem - ty * p.conv_tx;
    const int tap = kb / p.conv_cb, cb = kb - tap * p.conv_cb;
    const int ky = tap / p.conv_kw, kx = tap - ky * p.conv_kw;
    tma_load_4d(dst, ta, bar, cb * KBB, tx * p.conv_bw - p.conv_pad + kx, ty * p.conv_bh - p.conv_pad + ky, f);
}

// Phase B of the persistent epilogue for one 32-column chunk: lane (rq, cq)
// finishes columns cq..cq+3 of tile rows rq + 4*r8 from the raw int32
// accumulators in its warp's staging tile (rows kStgLd words apart):
// v = fma(acc*s_w, s_a, b), then ReLU / residual add / add + ReLU, stores, and
// the per-row |v| maximum for the absmax tap. MODE is the epilogue flag set
// (-1: read it at run time); the 32 element computations are straight-line
// code without per-row branches, so they interleave; only stores are predicated.
// Five instances in all (one per mode): the absmax upkeep is a uniform branch,
// not a template flag, to keep the kernel's code within the instruction cache.
constexpr int kStgLd = 36;   // words per staging row: 16-byte aligned, conflict-free per quarter warp

template <int MODE>
__device__ __forceinline__ void epi_rows(const EpiParams& p, const float* stg, int rq, int cq, const int (&mrow)[8],
                                         const float (&asr)[8], const float (&ws)[4], const float (&bb)[4],
                                         const float4 (&rv)[8], int n, bool full4, float (&rmax)[8]) {
    const int mode = MODE >= 0 ? MODE : p.mode;
    float v[8][4];
    #pragma unroll
    for (int r8 = 0; r8 < 8; ++r8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(stg + (rq + 4 * r8) * kStgLd + cq);
        const int32_t a4[4] = {static_cast<int32_t>(raw.x), static_cast<int32_t>(raw.y), static_cast<int32_t>(raw.z),
                               static_cast<int32_t>(raw.w)};
        const float* rvv = reinterpret_cast<const float*>(&rv[r8]);
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            float t = __fmaf_rn(__fmul_rn(__int2float_rn(a4[e]), ws[e]), asr[r8], bb[e]);
            if (mode & kEpiRelu) t = (t < 0.0f) ? 0.0f : t;            // tcpu::relu (eltwise.cpp:213-214)
            if (mode & kEpiAdd) t = __fadd_rn(rvv[e], t);               // x[i] += y[i]
            if (mode & kEpiAddRelu) {                                   // resnet_backbone.cpp:293-295
                t = __fadd_rn(t, rvv[e]);
                t = t > 0.0f ? t : 0.0f;
            }
            v[r8][e] = t;
        }
    }
    if (p.amax) {
        #pragma unroll
        for (int r8 = 0; r8 < 8; ++r8) {
            const bool row_ok = mrow[r8] >= 0 && n < p.N;
            #pragma unroll
            for (int e = 0; e < 4; ++e) rmax[r8] = fmaxf(rmax[r8], (row_ok && n + e < p.N) ? fabsf(v[r8][e]) : 0.0f);
        }
    }
    #pragma unroll
    for (int r8 = 0; r8 < 8; ++r8) {
        const int m = mrow[r8];
        const bool row_ok = m >= 0 && n < p.N;
        if (!row_ok) continue;
        float* o = static_cast<float*>(p.out) + (long long)m * p.ldo + n;
        if (p.vec_ok && full4) {
            *reinterpret_cast<float4*>(o) = make_float4(v[r8][0], v[r8][1], v[r8][2], v[r8][3]);
        } else {
            #pragma unroll
            for (int e = 0; e < 4; ++e)
                if (n + e < p.N) o[e] = v[r8][e];
        }
    }
}

template <int KBB>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
    if constexpr (KBB == 128) return sw128_kmajor_desc(saddr);
    else return sw64_kmajor_desc(saddr);
}

__device__ __forceinline__ float epi_value(int32_t acc, float ws, float as, float b, int mode,
                                           const float* resp) {
    float v = __fmaf_rn(__fmul_rn(__int2float_rn(acc), ws), as, b);
    if (mode & kEpiRelu) v = (v < 0.0f) ? 0.0f : v;                 // eltwise relu (eltwise.cpp:213-214)
    if (mode & kEpiAdd) v = __fadd_rn(*resp, v);                      // x[i] += y[i]
    if (mode & kEpiAddRelu) { v = __fadd_rn(v, *resp); v = v > 0.0f ? v : 0.0f; }  // resnet_backbone.cpp:293-295
    return v;
}

template <int BN, int KBB>
__global__ void __launch_bounds__(kThreads, 1)
w8a8_umma_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b,
                 const EpiParams p, const int stages) {
    constexpr int kABytes = kBM * KBB;
    constexpr int kBBytes = BN * KBB;
    constexpr uint32_t kIdesc = idesc_s8s8_s32(kBM, BN);
    constexpr int kStg = 32 * kStgLd;   // one epilogue warp's 32 x 32 staging tile
    constexpr int kEpiWarps = 8;

    extern __shared__ uint8_t smem_raw[];
    // SW128 tiles want 1024-byte alignment
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared-window pointer
    uint8_t* sA = smem;
    uint8_t* sB = smem + stages * kABytes;
    float* stg_all = reinterpret_cast<float*>(sB + stages * kBBytes);
    uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + kEpiWarps * kStg);
    uint64_t* empty = full + stages;
    uint64_t* acc_full = empty + stages;     // [2]: accumulator buffer ready for the epilogue
    uint64_t* acc_empty = acc_full + 2;      // [2]: epilogue done reading the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* s_consumed = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_tn = (p.N + BN - 1) / BN;
    const int n_tiles = n_tn * p.m_tiles;
    const int nkb = (p.K + KBB - 1) / KBB;
    // bytes one k-block brings in: a conv patch box may be under 128 rows
    const uint32_t stage_tx = (p.conv_bw ? KBB * p.conv_bw * p.conv_bh : kABytes) + kBBytes;
    // weights that a predecessor kernel may still be writing: wait up front
    if (!p.static_weights) pdl_wait();

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
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
            // of `stages` k-block slots shared across tiles. The weight halves of
            // the first slots go out before waiting for the predecessor kernel.
            const int pre = nkb < stages ? nkb : stages;
            {
                const int n0 = (blockIdx.x % n_tn) * BN;
                for (int kb = 0; kb < pre; ++kb) {
                    mbar_arrive_expect_tx(&full[kb], stage_tx);
                    tma_load_2d(sB + kb * kBBytes, &tmap_b, &full[kb], kb * KBB, n0);
                }
            }
            pdl_wait();
            int it = 0;
            bool fail = false;
            for (int t = blockIdx.x; t < n_tiles && !fail; t += gridDim.x) {
                const int mt = t / n_tn, n0 = (t % n_tn) * BN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % stages;
                    if (it < pre) {   // first tile's weights already in flight
                        load_a<KBB>(p, &tmap_a, sA + s * kABytes, &full[s], mt, kb);
                    } else {
                        const int use = it / stages;   // > 0 unless the ring is longer than the first tile
                        if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1)) { fail = true; break; }
                        mbar_arrive_expect_tx(&full[s], stage_tx);
                        load_a<KBB>(p, &tmap_a, sA + s * kABytes, &full[s], mt, kb);
                        tma_load_2d(sB + s * kBBytes, &tmap_b, &full[s], kb * KBB, n0);
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
                    const int s = it % stages;
                    if (!mbar_wait(&full[s], (it / stages) & 1)) { fail = true; break; }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + s * kABytes);
                    const uint32_t b_addr = smem_u32(sB + s * kBBytes);
                    #pragma unroll
                    for (int k = 0; k < KBB / kUmmaK; ++k) {
                        umma_s8(d_tmem, kmajor_desc<KBB>(a_addr + k * kUmmaK),
                                kmajor_desc<KBB>(b_addr + k * kUmmaK), kIdesc, (kb | k) != 0);
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
        // row, as TMEM hands it out) parks the raw int32 accumulators in this
        // warp's staging tile (16-byte stores, rows 36 words apart); phase B
        // (coalesced) - lane l owns columns 4*(l%8)..+3 of rows l/8 + 4i -
        // applies v = fma(acc*s_w, s_a, b), ReLU / residual, and stores four
        // whole 128-byte row segments per instruction. A lane's 4 column scales
        // and biases are one vector load per chunk, its 8 row scales one load
        // each per tile: no shuffles.
        const int quarter = warp & 3;   // TMEM lanes this warp may read: 32 * (warp id % 4)
        const int half = (warp - 2) >> 2;   // which column chunks: c % 2 == half
        float* stg = stg_all + (warp - 2) * kStg;
        const bool acc_mode = (p.mode & kEpiAcc) != 0;
        const int cq = (lane & 7) * 4;
        const int rq = lane >> 3;
        pdl_wait();   // activation scales / residual / output: predecessor data
        constexpr int kChunks = (BN / 32 + 1) / 2;   // column chunks per warp: c = half, half + 2, ...
        // residual of chunk c for this lane's 8 rows x 4 columns (phase B layout)
        auto load_res = [&](float4 (&rv)[8], const int (&mrow)[8], int n0, int c) {
            const int n = n0 + c * 32 + cq;
            const bool full4 = n + 4 <= p.N;
            #pragma unroll
            for (int r8 = 0; r8 < 8; ++r8) {
                const int m = mrow[r8];
                rv[r8] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (m < 0 || n >= p.N) continue;
                const float* rr = p.res + (long long)m * p.ldr + n;
                if (p.vec_ok && full4) {
                    rv[r8] = *reinterpret_cast<const float4*>(rr);
                } else {
                    float* t = reinterpret_cast<float*>(&rv[r8]);
                    #pragma unroll
                    for (int e = 0; e < 4; ++e) t[e] = n + e < p.N ? rr[e] : 0.0f;
                }
            }
        };
        // column scales / biases of chunk c for this lane's 4 columns
        auto load_cols = [&](float (&ws)[4], float (&bb)[4], int n0, int c) {
            const int n = n0 + c * 32 + cq;
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool ok = c < BN / 32 && n + e < p.N;
                ws[e] = ok ? p.wscale[n + e] : 0.0f;
                bb[e] = (ok && p.bias) ? p.bias[n + e] : 0.0f;
            }
        };
        const bool has_res = (p.mode & (kEpiAdd | kEpiAddRelu)) != 0;
        // The tile-invariant part of each phase-B row's output position, once
        // per CTA: the per-tile work below is then two divisions (conv) and a
        // multiply-add per row instead of out_row's divisions per row, which
        // measured ~6 K cycles per tile on the stem conv, longer than the
        // tile's loads and MMAs.
        int ly[8], lx[8];
        #pragma unroll
        for (int r8 = 0; r8 < 8; ++r8) {
            const int r = quarter * 32 + rq + 4 * r8;
            ly[r8] = p.conv_bw ? r / p.conv_bw : 0;
            lx[r8] = p.conv_bw ? r - ly[r8] * p.conv_bw : r;
        }
        int i = 0;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++i) {
            const int buf = i & 1;
            const int mt = t / n_tn, n0 = (t % n_tn) * BN;
            int mrow[8];                                                // phase B rows of this lane
            float asr[8];                                               // and their activation scales
            if (p.conv_bw) {
                // out_row: patch (f, ty, tx) of tile mt, pixel (ly, lx) of the patch
                const int per_f = p.conv_ty * p.conv_tx;
                const int f = mt / per_f, rem = mt - f * per_f;
                const int ty = rem / p.conv_tx, tx = rem - ty * p.conv_tx;
                const float fs = acc_mode ? 0.0f : p.ascale[f];        // row_ascale: one scale per frame
                #pragma unroll
                for (int r8 = 0; r8 < 8; ++r8) {
                    const int oy = ty * p.conv_bh + ly[r8], ox = tx * p.conv_bw + lx[r8];
                    const bool ok = ly[r8] < p.conv_bh && oy < p.conv_ho && ox < p.conv_wo;
                    mrow[r8] = ok ? (f * p.conv_ho + oy) * p.conv_wo + ox : -1;
                    asr[r8] = ok ? fs : 0.0f;
                }
            } else {
                #pragma unroll
                for (int r8 = 0; r8 < 8; ++r8) {
                    const int m = mt * kBM + lx[r8];
                    mrow[r8] = m < p.M ? m : -1;
                    asr[r8] = (mrow[r8] >= 0 && !acc_mode) ? p.ascale[(long long)m * p.as_stride] : 0.0f;
                }
            }
            // Everything the epilogue reads besides the accumulators is fetched
            // before waiting for them, so its latency hides behind the MMAs.
            // (Each lane later writes only elements it read here or reads
            // itself, so a residual aliasing out is never read after a store.)
            float ws[4], bb[4];
            if (!acc_mode) load_cols(ws, bb, n0, half);
            float4 rv[8];
            if (has_res && half < BN / 32) load_res(rv, mrow, n0, half);
            // warp-uniform: the tcgen05.ld below needs every lane
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&acc_full[buf], (i >> 1) & 1))) break;
            tc_fence_after();
            float rmax[8];                                              // |out| per phase B row (absmax tap)
            #pragma unroll
            for (int r8 = 0; r8 < 8; ++r8) rmax[r8] = 0.0f;
            #pragma unroll 1
            for (int ci = 0; ci < kChunks; ++ci) {                      // rolled: one copy of the chunk code
                const int c = half + 2 * ci;
                if (c >= BN / 32) break;
                if (n0 + c * 32 >= p.N) break;                          // warp-uniform; later chunks too
                uint32_t acc[32];
                tmem_ld_32x32b_x32(tmem_base + buf * BN + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, acc);
                tmem_ld_wait();
                #pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<uint4*>(stg + lane * kStgLd + j) = make_uint4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                __syncwarp();
                const int n = n0 + c * 32 + cq;
                const bool full4 = n + 4 <= p.N;
                // the next chunk's operands go out before this chunk's stores
                // (different columns, so no aliasing hazard)
                float4 rn[8];
                float wn[4], bn[4];
                const bool more = ci + 1 < kChunks && c + 2 < BN / 32;
                if (more && !acc_mode) load_cols(wn, bn, n0, c + 2);
                if (more && has_res) load_res(rn, mrow, n0, c + 2);
                // Straight-line over all 8 rows x 4 columns (no per-row
                // branches, mode flags as selects): one basic block, so the 32
                // independent element chains interleave; only the stores are
                // predicated.
                if (acc_mode) {
                    #pragma unroll
                    for (int r8 = 0; r8 < 8; ++r8) {
                        const uint4 raw = *reinterpret_cast<const uint4*>(stg + (rq + 4 * r8) * kStgLd + cq);
                        const int m = mrow[r8];
                        if (m < 0 || n >= p.N) continue;
                        const uint32_t a4[4] = {raw.x, raw.y, raw.z, raw.w};
                        int32_t* o = static_cast<int32_t*>(p.out) + (long long)m * p.ldo + n;
                        #pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (n + e < p.N) o[e] = static_cast<int32_t>(a4[e]);
                    }
                } else {
                    // the mode as a template flag: each instance carries only
                    // its own operations (see epi_rows)
                    const int mode = p.mode & (kEpiRelu | kEpiAdd | kEpiAddRelu);
                    #define VSB_EPI(M) epi_rows<M>(p, stg, rq, cq, mrow, asr, ws, bb, rv, n, full4, rmax)
                    if (mode == 0) VSB_EPI(0);
                    else if (mode == kEpiRelu) VSB_EPI(kEpiRelu);
                    else if (mode == kEpiAdd) VSB_EPI(kEpiAdd);
                    else if (mode == kEpiAddRelu) VSB_EPI(kEpiAddRelu);
                    else VSB_EPI(-1);
                    #undef VSB_EPI
                }
                if (more) {
                    #pragma unroll
                    for (int e = 0; e < 4; ++e) { ws[e] = wn[e]; bb[e] = bn[e]; }
                    if (has_res) {
                        #pragma unroll
                        for (int r8 = 0; r8 < 8; ++r8) rv[r8] = rn[r8];
                    }
                }
                __syncwarp();                                           // staging tile reused by the next chunk
            }
            // this tile's TMEM buffer may be reused by the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[buf]);
            if (p.amax) {
                // one atomic per warp when the warp's rows share a slot, else one
                // per row (its 8 lanes reduced first); rows past M count nothing
                unsigned key[8];
                bool same = true;
                const unsigned first = mrow[0] >= 0 ? static_cast<unsigned>(mrow[0] / p.amax_rows) : 0xFFFFFFFFu;
                #pragma unroll
                for (int r8 = 0; r8 < 8; ++r8) {
                    key[r8] = mrow[r8] >= 0 ? static_cast<unsigned>(mrow[r8] / p.amax_rows) : 0xFFFFFFFFu;
                    same = same && (key[r8] == first || key[r8] == 0xFFFFFFFFu);
                }
                const unsigned k0 = __shfl_sync(0xFFFFFFFFu, first, 0);
                if (__all_sync(0xFFFFFFFFu, same && (first == k0 || first == 0xFFFFFFFFu))) {
                    float wm = 0.0f;
                    #pragma unroll
                    for (int r8 = 0; r8 < 8; ++r8) wm = fmaxf(wm, rmax[r8]);
                    #pragma unroll
                    for (int off = 16; off > 0; off >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xFFFFFFFFu, wm, off));
                    if (lane == 0 && k0 != 0xFFFFFFFFu) atomicMax(&p.amax[k0], __float_as_uint(wm));
                } else {
                    #pragma unroll
                    for (int r8 = 0; r8 < 8; ++r8) {
                        float wm = rmax[r8];
                        #pragma unroll
                        for (int off = 4; off > 0; off >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xFFFFFFFFu, wm, off));
                        if ((lane & 7) == 0 && key[r8] != 0xFFFFFFFFu) atomicMax(&p.amax[key[r8]], __float_as_uint(wm));
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // never leave the CTA with TMA writes still landing in its shared memory
        for (int kb = *s_consumed; kb < issued; ++kb)
            if (!mbar_wait(&full[kb % stages], (kb / stages) & 1)) break;
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * BN);
    }
}

// -------------------------------------------------------- split-K (cluster)
// For GEMMs with few output tiles and a long K (the deep conv stages, the FFN
// down-projection) one tile per SM leaves most SMs idle and each busy one
// streaming every k-block alone. Here the `splits` CTAs of a thread-block
// cluster (grid = splits x tiles, cluster = splits x 1) take the same 128 x BN
// tile over disjoint k-block ranges, each into its own TMEM accumulator. The
// int32 partial tiles then go to shared memory and are summed through
// distributed shared memory - integer addition, so the sums are exact and
// equal to the single-pass accumulators whatever the order - and each CTA
// finishes the tile rows r = rank, rank + splits, ... through the same fp32
// epilogue as the persistent kernel (bit-identical outputs).
//   warp 0 lane 0: TMA producer; warp 1: TMEM + MMA issuer;
//   warps 2-9: TMEM -> shared partial tile, then the cross-CTA sum + epilogue.
template <int BN, bool GLOBAL>
__global__ void __launch_bounds__(kThreads, 1)
w8a8_splitk_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const EpiParams p, const int stages) {
    constexpr int kABytes = kBM * kBK;
    constexpr int kBBytes = BN * kBK;
    constexpr uint32_t kIdesc = idesc_s8s8_s32(kBM, BN);
    constexpr int kPS = BN + 4;           // partial tile row stride (int32): 16-byte rows, conflict-free v4
    constexpr int kC4 = BN / 4;           // 4-column groups per row
    constexpr int kRPP = 256 / kC4;       // tile rows per pass of the 256 epilogue threads
    // the host guarantees kBM * kPS * 4 <= stages * (kABytes + kBBytes): the
    // partial tile overlays the stage ring

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared-window pointer
    uint8_t* sA = smem;
    uint8_t* sB = smem + stages * kABytes;
    int32_t* part = reinterpret_cast<int32_t*>(smem);    // [kBM][kPS], once the ring is idle
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + stages * kBBytes);
    uint64_t* empty = full + stages;
    uint64_t* acc_full = empty + stages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* s_consumed = reinterpret_cast<volatile int*>(tmem_slot + 1);
    unsigned int* s_amax = reinterpret_cast<unsigned int*>(tmem_slot + 2);   // [4]
    volatile int* s_last = reinterpret_cast<volatile int*>(tmem_slot + 6);
    float* s_imscale = reinterpret_cast<float*>(tmem_slot + 8);              // [kBM], GLOBAL with im_x

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int splits = gridDim.x;
    const int rank = blockIdx.x;          // cluster (splits, 1, 1): rank in the cluster (GLOBAL: in the grid row)
    const int n_tn = (p.N + BN - 1) / BN;
    const int mt = blockIdx.y / n_tn, n0 = (blockIdx.y % n_tn) * BN;
    const int nkb = (p.K + kBK - 1) / kBK;
    const bool im_a = GLOBAL && p.im_x != nullptr;   // A computed by the epilogue warps
    const uint32_t stage_tx = (im_a ? 0u : p.conv_bw ? kBK * p.conv_bw * p.conv_bh : kABytes) + kBBytes;
    const int kb0 = static_cast<int>((long long)nkb * rank / splits);
    const int my_kb = static_cast<int>((long long)nkb * (rank + 1) / splits) - kb0;   // >= 1: splits <= nkb
    if (!p.static_weights) pdl_wait();

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) { mbar_init(&full[s], im_a ? 2 : 1); mbar_init(&empty[s], 1); }
        mbar_init(acc_full, 1);
        *s_consumed = 0;
        for (int i = 0; i < 4; ++i) s_amax[i] = 0u;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) tmem_alloc(tmem_slot, BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();

    int issued = 0;
    if (warp == 0) {
        if (lane == 0) {
            const int pre = my_kb < stages ? my_kb : stages;
            for (int i = 0; i < pre; ++i) {     // weights first: load-time constants
                mbar_arrive_expect_tx(&full[i], stage_tx);
                tma_load_2d(sB + i * kBBytes, &tmap_b, &full[i], (kb0 + i) * kBK, n0);
            }
            pdl_wait();
            for (int i = 0; i < my_kb; ++i) {
                const int s = i % stages;
                if (i >= pre) {
                    if (!mbar_wait(&empty[s], ((i / stages) - 1) & 1)) break;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    tma_load_2d(sB + s * kBBytes, &tmap_b, &full[s], (kb0 + i) * kBK, n0);
                }
                if (!im_a) load_a<kBK>(p, &tmap_a, sA + s * kABytes, &full[s], mt, kb0 + i);
                issued = i + 1;
            }
            if (issued < pre) issued = pre;     // the weight halves went out regardless
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool fail = false;
            for (int i = 0; i < my_kb; ++i) {
                const int s = i % stages;
                if (!mbar_wait(&full[s], (i / stages) & 1)) { fail = true; break; }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(sA + s * kABytes);
                const uint32_t b_addr = smem_u32(sB + s * kBBytes);
                #pragma unroll
                for (int k = 0; k < kBK / kUmmaK; ++k)
                    umma_s8(tmem_base, sw128_kmajor_desc(a_addr + k * kUmmaK),
                            sw128_kmajor_desc(b_addr + k * kUmmaK), kIdesc, (i | k) != 0);
                umma_commit(&empty[s]);
                *s_consumed = i + 1;
            }
            if (!fail) umma_commit(acc_full);
        }
        __syncwarp();
    } else {
        pdl_wait();                 // activation scales / residual: predecessor data
        // the conv input's im2col rows into the A stages (a timeout is recorded;
        // the MMA warp's bounded waits then end the tile)
        if (im_a) im2col_fill_a(p, sA, full, empty, stages, kb0, my_kb, s_imscale, threadIdx.x - 64);
        mbar_wait(acc_full, 0);     // a timeout is recorded in the status word
        tc_fence_after();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // the partial tile overlays the ring: no TMA write may still be landing
        for (int i = *s_consumed; i < issued; ++i)
            if (!mbar_wait(&full[i % stages], (i / stages) & 1)) break;
    }
    __syncthreads();

    // ---- phase 1: this CTA's partial accumulators -> shared [row][col] int32
    // (a plain GEMM's quadrants past the last row hold nothing anyone reads)
    if (warp >= 2 && (p.conv_bw || mt * kBM + (warp & 3) * 32 < p.M)) {
        const int quarter = warp & 3;
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        #pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
            uint32_t acc[32];
            tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + c * 32, acc);
            tmem_ld_wait();
            int4* dst = reinterpret_cast<int4*>(part + row * kPS + c * 32);
            #pragma unroll
            for (int j = 0; j < 8; ++j)
                dst[j] = make_int4(static_cast<int>(acc[4 * j]), static_cast<int>(acc[4 * j + 1]),
                                   static_cast<int>(acc[4 * j + 2]), static_cast<int>(acc[4 * j + 3]));
        }
    }
    tc_fence_before();
    if (!GLOBAL) {
        cluster_sync();      // every partial tile of the cluster is in shared memory
    } else {
        // the rows with an output go to this split's workspace slice; the CTA
        // that arrives last for the tile (counter) sums the slices in phase 2
        __syncthreads();
        if (warp >= 2) {
            int32_t* wsl = p.ws + ((long long)blockIdx.y * splits + rank) * p.M * BN;
            for (int idx = threadIdx.x - 64; idx < kBM * kC4; idx += 256) {
                const int r = idx / kC4, q = idx - r * kC4;
                if (r >= p.M) break;
                *reinterpret_cast<int4*>(wsl + (long long)r * BN + 4 * q) =
                    *reinterpret_cast<const int4*>(part + r * kPS + 4 * q);
            }
        }
        // one thread publishes the CTA's writes (the barrier orders them before
        // its fence) and counts the arrival; the last arrival acquires the others'
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (p.splitk_coop) {
                // every CTA of the grid is resident (cooperative launch): each
                // waits (bounded) until the tile's slices are all written, then
                // reduces its own interleaved rows, as the cluster form does
                unsigned int* arrive = p.counters + 2 * blockIdx.y;
                atomicAdd(arrive, 1u);
                int ok = 1;
                const uint64_t t0 = globaltimer_ns();
                while (*reinterpret_cast<volatile unsigned int*>(arrive) < static_cast<unsigned>(splits)) {
                    if (globaltimer_ns() - t0 > kWaitLimitNs) {
                        record_status(kStatusWaitTimeout);
                        ok = 0;
                        break;
                    }
                }
                __threadfence();
                *s_last = ok;
            } else {
                const bool last = atomicAdd(&p.counters[blockIdx.y], 1u) == static_cast<unsigned>(splits - 1);
                if (last) __threadfence();
                *s_last = last ? 1 : 0;
            }
        }
        __syncthreads();
    }

    // ---- phase 2: sum the cluster's partials for rows rank, rank + splits, ...
    // (GLOBAL: the last-arriving CTA sums every split's slice for all rows)
    if (warp >= 2) {
        const int et = threadIdx.x - 64;
        const int q = et % kC4, rsub = et / kC4;
        const int n = n0 + 4 * q;
        const bool acc_mode = (p.mode & kEpiAcc) != 0;
        const bool has_res = (p.mode & (kEpiAdd | kEpiAddRelu)) != 0;
        const bool vec = p.vec_ok && n + 4 <= p.N;
        float ws[4], bb[4];
        #pragma unroll
        for (int e = 0; e < 4; ++e) {
            const bool ok = n + e < p.N;
            ws[e] = ok ? p.wscale[n + e] : 0.0f;
            bb[e] = (ok && p.bias) ? p.bias[n + e] : 0.0f;
        }
        const uint32_t part_s = smem_u32(part);
        // tile row 0 always maps to an output row (the tile's origin)
        const unsigned key0 = p.amax ? static_cast<unsigned>(out_row(p, mt, 0) / p.amax_rows) : 0u;
        unsigned cur_key = 0xFFFFFFFFu;
        float cur_max = 0.0f;
        auto flush = [&]() {
            if (cur_key == 0xFFFFFFFFu) return;
            if (cur_key - key0 < 4u) atomicMax(&s_amax[cur_key - key0], __float_as_uint(cur_max));
            else atomicMax(&p.amax[cur_key], __float_as_uint(cur_max));
        };
        const bool one_reducer = GLOBAL && !p.splitk_coop;     // the last CTA to arrive sums every row
        const int r_first = one_reducer ? 0 : rank, r_step = one_reducer ? 1 : splits;
        const bool reduce_here = !GLOBAL || *s_last;
        // Over independent CTAs with at most two rows per thread (the batch-1
        // policies' skinny GEMMs): both rows' slices are summed up front, 16
        // loads in flight per thread, instead of eight per row in turn.
        int4 gsum0 = make_int4(0, 0, 0, 0), gsum1 = make_int4(0, 0, 0, 0);
        const bool gpre = one_reducer && reduce_here && p.M <= 2 * kRPP;
        if (gpre) {
            const long long sl = (long long)p.M * BN;
            const int32_t* base = p.ws + (long long)blockIdx.y * splits * p.M * BN + 4 * q;
            const bool ok0 = rsub < p.M && n < p.N, ok1 = rsub + kRPP < p.M && n < p.N;
            for (int s0 = 0; s0 < splits; s0 += 8) {
                int4 a[8], b[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const bool in = s0 + u < splits;
                    a[u] = (in && ok0) ? __ldcg(reinterpret_cast<const int4*>(base + (long long)rsub * BN + (s0 + u) * sl))
                                       : make_int4(0, 0, 0, 0);
                    b[u] = (in && ok1) ? __ldcg(reinterpret_cast<const int4*>(base + (long long)(rsub + kRPP) * BN +
                                                                               (s0 + u) * sl))
                                       : make_int4(0, 0, 0, 0);
                }
                #pragma unroll
                for (int u = 0; u < 8; ++u) {
                    gsum0.x += a[u].x; gsum0.y += a[u].y; gsum0.z += a[u].z; gsum0.w += a[u].w;
                    gsum1.x += b[u].x; gsum1.y += b[u].y; gsum1.z += b[u].z; gsum1.w += b[u].w;
                }
            }
        }
        // Every load a row needs (its partial sums from the cluster's CTAs, its
        // residual, its activation scale) is issued before any is used, rather
        // than one remote load-then-add per split (the backbone convs' split-K
        // launches: 11.6 vs 12.1 us; this phase is still ~1/3 of such a launch).
        for (int j = rsub; reduce_here && r_first + r_step * j < kBM; j += kRPP) {
            const int r = r_first + r_step * j;
            const int m = out_row(p, mt, r);
            if (m < 0 || n >= p.N) continue;
            float rv[4] = {0.f, 0.f, 0.f, 0.f};
            if (has_res && !acc_mode) {
                const float* rr = p.res + (long long)m * p.ldr + n;
                if (vec) {
                    const float4 t4 = *reinterpret_cast<const float4*>(rr);
                    rv[0] = t4.x; rv[1] = t4.y; rv[2] = t4.z; rv[3] = t4.w;
                } else {
                    #pragma unroll
                    for (int e = 0; e < 4; ++e) rv[e] = n + e < p.N ? rr[e] : 0.0f;
                }
            }
            const float as = acc_mode ? 0.0f : im_a ? s_imscale[r] : row_ascale(p, m);
            int4 sum = make_int4(0, 0, 0, 0);
            if (gpre) {
                sum = j == rsub ? gsum0 : gsum1;
            } else if (GLOBAL) {
                // eight slices' loads in flight at a time (integer sums: any order)
                const int32_t* src0 = p.ws + (long long)blockIdx.y * splits * p.M * BN + (long long)r * BN + 4 * q;
                const long long sl = (long long)p.M * BN;
                for (int s0 = 0; s0 < splits; s0 += 8) {
                    int4 v[8];
                    #pragma unroll
                    for (int u = 0; u < 8; ++u)
                        v[u] = s0 + u < splits ? __ldcg(reinterpret_cast<const int4*>(src0 + (s0 + u) * sl))
                                               : make_int4(0, 0, 0, 0);
                    #pragma unroll
                    for (int u = 0; u < 8; ++u) { sum.x += v[u].x; sum.y += v[u].y; sum.z += v[u].z; sum.w += v[u].w; }
                }
            } else {
                // the cluster's (at most 8) partial rows, all loads in flight (integer sums: any order)
                const uint32_t off = part_s + static_cast<uint32_t>((r * kPS + 4 * q) * 4);
                int4 v[8];
                #pragma unroll
                for (int u = 0; u < 8; ++u)
                    v[u] = u < splits ? dsmem_ld_v4(dsmem_map(off, static_cast<uint32_t>(u))) : make_int4(0, 0, 0, 0);
                #pragma unroll
                for (int u = 0; u < 8; ++u) { sum.x += v[u].x; sum.y += v[u].y; sum.z += v[u].z; sum.w += v[u].w; }
            }
            const int32_t a4[4] = {sum.x, sum.y, sum.z, sum.w};
            if (acc_mode) {
                int32_t* o = static_cast<int32_t*>(p.out) + (long long)m * p.ldo + n;
                #pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (n + e < p.N) o[e] = a4[e];
                continue;
            }
            float v[4];
            float lmax = 0.0f;
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[e] = epi_value(a4[e], ws[e], as, bb[e], p.mode, &rv[e]);
                if (n + e < p.N) lmax = fmaxf(lmax, fabsf(v[e]));
            }
            float* o = static_cast<float*>(p.out) + (long long)m * p.ldo + n;
            if (vec) {
                *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                #pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (n + e < p.N) o[e] = v[e];
            }
            if (p.amax) {
                const unsigned key = static_cast<unsigned>(m / p.amax_rows);
                if (key != cur_key) { flush(); cur_key = key; cur_max = 0.0f; }
                cur_max = fmaxf(cur_max, lmax);
            }
        }
        if (p.amax) {
            flush();
            asm volatile("bar.sync 1, 256;" ::: "memory");     // epilogue warps only
            if (et < 4 && s_amax[et] != 0u) atomicMax(&p.amax[key0 + et], s_amax[et]);
        }
    }
    if (!GLOBAL) {
        cluster_sync();      // no CTA leaves while another still reads its partial tile
    } else if (p.splitk_coop) {
        __syncthreads();
        if (threadIdx.x == 0) {
            // the tile's last CTA to leave: every CTA of it is past the wait and
            // done reading the slices; both counters ready for the next launch
            unsigned int* depart = p.counters + 2 * blockIdx.y + 1;
            if (atomicAdd(depart, 1u) + 1 == static_cast<unsigned>(splits)) {
                p.counters[2 * blockIdx.y] = 0u;
                *depart = 0u;
            }
        }
    } else if (threadIdx.x == 0 && *s_last) {
        p.counters[blockIdx.y] = 0u;     // ready for the next launch (stream-ordered after this one)
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, BN);
    }
}

#include "gemm_slab.cuh"

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

// A few rows (1-4: the diffusion heads' one-query GEMMs): a warp per output
// column n, its lanes over 16-byte chunks of the weight row (coalesced) and
// of each A row, dp4a into int32 (exact: integer sums in any order), a warp
// reduction, then the same fp32 epilogue. K % 16 == 0, 16-byte aligned rows.
// The weights are load-time constants when static_weights: requested before
// the wait on the previous kernel.
constexpr int kGemvMaxRows = 4;

__global__ void __launch_bounds__(256)
w8a8_gemv_kernel(const int8_t* __restrict__ A, long long lda, const int8_t* __restrict__ B, long long ldb,
                 const EpiParams p) {
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
    const bool live = n < p.N;
    const int nch = p.K >> 4;                       // 16-byte chunks per row
    const int4* b = reinterpret_cast<const int4*>(B + (long long)(live ? n : 0) * ldb);
    // up to 4 chunks per lane (K <= 2048) in registers
    int4 bw[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * i;
        bw[i] = (live && c < nch && p.static_weights) ? b[c] : make_int4(0, 0, 0, 0);
    }
    pdl_wait();     // A (and the residual) come from the previous kernel
    pdl_trigger();
    if (!p.static_weights) {
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            bw[i] = (live && c < nch) ? b[c] : make_int4(0, 0, 0, 0);
        }
    }
    int32_t acc[kGemvMaxRows];
    #pragma unroll
    for (int m = 0; m < kGemvMaxRows; ++m) {
        acc[m] = 0;
        if (m >= p.M) continue;
        const int4* a = reinterpret_cast<const int4*>(A + (long long)m * lda);
        #pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int c = lane + 32 * i;
            if (c < nch) {
                const int4 av = a[c];
                acc[m] = __dp4a(av.x, bw[i].x, acc[m]);
                acc[m] = __dp4a(av.y, bw[i].y, acc[m]);
                acc[m] = __dp4a(av.z, bw[i].z, acc[m]);
                acc[m] = __dp4a(av.w, bw[i].w, acc[m]);
            }
        }
        #pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xFFFFFFFFu, acc[m], off);
    }
    if (!live || lane >= p.M) return;
    const int m = lane;
    int32_t am = acc[0];
    #pragma unroll
    for (int i = 1; i < kGemvMaxRows; ++i)
        if (m == i) am = acc[i];
    if (p.mode & kEpiAcc) {
        static_cast<int32_t*>(p.out)[(long long)m * p.ldo + n] = am;
        return;
    }
    const float rv = p.res ? p.res[(long long)m * p.ldr + n] : 0.0f;
    const float v = epi_value(am, p.wscale[n], p.ascale[(long long)m * p.as_stride], p.bias ? p.bias[n] : 0.0f,
                              p.mode, &rv);
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

// 4D map over an int8 NHWC tensor [F][H][W][C]: box {kbb channels, bw, bh, 1},
// swizzled like the K-major operand tiles the MMA reads (128- or 64-byte rows).
bool make_tmap_nhwc_i8(CUtensorMap* map, const void* base, int F, int H, int W, int C, int kbb, int bw, int bh) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || C % kbb || (kbb != 64 && kbb != 128)) return false;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                                static_cast<cuuint64_t>(F)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W) * C,
                                   static_cast<cuuint64_t>(H) * W * C};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(kbb), static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh),
                               1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          kbb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 2D K-major weight map with kbb-byte k-blocks (the 64-byte form for 64-channel convs)
bool make_tmap_i8_kmajor_kb(CUtensorMap* map, const void* base, int rows, int K, long long ld, int box_rows,
                            int kbb) {
    if (kbb == 128) return make_tmap_i8_kmajor(map, base, rows, K, ld, box_rows);
    auto fn = get_encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 15) || K <= 0 || rows <= 0) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kbb), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

constexpr size_t kMaxDynSmem = 227 * 1024;   // per-CTA dynamic shared memory limit (sm_100)

constexpr size_t umma_smem_bytes(int bn, int stages, int kbb = kBK) {
    return 1024 + (size_t)stages * (kBM * kbb + bn * kbb) + 8 * 32 * 36 * 4 + (2 * stages + 4) * 8 + 16;
}

constexpr size_t splitk_smem_bytes(int bn, int stages) {
    // ring, barriers, then 32 bytes of slots and the rows' im2col scales
    return 1024 + (size_t)stages * (kBM * kBK + bn * kBK) + (2 * stages + 1) * 8 + 32 + kBM * 4;
}

// deepest ring that fits (capped at 8 stages)
constexpr int umma_max_stages(int bn) {
    int s = 8;
    while (s > 2 && umma_smem_bytes(bn, s) > kMaxDynSmem) --s;
    return s;
}
constexpr int splitk_max_stages(int bn) {
    int s = 8;
    while (s > 2 && splitk_smem_bytes(bn, s) > kMaxDynSmem) --s;
    return s;
}
// the split-K partial tile [128][bn + 4] int32 overlays the ring
constexpr int splitk_min_stages(int bn) {
    int s = 2;
    while ((size_t)s * (kBM * kBK + bn * kBK) < (size_t)kBM * (bn + 4) * 4) ++s;
    return s;
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

// cudaFuncSetAttribute is per device: one bit per device that has it. Every
// GEMM kernel may use up to the full dynamic shared memory; occupancy still
// follows the size each launch asks for.
template <typename Kern>
cudaError_t set_smem_attr_once(Kern kernel, std::atomic<unsigned long long>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kMaxDynSmem));
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

template <int BN, int KBB>
cudaError_t umma_ready() {
    static std::atomic<unsigned long long> done{0};
    return set_smem_attr_once(w8a8_umma_kernel<BN, KBB>, done);
}
template <int BN, bool GLOBAL = false>
cudaError_t splitk_ready() {
    static std::atomic<unsigned long long> done{0};
    return set_smem_attr_once(w8a8_splitk_kernel<BN, GLOBAL>, done);
}

// Persistent launch: at most (SMs x resident CTAs) CTAs, each looping over
// output tiles t = blockIdx.x, +gridDim.x, ...
template <int BN, int KBB = kBK>
cudaError_t launch_umma(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& p, int stages,
                        cudaStream_t st) {
    const size_t smem = umma_smem_bytes(BN, stages, KBB);
    cudaError_t e = umma_ready<BN, KBB>();
    if (e != cudaSuccess) return e;
    static std::atomic<int> per_sm[9];     // resident CTAs per SM (registers and shared memory), by stages
    int occ = per_sm[stages].load(std::memory_order_relaxed);
    if (!occ) {
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, w8a8_umma_kernel<BN, KBB>, kThreads, smem);
        if (occ <= 0) occ = 1;
        per_sm[stages].store(occ, std::memory_order_relaxed);
    }
    const long long tiles = (long long)((p.N + BN - 1) / BN) * p.m_tiles;
    const long long cap = (long long)sm_count() * occ;
    const int grid = static_cast<int>(tiles < cap ? tiles : cap);
    e = launch_k(w8a8_umma_kernel<BN, KBB>, grid, kThreads, smem, st, ta, tb, p, stages);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// How many clusters of `splits` split-K CTAs can be resident at once (the
// GPCs' SM counts, not just the SM total, bound this: a cluster lives in one
// GPC). Cached per device, cluster size and ring depth.
template <int BN>
int splitk_max_clusters(int splits, int stages) {
    static std::atomic<int> cache[64][9][9];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || splits < 2 || splits > 8 || stages < 2 || stages > 8) return 0;
    dev &= 63;
    int v = cache[dev][splits][stages].load(std::memory_order_relaxed);
    if (v) return v;
    if (splitk_ready<BN>() != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = splitk_smem_bytes(BN, stages);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&v, w8a8_splitk_kernel<BN, false>, &cfg) != cudaSuccess || v <= 0) {
        cudaGetLastError();
        return 0;
    }
    cache[dev][splits][stages].store(v, std::memory_order_relaxed);
    return v;
}

int splitk_clusters(int bn, int splits, int stages) {
    switch (bn) {
        case 32: return splitk_max_clusters<32>(splits, stages);
        case 64: return splitk_max_clusters<64>(splits, stages);
        case 256: return splitk_max_clusters<256>(splits, stages);
        default: return splitk_max_clusters<128>(splits, stages);
    }
}

// Split-K launch: grid (splits, tiles), clusters of `splits` CTAs.
template <int BN>
cudaError_t launch_splitk(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& p, int splits, int stages,
                          cudaStream_t st) {
    cudaError_t e = splitk_ready<BN>();
    if (e != cudaSuccess) return e;
    const long long tiles = (long long)((p.N + BN - 1) / BN) * p.m_tiles;
    if (tiles > 65535 || splits < 2 || splits > 8) return cudaErrorInvalidValue;
    e = launch_k_cluster(w8a8_splitk_kernel<BN, false>, dim3(splits, (unsigned)tiles), kThreads, dim3(splits, 1, 1),
                         splitk_smem_bytes(BN, stages), st, ta, tb, p, stages);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// Split-K over independent CTAs: grid (splits, tiles), no clusters; partial
// tiles meet in the caller's workspace (p.ws / p.counters).
template <int BN>
cudaError_t launch_splitk_global(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& p, int splits,
                                 int stages, cudaStream_t st) {
    cudaError_t e = splitk_ready<BN, true>();
    if (e != cudaSuccess) return e;
    const long long tiles = (long long)((p.N + BN - 1) / BN) * p.m_tiles;
    if (tiles > 65535 || splits < 2 || splits > kMaxGlobalSplits || !p.ws || !p.counters || p.m_tiles != 1 ||
        p.conv_bw)
        return cudaErrorInvalidValue;
    const size_t smem = splitk_smem_bytes(BN, stages);
    if (p.splitk_coop) {
        // every CTA reduces after all have written: a cooperative launch (whether
        // the driver takes it with programmatic dependent launch as well is found
        // on the first uncaptured launch and remembered)
        static std::atomic<int> with_pdl{-1};
        int wp = with_pdl.load(std::memory_order_relaxed);
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (wp < 0 && cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone) {
            e = launch_k_coop(w8a8_splitk_kernel<BN, true>, dim3(splits, (unsigned)tiles), kThreads, smem, st, true,
                              ta, tb, p, stages);
            if (e == cudaSuccess) {
                with_pdl.store(1, std::memory_order_relaxed);
                return cudaGetLastError();
            }
            cudaGetLastError();
            with_pdl.store(0, std::memory_order_relaxed);
            wp = 0;
        }
        e = launch_k_coop(w8a8_splitk_kernel<BN, true>, dim3(splits, (unsigned)tiles), kThreads, smem, st, wp > 0, ta,
                          tb, p, stages);
    } else {
        e = launch_k(w8a8_splitk_kernel<BN, true>, dim3(splits, (unsigned)tiles), kThreads, smem, st, ta, tb, p, stages);
    }
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

// fp32 [rows][cols] output map for TMA stores: box 32 x 32 (128-byte rows,
// 128-byte swizzle, the slab kernel's staging layout).
bool make_tmap_f32_out(CUtensorMap* map, const void* base, int rows, int cols, long long ld) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 3) || rows <= 0 || cols <= 0 || ld < cols) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
    const cuuint32_t box[2] = {32, 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// fp32 NHWC output [F][Ho][Wo][C] map for TMA stores: box {32 channels, 32
// pixels, 1, 1} with the 128-byte swizzle (the same staging tile layout).
bool make_tmap_f32_nhwc_out(CUtensorMap* map, const void* base, int F, int Ho, int Wo, int C) {
    auto fn = get_encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (C & 3) || F <= 0 || Ho <= 0 || Wo <= 0 || C <= 0) return false;
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(Wo), static_cast<cuuint64_t>(Ho),
                                static_cast<cuuint64_t>(F)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 4, static_cast<cuuint64_t>(Wo) * C * 4,
                                   static_cast<cuuint64_t>(Ho) * Wo * C * 4};
    const cuuint32_t box[4] = {32, 32, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

struct SlabPlan {
    int bn = 0;        // columns per CTA (a multiple of sl)
    int sl = 32;       // B slice rows = MMA N
    int stages = 1;    // B slices in flight
    int nstg = 2;      // staging tiles per epilogue warp
};

size_t slab_smem_bytes(int K, int bn, int sl, int stages, int nstg, int kbb = kBK) {
    const int nkb = (K + kbb - 1) / kbb;
    return 1024 + (size_t)nkb * kBM * kbb + (size_t)stages * nkb * sl * kbb + (size_t)8 * nstg * kSlabStgFloats * 4 +
           (size_t)2 * 4 * bn + 8 * (kSlabMaxKb + 2 * stages + kSlabMaxSlices + 1) + 16;   // TMEM slot, 3 flags
}

// Ring depth and staging tiles for a slab shape: as many B slices in flight
// as fit (all of them when they do), two staging tiles per warp when a warp
// stores more than one chunk. False when even one slice does not fit.
bool slab_fit(int K, SlabPlan* sp, int kbb = kBK) {
    if ((K + kbb - 1) / kbb > kSlabMaxKb) return false;
    const int nsl = sp->bn / sp->sl;
    const int chunks_per_warp = (sp->bn / 32 + 1) / 2;
    for (int nstg = chunks_per_warp > 1 ? 2 : 1; nstg >= 1; --nstg) {
        for (int st = nsl; st >= 1; --st) {
            if (slab_smem_bytes(K, sp->bn, sp->sl, st, nstg, kbb) <= kMaxDynSmem) {
                sp->stages = st;
                sp->nstg = nstg;
                return true;
            }
        }
    }
    return false;
}

// The slab kernel takes a plain GEMM (fp32 output through TMA stores, K <=
// 1024) when its output fits one wave: the narrowest multiple of 32 columns
// per CTA that needs at most one CTA per SM. VLA_GEMM_SLAB=0 turns it off,
// VLA_GEMM_SLAB=<bn>:<sl>[:<stages>] forces a shape; VLA_GEMM_PLAN (a forced
// persistent / split-K plan) also keeps GEMMs off it.
bool slab_plan(int M, int N, int K, SlabPlan* sp) {
    const int nkb = (K + kBK - 1) / kBK;
    if (nkb > 8 || M <= 0 || N <= 0) return false;   // plain GEMMs: K <= 1024
    const char* env = std::getenv("VLA_GEMM_SLAB");
    if (env && env[0] == '0' && env[1] == '\0') return false;
    const long long m_tiles = (M + kBM - 1) / kBM;
    if (env) {
        int bn = 0, sl = 0, st = 0;
        const int n = std::sscanf(env, "%d:%d:%d", &bn, &sl, &st);
        if (n >= 2 && (sl == 32 || sl == 64 || sl == 128) && bn >= sl && bn <= kSlabMaxBn && bn % sl == 0) {
            sp->bn = bn;
            sp->sl = sl;
            if (!slab_fit(K, sp)) return false;
            if (n == 3 && st >= 1 && st < sp->stages) sp->stages = st;
            return m_tiles * ((N + bn - 1) / bn) <= 0x7FFFFFFF;
        }
        return false;
    }
    if (std::getenv("VLA_GEMM_PLAN")) return false;
    // One MMA chain per CTA (slice = the whole slab): measured on the B200,
    // a 128 x 32 x 32 MMA chain runs at well under a quarter of the rate of a
    // 128 x 128 x 32 one (each step waits for the previous accumulation), so
    // narrow slices cost more in MMA time than their epilogue overlap returns.
    const long long sms = sm_count();
    for (int bn : {32, 64, 128}) {
        if (m_tiles * ((N + bn - 1) / bn) <= sms) {
            sp->bn = bn;
            sp->sl = bn;
            return slab_fit(K, sp);
        }
    }
    return false;
}

template <int SL, int KBB>
cudaError_t slab_ready() {
    static std::atomic<unsigned long long> done{0};
    return set_smem_attr_once(w8a8_slab_kernel<SL, KBB>, done);
}

template <int SL, int KBB = kBK>
cudaError_t launch_slab_sl(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const EpiParams& p,
                           const SlabPlan& sp, cudaStream_t st) {
    cudaError_t e = slab_ready<SL, KBB>();
    if (e != cudaSuccess) return e;
    const long long grid = (long long)p.m_tiles * p.slab_groups;
    const size_t smem = slab_smem_bytes(p.K, sp.bn, SL, sp.stages, sp.nstg, KBB);
    if (p.qout) {
        // the CTAs of an M tile wait for one another: a cooperative launch.
        // Whether the driver takes it together with programmatic dependent
        // launch is found on the first (uncaptured) launch and remembered.
        static std::atomic<int> with_pdl{-1};
        int wp = with_pdl.load(std::memory_order_relaxed);
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (wp < 0 && cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone) {
            e = launch_k_coop(w8a8_slab_kernel<SL, KBB>, dim3(static_cast<unsigned>(grid)), kThreads, smem, st, true,
                              ta, tb, to, p, sp.stages);
            if (e == cudaSuccess) {
                with_pdl.store(1, std::memory_order_relaxed);
                return cudaGetLastError();
            }
            cudaGetLastError();
            with_pdl.store(0, std::memory_order_relaxed);
            wp = 0;
        }
        e = launch_k_coop(w8a8_slab_kernel<SL, KBB>, dim3(static_cast<unsigned>(grid)), kThreads, smem, st, wp > 0,
                          ta, tb, to, p, sp.stages);
    } else {
        e = launch_k(w8a8_slab_kernel<SL, KBB>, dim3(static_cast<unsigned>(grid)), kThreads, smem, st, ta, tb, to, p,
                     sp.stages);
    }
    if (e != cudaSuccess) return e;
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
    p.m_tiles = (a.M + kBM - 1) / kBM;
    p.qout = a.qout;
    p.ldq = a.ldq;
    p.qscale = a.qscale;
    p.qamax = a.qamax;
    p.qsync = a.qsync;
    p.im_x = a.im_x;
    p.im_rowmax = a.im_rowmax;
    p.im_T = a.im_T;
    p.im_C = a.im_C;
    p.im_k = a.im_k;
    p.im_stride = a.im_stride;
    p.im_pad = a.im_pad;
    p.im_Tout = a.im_Tout;
    const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out), rb = reinterpret_cast<uintptr_t>(a.res);
    p.vec_ok = !(a.mode & kEpiAcc) && (ob & 15) == 0 && (a.ldo & 3) == 0 &&
               (!a.res || ((rb & 15) == 0 && (a.ldr & 3) == 0));
    return p;
}

}  // namespace

GemmPlan gemm_i8_plan(int M, int N, int K) {
    GemmPlan plan;
    const int nkb = (K + kBK - 1) / kBK;
    // VLA_GEMM_PLAN=<bn>:<splits>[:<stages>] forces one plan (tuning and tests)
    if (const char* e = std::getenv("VLA_GEMM_PLAN")) {
        int bn = 0, sp = 0, stg = 0;
        const int n = std::sscanf(e, "%d:%d:%d", &bn, &sp, &stg);
        if (n >= 2 && (bn == 32 || bn == 64 || bn == 128 || bn == 256) && sp >= 1 && sp <= 8) {
            plan.bn = bn;
            plan.splits = sp <= nkb ? sp : nkb;
            const int lo = plan.splits > 1 ? splitk_min_stages(bn) : 2;
            const int hi = plan.splits > 1 ? splitk_max_stages(bn) : umma_max_stages(bn);
            plan.stages = n == 3 ? (stg < lo ? lo : stg > hi ? hi : stg) : (plan.splits > 1 ? (lo > 4 ? lo : 4) : hi);
            return plan;
        }
    }
    // Cost model (relative units), fitted to device timings of every plan on
    // the ACT policy's GEMM shapes (graph-replayed launches on cold data):
    //   rounds x (k-blocks per CTA x bytes per k-block + output tile bytes)
    //   + for split K: a fixed cluster cost + the partial-tile exchange.
    // rounds = how many times the slowest SM runs a work unit.
    const int sms = sm_count();
    const int mt = (M + kBM - 1) / kBM;
    double best = 1e30;
    for (int bn : {32, 64, 128}) {
        const long long tiles = (long long)mt * ((N + bn - 1) / bn);
        for (int sp = 1; sp <= 8 && sp <= nkb; ++sp) {
            long long slots;
            int stages;
            if (sp == 1) {
                stages = 4;
                slots = sms;               // one persistent CTA per SM (register bound)
            } else {
                stages = splitk_min_stages(bn) > 4 ? splitk_min_stages(bn) : 4;
                if (tiles > 65535) continue;
                slots = (long long)splitk_clusters(bn, sp, stages) * sp;
                if (slots <= 0) continue;
            }
            const long long units = tiles * sp;
            const long long rounds = (units + slots - 1) / slots;
            const int kbc = (nkb + sp - 1) / sp;
            double cost = (double)rounds * ((double)kbc * (kBM * kBK + bn * kBK) + 4.0 * kBM * bn);
            if (sp > 1) cost += 31250.0 + 2.0 * 4.0 * kBM * bn * (sp - 1) / sp;
            if (cost < best) {
                best = cost;
                plan.bn = bn;
                plan.splits = sp;
                plan.stages = stages;
            }
        }
    }
    return plan;
}

cudaError_t gemm_i8_umma(const GemmI8Args& a, const CUtensorMap& ta, const CUtensorMap& tb, const GemmPlan& plan,
                         cudaStream_t st) {
    const EpiParams p = make_epi(a);
    const int bn = plan.bn;
    if (bn != 32 && bn != 64 && bn != 128 && bn != 256) return cudaErrorInvalidValue;
    if (plan.global) {
        if (plan.stages < splitk_min_stages(bn) || plan.stages > splitk_max_stages(bn)) return cudaErrorInvalidValue;
        EpiParams pg = p;
        pg.ws = a.splitk_ws;
        pg.counters = a.splitk_counters;
        // co-resident form: two counters per tile, and the whole grid at once
        // on the SMs (one CTA per SM at this ring depth)
        const long long tiles = (long long)((a.N + bn - 1) / bn);
        pg.splitk_coop = (2 * tiles <= a.splitk_counters_n && tiles * plan.splits <= sm_count()) ? 1 : 0;
        switch (bn) {
            case 32: return launch_splitk_global<32>(ta, tb, pg, plan.splits, plan.stages, st);
            case 64: return launch_splitk_global<64>(ta, tb, pg, plan.splits, plan.stages, st);
            case 256: return launch_splitk_global<256>(ta, tb, pg, plan.splits, plan.stages, st);
            default: return launch_splitk_global<128>(ta, tb, pg, plan.splits, plan.stages, st);
        }
    }
    if (plan.splits > 1) {
        if (plan.stages < splitk_min_stages(bn) || plan.stages > splitk_max_stages(bn)) return cudaErrorInvalidValue;
        switch (bn) {
            case 32: return launch_splitk<32>(ta, tb, p, plan.splits, plan.stages, st);
            case 64: return launch_splitk<64>(ta, tb, p, plan.splits, plan.stages, st);
            case 256: return launch_splitk<256>(ta, tb, p, plan.splits, plan.stages, st);
            default: return launch_splitk<128>(ta, tb, p, plan.splits, plan.stages, st);
        }
    }
    if (plan.stages < 2 || plan.stages > umma_max_stages(bn)) return cudaErrorInvalidValue;
    switch (bn) {
        case 32: return launch_umma<32>(ta, tb, p, plan.stages, st);
        case 64: return launch_umma<64>(ta, tb, p, plan.stages, st);
        case 256: return launch_umma<256>(ta, tb, p, plan.stages, st);
        default: return launch_umma<128>(ta, tb, p, plan.stages, st);
    }
}

bool gemm_i8_skinny_plan(const GemmI8Args& a, GemmPlan* plan) {
    // one 128-row M tile and a long K: the weights are the traffic. Spread the
    // (N tile, k-block) work over one CTA per SM, K split across independent
    // CTAs whose int32 partials meet in the caller's workspace.
    if (!a.splitk_ws || !a.splitk_counters || a.M > kBM || std::getenv("VLA_GEMM_PLAN")) return false;
    const int nkb = (a.K + kBK - 1) / kBK;
    const int bn = a.N >= 1024 ? 128 : a.N >= 256 ? 64 : 32;
    const int n_tiles = (a.N + bn - 1) / bn;
    int splits = sm_count() / n_tiles;
    if (splits > nkb / 2) splits = nkb / 2;      // at least two k-blocks per CTA
    if (splits > kMaxGlobalSplits) splits = kMaxGlobalSplits;
    if (nkb < 4 || splits < 2 || n_tiles > a.splitk_counters_n ||
        (long long)n_tiles * splits * a.M * bn > a.splitk_ws_elems)
        return false;
    plan->bn = bn;
    plan->splits = splits;
    plan->stages = splitk_max_stages(bn);
    plan->global = true;
    return true;
}

bool gemm_i8_rowq_supported(int M, int N, int K) {
    SlabPlan sp;
    if (M <= 0 || N <= 0 || N % 32 || !slab_plan(M, N, K, &sp)) return false;
    const long long grid = (long long)((M + kBM - 1) / kBM) * ((N + sp.bn - 1) / sp.bn);
    return grid <= sm_count();
}

// The row-quantized output (GemmI8Args::qout) on the slab kernel.
static cudaError_t gemm_i8_rowq(const GemmI8Args& a, cudaStream_t st) {
    const uintptr_t qb = reinterpret_cast<uintptr_t>(a.qout);
    if (!gemm_i8_rowq_supported(a.M, a.N, a.K) || a.ldq != a.N || (qb & 15) || (a.ldq & 15) || !a.qscale ||
        !a.qamax || !a.qsync || a.res || a.amax || (a.mode & ~kEpiRelu) || !a.ascale_per_row || a.force_simt ||
        ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) || (a.lda & 15) || (a.ldb & 15))
        return cudaErrorInvalidValue;
    SlabPlan sp;
    slab_plan(a.M, a.N, a.K, &sp);
    EpiParams p = make_epi(a);
    p.out = nullptr;
    p.slab_bn = sp.bn;
    p.slab_groups = (a.N + sp.bn - 1) / sp.bn;
    p.slab_nstg = sp.nstg;
    CUtensorMap ta, tb;
    if (!make_tmap_i8_kmajor(&ta, a.A, a.M, a.K, a.lda, kBM) || !make_tmap_i8_kmajor(&tb, a.B, a.N, a.K, a.ldb, sp.sl))
        return cudaErrorInvalidConfiguration;
    // the fp32 output map is never used on this path: the A map stands in
    switch (sp.sl) {
        case 64: return launch_slab_sl<64>(ta, tb, ta, p, sp, st);
        case 128: return launch_slab_sl<128>(ta, tb, ta, p, sp, st);
        default: return launch_slab_sl<32>(ta, tb, ta, p, sp, st);
    }
}

// Every N tile's CTAs quantize their own A rows, so the work repeats per N
// tile: worth the saved launch only for few rows. Measured on the Diffusion
// Policy U-Net: 16-row convs gain (batch 1: 5.10 -> 4.83 ms a query), 32-row
// ones lose (13.1 vs 10.1 us per launch), 128-row ones more (6.6 vs 5.9 ms).
constexpr int kIm2colMaxRows = 16;

static bool im2col_plan(const GemmI8Args& a, GemmPlan* plan) {
    if (!a.im_x || !a.im_rowmax || a.M > kIm2colMaxRows || a.im_C <= 0 || a.im_C % 16 || a.im_k <= 0 || a.im_T <= 0 || a.im_Tout <= 0 ||
        a.im_stride <= 0 || a.im_pad < 0 || (long long)a.im_k * a.im_C != a.K || a.M % a.im_Tout ||
        (a.mode & kEpiAcc) || a.qout || a.force_simt || (reinterpret_cast<uintptr_t>(a.im_x) & 15) ||
        (reinterpret_cast<uintptr_t>(a.B) & 15) || (a.ldb & 15))
        return false;
    *plan = gemm_i8_plan(a.M, a.N, a.K);
    return gemm_i8_skinny_plan(a, plan) && plan->global;
}

bool gemm_i8_takes_gemv(const GemmI8Args& a) {
    const bool tma_ok = ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) == 0 &&
                        (a.lda & 15) == 0 && (a.ldb & 15) == 0;
    return !a.im_x && !a.qout && !a.force_simt && tma_ok && a.M > 0 && a.M <= kGemvMaxRows && a.K % 16 == 0 &&
           a.K <= 2048;
}

bool gemm_i8_im2col_supported(const GemmI8Args& a) {
    GemmPlan plan;
    return a.M > 0 && a.N > 0 && a.K > 0 && im2col_plan(a, &plan);
}

cudaError_t gemm_i8(const GemmI8Args& a, cudaStream_t st) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return cudaErrorInvalidValue;
    if (a.im_x) {
        // the split-K kernel's epilogue warps build A; its map is never read
        GemmPlan plan;
        if (!im2col_plan(a, &plan)) return cudaErrorNotSupported;
        CUtensorMap tb;
        if (!make_tmap_i8_kmajor(&tb, a.B, a.N, a.K, a.ldb, plan.bn)) return cudaErrorInvalidConfiguration;
        return gemm_i8_umma(a, tb, tb, plan, st);
    }
    if (a.qout) return gemm_i8_rowq(a, st);
    const bool tma_ok = ((reinterpret_cast<uintptr_t>(a.A) | reinterpret_cast<uintptr_t>(a.B)) & 15) == 0 &&
                        (a.lda & 15) == 0 && (a.ldb & 15) == 0;
    if (gemm_i8_takes_gemv(a)) {
        // a few rows: the warp-per-column GEMV (latency: no tensor-core set-up)
        const EpiParams p = make_epi(a);
        const cudaError_t le_ = launch_k(w8a8_gemv_kernel, (a.N + 7) / 8, 256, 0, st, a.A, a.lda, a.B, a.ldb, p);
        if (le_ != cudaSuccess) return le_;
        return cudaGetLastError();
    }
    if (!a.force_simt && tma_ok) {
        // operands TMA can describe always take the tensor-core kernels; a tensor
        // map the driver refuses is an error, never a silent detour
        SlabPlan sp;
        const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out);
        if (!(a.mode & kEpiAcc) && (ob & 15) == 0 && (a.ldo & 3) == 0 && a.ldo >= a.N &&
            slab_plan(a.M, a.N, a.K, &sp)) {
            EpiParams p = make_epi(a);
            p.slab_bn = sp.bn;
            p.slab_groups = (a.N + sp.bn - 1) / sp.bn;
            p.slab_nstg = sp.nstg;
            CUtensorMap ta, tb, to;
            if (!make_tmap_i8_kmajor(&ta, a.A, a.M, a.K, a.lda, kBM) ||
                !make_tmap_i8_kmajor(&tb, a.B, a.N, a.K, a.ldb, sp.sl) ||
                !make_tmap_f32_out(&to, a.out, a.M, a.N, a.ldo))
                return cudaErrorInvalidConfiguration;
            switch (sp.sl) {
                case 64: return launch_slab_sl<64>(ta, tb, to, p, sp, st);
                case 128: return launch_slab_sl<128>(ta, tb, to, p, sp, st);
                default: return launch_slab_sl<32>(ta, tb, to, p, sp, st);
            }
        }
        GemmPlan plan = gemm_i8_plan(a.M, a.N, a.K);
        gemm_i8_skinny_plan(a, &plan);
        CUtensorMap ta, tb;
        if (!make_tmap_i8_kmajor(&ta, a.A, a.M, a.K, a.lda, kBM) ||
            !make_tmap_i8_kmajor(&tb, a.B, a.N, a.K, a.ldb, plan.bn))
            return cudaErrorInvalidConfiguration;
        return gemm_i8_umma(a, ta, tb, plan, st);
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

bool conv_i8_implicit_supported(int C, int k, int stride) {
    return stride == 1 && k >= 1 && C > 0 && C % 64 == 0;
}

cudaError_t conv_i8_implicit(const ConvI8Args& a, cudaStream_t st) {
    if (!a.x || !a.Wq || !a.fscale || !a.wscale || !a.out || a.F <= 0 || a.H <= 0 || a.W <= 0 || a.N <= 0 ||
        a.pad < 0 || !conv_i8_implicit_supported(a.C, a.k, 1))
        return cudaErrorInvalidValue;
    const int kw = a.kw > 0 ? a.kw : a.k;
    const int Ho = a.H + 2 * a.pad - a.k + 1, Wo = a.W + 2 * a.pad - kw + 1;
    const long long K = (long long)a.k * kw * a.C;
    if (Ho <= 0 || Wo <= 0 || K > INT_MAX / (255 * 127) || a.ldw < K || (a.ldw & 15) ||
        (long long)a.F * Ho * Wo >= (1LL << 31) || (long long)a.F * a.H * a.W * a.C >= (1LL << 40))
        return cudaErrorInvalidValue;
    // Output patch per 128-row tile: the width (power of two, or the whole
    // row) giving the fewest tiles; ties to the wider patch.
    int bw = 0, bh = 0;
    long long best = 0;
    for (int cw : {Wo, 128, 64, 32, 16, 8, 4, 2, 1}) {
        if (cw <= 0 || cw > 128) continue;
        const int ch = 128 / cw;
        const long long tiles = (long long)((Wo + cw - 1) / cw) * ((Ho + ch - 1) / ch);
        if (!bw || tiles < best) { best = tiles; bw = cw; bh = ch; }
    }
    const int kbb = a.C % 128 == 0 ? 128 : 64;
    EpiParams p{};
    p.out = a.out;
    p.ldo = a.N;
    p.res = a.res;
    p.ldr = a.N;
    p.ascale = a.fscale;
    p.wscale = a.wscale;
    p.bias = a.bias;
    p.amax = a.amax;
    p.amax_rows = Ho * Wo;
    p.mode = a.mode;
    p.M = a.F * Ho * Wo;
    p.N = a.N;
    p.K = static_cast<int>(K);
    p.static_weights = a.static_weights ? 1 : 0;
    const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out), rb = reinterpret_cast<uintptr_t>(a.res);
    p.vec_ok = !(a.mode & kEpiAcc) && (ob & 15) == 0 && (a.N & 3) == 0 && (!a.res || (rb & 15) == 0);
    p.conv_bw = bw;
    p.conv_bh = bh;
    p.conv_tx = (Wo + bw - 1) / bw;
    p.conv_ty = (Ho + bh - 1) / bh;
    p.conv_ho = Ho;
    p.conv_wo = Wo;
    p.conv_k = a.k;
    p.conv_kw = kw;
    p.conv_pad = a.pad;
    p.conv_cb = a.C / kbb;
    p.m_tiles = a.F * p.conv_ty * p.conv_tx;
    // 64-channel inputs with one wave or a few of output patches: the slab
    // kernel (the whole tap set of the patch and all weights resident, TMA-store
    // epilogue through a 4D output map; patch rows in runs of 32 pixels)
    {
        SlabPlan sp;
        sp.bn = a.N <= 128 ? (a.N + 31) / 32 * 32 : 0;
        sp.sl = sp.bn;
        const char* env = std::getenv("VLA_GEMM_SLAB");
        const bool off = (env && env[0] == '0') || std::getenv("VLA_GEMM_PLAN");
        const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out);
        if (!off && kbb == 64 && bw % 32 == 0 && (sp.bn == 32 || sp.bn == 64 || sp.bn == 128) && (a.N & 3) == 0 &&
            (ob & 15) == 0 && !(a.mode & kEpiAcc) && p.m_tiles <= 3LL * sm_count() && slab_fit((int)K, &sp, 64)) {
            p.slab_bn = sp.bn;
            p.slab_groups = (a.N + sp.bn - 1) / sp.bn;
            p.slab_nstg = sp.nstg;
            CUtensorMap ta, tb, to;
            if (!make_tmap_nhwc_i8(&ta, a.x, a.F, a.H, a.W, a.C, 64, bw, bh) ||
                !make_tmap_i8_kmajor_kb(&tb, a.Wq, a.N, static_cast<int>(K), a.ldw, sp.sl, 64) ||
                !make_tmap_f32_nhwc_out(&to, a.out, a.F, Ho, Wo, a.N))
                return cudaErrorInvalidConfiguration;
            switch (sp.sl) {
                case 32: return launch_slab_sl<32, 64>(ta, tb, to, p, sp, st);
                case 64: return launch_slab_sl<64, 64>(ta, tb, to, p, sp, st);
                default: return launch_slab_sl<128, 64>(ta, tb, to, p, sp, st);
            }
        }
    }
    GemmPlan plan;
    if (kbb == 64) {
        // 64-channel inputs: 64-byte k-blocks (one tap each), persistent kernel
        plan.bn = a.N >= 64 ? 64 : 32;
        plan.splits = 1;
        plan.stages = 8;
        if (const char* e = std::getenv("VLA_GEMM_PLAN")) {
            int bn = 0, sp = 0;
            if (std::sscanf(e, "%d:%d", &bn, &sp) >= 1 && (bn == 32 || bn == 64)) plan.bn = bn;
        }
    } else {
        plan = gemm_i8_plan(p.m_tiles * kBM, a.N, static_cast<int>(K));
    }
    CUtensorMap ta, tb;
    if (!make_tmap_nhwc_i8(&ta, a.x, a.F, a.H, a.W, a.C, kbb, bw, bh) ||
        !make_tmap_i8_kmajor_kb(&tb, a.Wq, a.N, static_cast<int>(K), a.ldw, plan.bn, kbb))
        return cudaErrorInvalidConfiguration;
    if (kbb == 64) {
        if (plan.bn == 32) return launch_umma<32, 64>(ta, tb, p, plan.stages, st);
        return launch_umma<64, 64>(ta, tb, p, plan.stages, st);
    }
    if (plan.splits > 1) {
        if (plan.stages < splitk_min_stages(plan.bn) || plan.stages > splitk_max_stages(plan.bn))
            return cudaErrorInvalidValue;
        switch (plan.bn) {
            case 32: return launch_splitk<32>(ta, tb, p, plan.splits, plan.stages, st);
            case 64: return launch_splitk<64>(ta, tb, p, plan.splits, plan.stages, st);
            case 256: return launch_splitk<256>(ta, tb, p, plan.splits, plan.stages, st);
            default: return launch_splitk<128>(ta, tb, p, plan.splits, plan.stages, st);
        }
    }
    if (plan.stages < 2 || plan.stages > umma_max_stages(plan.bn)) return cudaErrorInvalidValue;
    switch (plan.bn) {
        case 32: return launch_umma<32>(ta, tb, p, plan.stages, st);
        case 64: return launch_umma<64>(ta, tb, p, plan.stages, st);
        case 256: return launch_umma<256>(ta, tb, p, plan.stages, st);
        default: return launch_umma<128>(ta, tb, p, plan.stages, st);
    }
}

void* device_status_address() {
    void* p = nullptr;
    return cudaGetSymbolAddress(&p, g_vsb_status) == cudaSuccess ? p : nullptr;
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
