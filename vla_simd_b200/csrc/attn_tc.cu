// Tensor-core attention (opt-in: VLA_ATT_TC=1): QK^T and PV on the 5th-gen
// tensor cores (tcgen05.mma kind::tf32) in split precision, the online
// softmax in registers, no score matrix outside the SM.
//
// Why it is not the default: the policies' parity is bit-identity with the
// reference's CPU attention (an fp32 fma chain over d, then its Cephes exp and
// 8 in-order lane sums, src/hal/avx2/attn.cpp:134-251), which the exact kernels
// of nn.cu reproduce. Any other summation order moves scores by an ulp or so,
// and upstream of an int8 quantizer an ulp can flip a code. This kernel is the
// measured alternative; tests/test_attention_tc_gpu.py records what it does
// to the actions.
//
// Split precision (3xTF32): a tcgen05 tf32 MMA reads the top 19 bits of each
// fp32 operand. Each operand x becomes hi = x with the low 13 mantissa bits
// cleared (exact in tf32) and lo = x - hi (exact in fp32); a.b is then
// hi_a.hi_b + hi_a.lo_b + lo_a.hi_b, three MMAs into one fp32 accumulator,
// dropping lo_a.lo_b (2^-22 relative) and lo's own truncation (2^-21
// relative of the product at most).
//
// CTA = 128 query rows of one head (thread = row = TMEM lane; 4 warps, one per
// TMEM lane quarter), keys in blocks of 64:
//   K block -> hi/lo tiles (row = key, K-major over d); V block -> hi/lo tiles
//   of V^T (row = d, K-major over keys), both with the 128-byte swizzle;
//   S = Q K^T  (M=128, N=64, K=64: 3 x 8 MMAs) into TMEM columns [0, 64);
//   thread r: s = S[r,:] * scale (+ mask), running max m, p = exp(s - m)
//   (the reference's Cephes exp), running sum l, rescale factor alpha; p ->
//   hi/lo tiles (row = query, K-major over keys);
//   O_blk = P V (M=128, N=64, K=64: 3 x 8 MMAs) into TMEM columns [64, 128);
//   thread r: o = o * alpha + O_blk[r,:] in registers.
// Finally o / l, or the mean of V for a row whose every key is blocked (the
// reference's uniform-weights rule). Rows past seq_q and keys past seq_k are
// zero tiles, the latter masked to -inf.
//
// Key split: a query tile's key blocks are divided among the `splits` CTAs
// of a thread-block cluster (so a small head count still fills the SMs); each
// CTA leaves its running (m, l, o) per row in shared memory and, after a
// cluster barrier, finalizes rows r with r % splits == its rank by merging
// the partial states through distributed shared memory:
//   M = max m_i,  o = sum o_i exp(m_i - M),  l = sum l_i exp(m_i - M).
#include "sm100.cuh"
#include "launch.cuh"
#include "nn.h"

#include <atomic>
#include <cfloat>
#include <cstdlib>

namespace vsb {

namespace {

constexpr int kTcRows = 128;     // query rows per CTA
constexpr int kTcKeys = 64;      // keys per block
constexpr int kTcThreads = 128;
constexpr uint32_t kTcQBytes = kTcRows * kAttD * 4;    // one hi or lo Q / P tile: 32 KB
constexpr uint32_t kTcKBytes = kTcKeys * kAttD * 4;    // one hi or lo K / V^T tile: 16 KB
constexpr size_t kTcSmem = 1024 + 4 * (size_t)kTcQBytes + 4 * (size_t)kTcKBytes + 64;

// kind::tf32 instruction descriptor: F32 accumulator, TF32 A and B, both K-major
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Byte offset of fp32 element (r, k) of a K-major tile of R rows with the
// 128-byte swizzle: k-blocks of 32 floats (128 bytes per row), 8-row atoms of
// 1024 bytes, 16-byte chunk c of row r at chunk c ^ (r % 8).
__device__ __forceinline__ uint32_t sw_off(int r, int k, int R) {
    return static_cast<uint32_t>((k >> 5) * (R * 128) + (r >> 3) * 1024 + (r & 7) * 128 +
                                 ((((k >> 2) & 7) ^ (r & 7)) << 4) + ((k & 3) << 2));
}

__device__ __forceinline__ float tf32_hi(float x) { return __int_as_float(__float_as_int(x) & 0xFFFFE000); }

__device__ __forceinline__ void put_split4(uint8_t* hi, uint8_t* lo, uint32_t off, float4 v) {
    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
    *reinterpret_cast<float4*>(hi + off) = h;
    *reinterpret_cast<float4*>(lo + off) =
        make_float4(__fsub_rn(v.x, h.x), __fsub_rn(v.y, h.y), __fsub_rn(v.z, h.z), __fsub_rn(v.w, h.w));
}

__global__ void __launch_bounds__(kTcThreads, 1)
attention_tc_kernel(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                    float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, float scale,
                    const float* mask, const AttBatch bs, const int splits) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared-window pointer
    uint8_t* sQh = sm;
    uint8_t* sQl = sQh + kTcQBytes;
    uint8_t* sPh = sQl + kTcQBytes;
    uint8_t* sPl = sPh + kTcQBytes;
    uint8_t* sKh = sPl + kTcQBytes;
    uint8_t* sKl = sKh + kTcKBytes;
    uint8_t* sVh = sKl + kTcKBytes;
    uint8_t* sVl = sVh + kTcKBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(sVl + kTcKBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int rank = blockIdx.x % splits;                  // rank in the cluster (clusters run along x)
    const int q0 = (blockIdx.x / splits) * kTcRows, h = blockIdx.y, kvh = h / (n_q / n_kv);
    VSB_ATT_BATCH_OFFSET(bs);

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) tmem_alloc(tslot, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tS = *tslot, tO = *tslot + kTcKeys;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    pdl_trigger();   // after the TMEM allocation: a dependent may now take the rest
    pdl_wait();      // Q / K / V come from the previous kernels

    // Q tile, split once
    for (int i = tid; i < kTcRows * (kAttD / 4); i += kTcThreads) {
        const int r = i >> 4, c4 = i & 15;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (q0 + r < seq_q) v = *reinterpret_cast<const float4*>(Q + (long long)(q0 + r) * ldq + h * kAttD + 4 * c4);
        put_split4(sQh, sQl, sw_off(r, 4 * c4, kTcRows), v);
    }

    constexpr uint32_t kIdesc = idesc_tf32(kTcRows, kTcKeys);   // both GEMMs: M=128, N=64
    const int row = q0 + tid;
    const bool row_ok = row < seq_q;
    const float* mrow = (mask && row_ok) ? mask + (long long)row * seq_k : nullptr;
    float o[kAttD];
    #pragma unroll
    for (int d = 0; d < kAttD; ++d) o[d] = 0.0f;
    float m = -INFINITY, l = 0.0f;
    uint32_t phase = 0;
    bool ok = true;
    const int nblk_all = (seq_k + kTcKeys - 1) / kTcKeys;
    const int blk_lo = static_cast<int>((long long)nblk_all * rank / splits);
    const int blk_hi = static_cast<int>((long long)nblk_all * (rank + 1) / splits);
    for (int blk = blk_lo; blk < blk_hi && ok; ++blk) {
        const int k0 = blk * kTcKeys;
        // K block (row = key) and V^T block (row = d), split
        for (int i = tid; i < kTcKeys * (kAttD / 4); i += kTcThreads) {
            const int kr = i >> 4, c4 = i & 15;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (k0 + kr < seq_k) {
                kv = *reinterpret_cast<const float4*>(K + (long long)(k0 + kr) * ldk + kvh * kAttD + 4 * c4);
                vv = *reinterpret_cast<const float4*>(V + (long long)(k0 + kr) * ldv + kvh * kAttD + 4 * c4);
            }
            put_split4(sKh, sKl, sw_off(kr, 4 * c4, kTcKeys), kv);
            const float ve[4] = {vv.x, vv.y, vv.z, vv.w};
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t off = sw_off(4 * c4 + e, kr, kAttD);
                const float hv = tf32_hi(ve[e]);
                *reinterpret_cast<float*>(sVh + off) = hv;
                *reinterpret_cast<float*>(sVl + off) = __fsub_rn(ve[e], hv);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            // S = Qh Kh^T + Qh Kl^T + Ql Kh^T
            uint32_t acc = 0;
            #pragma unroll 1
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t a = smem_u32(pass == 2 ? sQl : sQh), b = smem_u32(pass == 1 ? sKl : sKh);
                #pragma unroll
                for (int kb = 0; kb < kAttD / 32; ++kb)
                    #pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        umma_tf32(tS, sw128_kmajor_desc(a + kb * (kTcRows * 128) + 32 * ks),
                                  sw128_kmajor_desc(b + kb * (kTcKeys * 128) + 32 * ks), kIdesc, acc);
                        acc = 1;
                    }
            }
            umma_commit(bar);
        }
        ok = __syncthreads_and(mbar_wait(bar, phase)) != 0;
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        float s[kTcKeys];
        {
            uint32_t raw[32];
            #pragma unroll
            for (int half = 0; half < 2; ++half) {
                tmem_ld_32x32b_x32(tS + lane_base + 32 * half, raw);
                tmem_ld_wait();
                #pragma unroll
                for (int j = 0; j < 32; ++j) s[32 * half + j] = __uint_as_float(raw[j]);
            }
        }
        float mb = -INFINITY;
        #pragma unroll
        for (int j = 0; j < kTcKeys; ++j) {
            float v = __fmul_rn(s[j], scale);
            if (k0 + j >= seq_k) v = -INFINITY;
            else if (mrow) v = __fadd_rn(v, mrow[k0 + j]);
            s[j] = v;
            mb = fmaxf(mb, v);
        }
        const float mn = fmaxf(m, mb);
        const bool live = mn != -INFINITY;
        const float alpha = live ? ref_exp(__fsub_rn(m, mn)) : 1.0f;   // exp(-inf) = 0 on the first live block
        float ps = 0.0f;
        #pragma unroll
        for (int c = 0; c < kTcKeys / 4; ++c) {
            float4 p4;
            float* pe = reinterpret_cast<float*>(&p4);
            #pragma unroll
            for (int e = 0; e < 4; ++e) {
                pe[e] = live ? ref_exp(__fsub_rn(s[4 * c + e], mn)) : 0.0f;
                ps = __fadd_rn(ps, pe[e]);
            }
            put_split4(sPh, sPl, sw_off(tid, 4 * c, kTcRows), p4);
        }
        l = __fmaf_rn(l, alpha, ps);
        m = mn;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            // O_blk = Ph Vh + Ph Vl + Pl Vh
            uint32_t acc = 0;
            #pragma unroll 1
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t a = smem_u32(pass == 2 ? sPl : sPh), b = smem_u32(pass == 1 ? sVl : sVh);
                #pragma unroll
                for (int kb = 0; kb < kTcKeys / 32; ++kb)
                    #pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        umma_tf32(tO, sw128_kmajor_desc(a + kb * (kTcRows * 128) + 32 * ks),
                                  sw128_kmajor_desc(b + kb * (kAttD * 128) + 32 * ks), kIdesc, acc);
                        acc = 1;
                    }
            }
            umma_commit(bar);
        }
        ok = __syncthreads_and(mbar_wait(bar, phase)) != 0;
        phase ^= 1;
        if (!ok) break;
        tc_fence_after();
        {
            uint32_t raw[32];
            #pragma unroll
            for (int half = 0; half < 2; ++half) {
                tmem_ld_32x32b_x32(tO + lane_base + 32 * half, raw);
                tmem_ld_wait();
                #pragma unroll
                for (int j = 0; j < 32; ++j) o[32 * half + j] = __fmaf_rn(o[32 * half + j], alpha, __uint_as_float(raw[j]));
            }
        }
        tc_fence_before();
        __syncthreads();   // S / O columns and the K / V / P tiles are rewritten next block
    }

    if (splits > 1) {
        // this CTA's partial state per row -> shared memory (the P tiles are
        // free: the last P.V MMA completed before the loop's final barrier)
        constexpr int kPs = kAttD + 4;   // o[64], m, l, 2 pad: 16-byte rows
        float* part = reinterpret_cast<float*>(sPh);
        #pragma unroll
        for (int c = 0; c < kAttD / 4; ++c)
            *reinterpret_cast<float4*>(part + tid * kPs + 4 * c) = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
        part[tid * kPs + kAttD] = m;
        part[tid * kPs + kAttD + 1] = l;
        cluster_sync();
        if (tid % splits == rank) {
            const uint32_t base = smem_u32(part + tid * kPs);
            float mi[8], li[8];
            float M = -INFINITY;
            for (int i = 0; i < splits; ++i) {
                const int4 ml = dsmem_ld_v4(dsmem_map(base + kAttD * 4, static_cast<uint32_t>(i)));
                mi[i] = __int_as_float(ml.x);
                li[i] = __int_as_float(ml.y);
                M = fmaxf(M, mi[i]);
            }
            float L = 0.0f;
            #pragma unroll
            for (int d = 0; d < kAttD; ++d) o[d] = 0.0f;
            if (M != -INFINITY) {
                for (int i = 0; i < splits; ++i) {
                    const float w = mi[i] == -INFINITY ? 0.0f : ref_exp(__fsub_rn(mi[i], M));
                    L = __fmaf_rn(li[i], w, L);
                    #pragma unroll
                    for (int c = 0; c < kAttD / 4; ++c) {
                        const int4 v = dsmem_ld_v4(dsmem_map(base + 16 * c, static_cast<uint32_t>(i)));
                        o[4 * c] = __fmaf_rn(__int_as_float(v.x), w, o[4 * c]);
                        o[4 * c + 1] = __fmaf_rn(__int_as_float(v.y), w, o[4 * c + 1]);
                        o[4 * c + 2] = __fmaf_rn(__int_as_float(v.z), w, o[4 * c + 2]);
                        o[4 * c + 3] = __fmaf_rn(__int_as_float(v.w), w, o[4 * c + 3]);
                    }
                }
            }
            m = M;
            l = L;
        }
        cluster_sync();   // no CTA leaves while another still reads its partial rows
    }
    if (ok && row_ok && tid % splits == rank) {
        float* orow = O + (long long)row * ldo + h * kAttD;
        if (!(m > -FLT_MAX)) {
            // every key blocked: uniform weights over all keys (the mean of V)
            const float u = __fdiv_rn(1.0f, (float)seq_k);
            #pragma unroll
            for (int d = 0; d < kAttD; ++d) o[d] = 0.0f;
            for (int j = 0; j < seq_k; ++j) {
                const float* vr = V + (long long)j * ldv + kvh * kAttD;
                #pragma unroll
                for (int d = 0; d < kAttD; ++d) o[d] = __fmaf_rn(u, vr[d], o[d]);
            }
        } else {
            const float inv = __fdiv_rn(1.0f, l);
            #pragma unroll
            for (int d = 0; d < kAttD; ++d) o[d] = __fmul_rn(o[d], inv);
        }
        #pragma unroll
        for (int c = 0; c < kAttD / 4; ++c)
            *reinterpret_cast<float4*>(orow + 4 * c) = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tS, 128);
    }
}

}  // namespace

bool attention_tc_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("VLA_ATT_TC");
        return e && e[0] == '1';
    }();
    return on;
}

cudaError_t attention_tc(const float* Q, long long ldq, const float* K, long long ldk, const float* V, long long ldv,
                         float* O, long long ldo, int seq_q, int seq_k, int n_q, int n_kv, float scale,
                         const float* mask, const AttBatch& bs, cudaStream_t st) {
    static std::atomic<unsigned long long> ready{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(ready.load() & bit)) {
        e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kTcSmem));
        if (e != cudaSuccess) return e;
        ready.fetch_or(bit);
    }
    // key split: as many CTAs per query tile (a cluster, up to 8) as keep the
    // grid within one CTA per SM, and at least one 64-key block each
    const long long tiles = (long long)((seq_q + kTcRows - 1) / kTcRows) * n_q * bs.n;
    const int nblk = (seq_k + kTcKeys - 1) / kTcKeys;
    int splits = static_cast<int>(148 / (tiles > 0 ? tiles : 1));
    if (splits > 8) splits = 8;
    if (splits > nblk) splits = nblk;
    if (splits < 1) splits = 1;
    const dim3 grid(static_cast<unsigned>((seq_q + kTcRows - 1) / kTcRows * splits), n_q, bs.n);
    if (splits > 1)
        e = launch_k_cluster(attention_tc_kernel, grid, kTcThreads, dim3(splits, 1, 1), kTcSmem, st, Q, ldq, K, ldk,
                             V, ldv, O, ldo, seq_q, seq_k, n_q, n_kv, scale, mask, bs, splits);
    else
        e = launch_k(attention_tc_kernel, grid, kTcThreads, kTcSmem, st, Q, ldq, K, ldk, V, ldv, O, ldo, seq_q, seq_k,
                     n_q, n_kv, scale, mask, bs, splits);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace vsb
