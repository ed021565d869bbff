// Slab W8A8 GEMM: one output slab per CTA, for GEMMs whose output fits one
// wave of CTAs (the policies' 100- to 602-row linears with K <= 1024).
//
// CTA = M tile mt (128 rows) x columns [n0, n0 + bn). The CTA's whole A tile
// (128 x K int8, at most 8 k-blocks of 128 bytes) is loaded once and stays in
// shared memory; B streams through a ring in slices of SL rows, each slice
// carrying all of K. Slice j's MMAs (tcgen05.mma M=128 N=SL K=32) accumulate
// into their own TMEM columns [j*SL, j*SL + SL) and commit on their own
// mbarrier, so the epilogue of slice j runs while later slices still load and
// multiply - the overlap a persistent kernel gets from a second tile, inside
// one tile. The epilogue is the reference's delayed-scaling
//   out[m,n] = fma((float)acc * s_w[n], s_a[m], bias[n])  (+ ReLU / residual)
// (src/hal/common/gemm_i8.cpp:278, src/hal/avx2/gemm_i8.cpp:101-104) with the
// same explicitly rounded intrinsics as the persistent kernel, so the bits are
// identical. Each thread owns one tile row (the TMEM lane it reads), so the
// row scale is one register and the absmax tap a per-thread maximum; results
// go through a 128-byte-swizzled 32 x 32 fp32 staging tile per warp
// (conflict-free 16-byte stores) and leave by TMA stores, which also clip the
// rows past M and the columns past N.
//   warp 0 lane 0: TMA producer (B slices first: load-time constants may be
//                  fetched before the predecessor kernel ends; then A)
//   warp 1:        TMEM allocation; lane 0 issues the MMAs slice by slice
//   warps 2-9:     epilogue; warp w takes TMEM lanes 32*(w%4).. and the
//                  32-column chunks g with g % 2 == (w-2)/4
//
// Implicit convolutions (p.conv_bw > 0) run through the same kernel: the A
// k-blocks are 4D tensor-map taps of the int8 NHWC input (load_a), a tile row
// is a pixel of the tile's output patch (out_row), and the stores go through a
// 4D output map [F][Ho][Wo][N] - each warp quarter's 32 tile rows are 32
// consecutive pixels of one output row (the host requires patch widths that
// are multiples of 32). KBB is the k-block width in bytes: 128 (128-byte
// swizzle) or 64 (64-byte swizzle, for 64-channel convolution inputs).
// Included by gemm_i8.cu inside its anonymous namespace (EpiParams, kBM, kBK,
// kUmmaK, kThreads, row_ascale, out_row, load_a, kmajor_desc come from there).

constexpr int kSlabMaxKb = 16;       // k-blocks of the resident A tile (K <= 1024 for plain GEMMs)
constexpr int kSlabMaxBn = 256;      // columns per CTA
constexpr int kSlabMaxSlices = kSlabMaxBn / 32;
constexpr int kSlabStgFloats = 32 * 32;   // one warp's staging tile: 32 rows x 128 bytes

// Row-quantized output (EpiParams::qout; plain GEMMs, mode 0 or ReLU, N a
// multiple of 32): pass 1 folds |v| of this thread's row over the CTA's columns
// into qamax[m]; the CTAs of the M tile meet at qsync[2 mt] (a cooperative
// launch: all are resident, the wait is bounded); pass 2 reloads the
// accumulators, recomputes v bit for bit and writes
// q = clamp(rne(v / s)), s = max(amax / 127, FLT_MIN) (quantize_rows'
// arithmetic, src/hal/common/gemm_i8.cpp:209-244 over the row's N values).
// The last CTA of the tile to leave (qsync[2 mt + 1]) zeroes the tile's qamax
// slots and both counters for the next launch.
// (rowq_scale / rowq_q8: gemm_i8.cu)

template <int SL>
__device__ __forceinline__ void slab_rowq_epilogue(const EpiParams& p, uint64_t* accfull, uint32_t tmem_base,
                                                   const float* s_ws, const float* s_bias, int q, int h, int lane,
                                                   int m, bool row_ok, float sa, int mt, int ng, int nch,
                                                   volatile int* s_qfail) {
    const bool relu = (p.mode & kEpiRelu) != 0;
    auto values = [&](int g, float (&v)[32]) -> bool {
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&accfull[(g * 32) / SL], 0))) return false;
        tc_fence_after();
        uint32_t acc[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + g * 32, acc);
        tmem_ld_wait();
        #pragma unroll
        for (int e = 0; e < 32; ++e) {
            const float t = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(acc[e])), s_ws[g * 32 + e]), sa,
                                      s_bias[g * 32 + e]);
            v[e] = (relu && t < 0.0f) ? 0.0f : t;                     // tcpu::relu (eltwise.cpp:213-214)
        }
        return true;
    };
    bool ok = true;
    float qmax = 0.0f;
    for (int g = h; g < nch; g += 2) {
        float v[32];
        if (!(ok = values(g, v))) break;
        #pragma unroll
        for (int e = 0; e < 32; ++e) qmax = fmaxf(qmax, fabsf(v[e]));
    }
    if (ok && row_ok) atomicMax(&p.qamax[m], __float_as_uint(qmax));
    __syncwarp();
    named_sync(1, 256);
    if (threadIdx.x == 64) {
        unsigned int* arrive = p.qsync + 2 * mt;
        int fail = 0;
        __threadfence();
        atomicAdd(arrive, 1u);
        const uint64_t t0 = globaltimer_ns();
        while (*reinterpret_cast<volatile unsigned int*>(arrive) < static_cast<unsigned>(p.slab_groups)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                record_status(kStatusWaitTimeout);
                fail = 1;
                break;
            }
        }
        __threadfence();
        *s_qfail = fail;
    }
    __syncwarp();
    named_sync(1, 256);
    if (ok && !*s_qfail) {
        const float sc = rowq_scale(row_ok ? __uint_as_float(__ldcg(p.qamax + m)) : 0.0f);
        const float inv = __fdiv_rn(1.0f, sc);
        const int n0 = ng * p.slab_bn;
        for (int g = h; g < nch; g += 2) {
            float v[32];
            if (!values(g, v)) break;
            if (!row_ok) continue;
            uint32_t w[8];
            #pragma unroll
            for (int i = 0; i < 8; ++i)
                w[i] = rowq_q8(v[4 * i], inv) | (rowq_q8(v[4 * i + 1], inv) << 8) |
                       (rowq_q8(v[4 * i + 2], inv) << 16) | (rowq_q8(v[4 * i + 3], inv) << 24);
            uint4* dst = reinterpret_cast<uint4*>(p.qout + (long long)m * p.ldq + n0 + g * 32);
            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        if (row_ok && ng == 0 && h == 0) p.qscale[m] = sc;
    }
    __syncwarp();
    named_sync(1, 256);
    if (threadIdx.x == 64) {
        unsigned int* depart = p.qsync + 2 * mt + 1;
        if (atomicAdd(depart, 1u) + 1 == static_cast<unsigned>(p.slab_groups)) {
            // the tile's last CTA to leave: every CTA of it has read qamax
            const int m0 = mt * kBM;
            for (int r = 0; r < kBM && m0 + r < p.M; ++r) p.qamax[m0 + r] = 0u;
            p.qsync[2 * mt] = 0u;
            *depart = 0u;
        }
    }
}

template <int SL, int KBB>
__global__ void __launch_bounds__(kThreads, 1)
w8a8_slab_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b,
                 const __grid_constant__ CUtensorMap tmap_out,
                 const EpiParams p, const int stages) {
    static_assert(SL == 32 || SL == 64 || SL == 128, "slice width");
    static_assert(KBB == 64 || KBB == 128, "k-block bytes");
    constexpr uint32_t kIdesc = idesc_s8s8_s32(kBM, SL);
    constexpr int kSliceKb = SL * KBB;          // bytes of one k-block of a B slice
    constexpr int kAKb = kBM * KBB;             // bytes of one k-block of the A tile
    const int nkb = (p.K + KBB - 1) / KBB;
    // bytes one A k-block brings in: a conv patch box may be under 128 rows
    const uint32_t a_tx = p.conv_bw ? static_cast<uint32_t>(KBB * p.conv_bw * p.conv_bh) : static_cast<uint32_t>(kAKb);
    const int slice_bytes = nkb * kSliceKb;
    const int bn = p.slab_bn;
    const int mt = blockIdx.x / p.slab_groups, ng = blockIdx.x - mt * p.slab_groups;
    const int m0 = mt * kBM, n0 = ng * bn;
    const int ncols = p.N - n0 < bn ? p.N - n0 : bn;    // >= 1 by construction of the grid
    const int nsl = (ncols + SL - 1) / SL;
    const int nch = (ncols + 31) / 32;
    const int nstg = p.slab_nstg;
    int tcols = 32;
    while (tcols < bn) tcols <<= 1;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // stays a shared-window pointer
    uint8_t* sA = smem;                                            // nkb x 16 KB
    uint8_t* sB = sA + nkb * kAKb;                                 // stages x slice_bytes
    float* stg = reinterpret_cast<float*>(sB + stages * slice_bytes);   // 8 warps x nstg x 4 KB
    float* s_ws = stg + 8 * nstg * kSlabStgFloats;                 // [bn] column scales
    float* s_bias = s_ws + bn;                                     // [bn] biases
    uint64_t* afull = reinterpret_cast<uint64_t*>(s_bias + bn);    // [kSlabMaxKb]
    uint64_t* bfull = afull + kSlabMaxKb;                          // [stages]
    uint64_t* bempty = bfull + stages;                             // [stages]
    uint64_t* accfull = bempty + stages;                           // [kSlabMaxSlices]
    uint64_t* mma_done = accfull + kSlabMaxSlices;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile int* s_bdone = reinterpret_cast<volatile int*>(tmem_slot + 1);   // B slices the MMA thread saw land
    volatile int* s_adone = s_bdone + 1;                                      // 1 once the whole A tile landed
    volatile int* s_qfail = s_adone + 1;                                      // row-quantized output: the tile wait gave up

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // On-chip set-up first: it touches nothing a predecessor kernel writes, so
    // under programmatic dependent launch it overlaps the predecessor's tail.
    if (threadIdx.x == 0) {
        for (int kb = 0; kb < nkb; ++kb) mbar_init(&afull[kb], 1);
        for (int s = 0; s < stages; ++s) { mbar_init(&bfull[s], 1); mbar_init(&bempty[s], 1); }
        for (int j = 0; j < nsl; ++j) mbar_init(&accfull[j], 1);
        mbar_init(mma_done, 1);
        *s_bdone = 0;
        *s_adone = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
        tma_prefetch_desc(&tmap_out);
    }
    if (warp == 1) tmem_alloc(tmem_slot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // The TMEM columns are held: the next kernel may be scheduled now.
    pdl_trigger();
    // weights that a predecessor kernel may still be writing: wait before any load
    if (!p.static_weights) pdl_wait();

    int b_issued = 0;
    bool a_issued = false;
    if (warp == 0) {
        if (lane == 0) {
            auto load_slice = [&](int j, int s) {
                mbar_arrive_expect_tx(&bfull[s], static_cast<uint32_t>(slice_bytes));
                for (int kb = 0; kb < nkb; ++kb)
                    tma_load_2d(sB + s * slice_bytes + kb * kSliceKb, &tmap_b, &bfull[s], kb * KBB, n0 + j * SL);
            };
            const int pre = nsl < stages ? nsl : stages;
            for (int j = 0; j < pre; ++j) load_slice(j, j);
            b_issued = pre;
            pdl_wait();   // A is the predecessor's output
            for (int kb = 0; kb < nkb; ++kb) {
                mbar_arrive_expect_tx(&afull[kb], a_tx);
                load_a<KBB>(p, &tmap_a, sA + kb * kAKb, &afull[kb], mt, kb);
            }
            a_issued = true;
            for (int j = pre; j < nsl; ++j) {
                const int s = j % stages;
                if (!mbar_wait(&bempty[s], ((j / stages) - 1) & 1)) break;
                load_slice(j, s);
                b_issued = j + 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool fail = false;
            for (int j = 0; j < nsl && !fail; ++j) {
                const int s = j % stages;
                if (!mbar_wait(&bfull[s], (j / stages) & 1)) break;
                *s_bdone = j + 1;
                tc_fence_after();
                const uint32_t b_addr = smem_u32(sB + s * slice_bytes);
                const uint32_t d_tmem = tmem_base + j * SL;
                for (int kb = 0; kb < nkb; ++kb) {
                    if (j == 0) {     // the first slice meets each A k-block as it lands
                        if (!mbar_wait(&afull[kb], 0)) { fail = true; break; }
                        tc_fence_after();
                    }
                    const uint32_t a_addr = smem_u32(sA + kb * kAKb);
                    #pragma unroll
                    for (int k = 0; k < KBB / kUmmaK; ++k)
                        umma_s8(d_tmem, kmajor_desc<KBB>(a_addr + k * kUmmaK),
                                kmajor_desc<KBB>(b_addr + kb * kSliceKb + k * kUmmaK), kIdesc, (kb | k) != 0);
                }
                if (fail) break;
                if (j == 0) *s_adone = 1;
                umma_commit(&bempty[s]);
                umma_commit(&accfull[j]);
            }
            // TMEM is released at the end: wait for every MMA issued above
            umma_commit(mma_done);
            mbar_wait(mma_done, 0);
        }
        __syncwarp();
    } else {
        const int q = warp & 3;            // TMEM lanes this warp may read: 32 * (warp id % 4)
        const int h = (warp - 2) >> 2;     // chunk parity
        for (int i = threadIdx.x - 64; i < bn; i += 256) {
            const int n = n0 + i;
            s_ws[i] = n < p.N ? p.wscale[n] : 0.0f;
            s_bias[i] = (n < p.N && p.bias) ? p.bias[n] : 0.0f;
        }
        named_sync(1, 256);
        pdl_wait();   // activation scales / residual: predecessor data
        // output row of this thread's tile row (-1: no output), and whether the
        // quarter's first row has one (then the quarter's store is issued)
        const int m = out_row(p, mt, q * 32 + lane);
        const bool row_ok = m >= 0;
        const bool quarter_live = __shfl_sync(0xFFFFFFFFu, m, 0) >= 0;   // warp-uniform
        // store origin of the quarter: plain GEMM (n, row); convolution the
        // pixel (ox, oy) of frame f of the quarter's first row
        int st_x = 0, st_y = m0 + q * 32, st_f = 0;
        if (p.conv_bw) {
            const int m_first = __shfl_sync(0xFFFFFFFFu, m, 0);
            const int per_f = p.conv_ho * p.conv_wo;
            st_f = m_first / per_f;
            const int rem = m_first - st_f * per_f;
            st_y = rem / p.conv_wo;
            st_x = rem - st_y * p.conv_wo;
        }
        const float sa = row_ok ? row_ascale(p, m) : 0.0f;
        const int mode = p.mode;
        const bool has_res = (mode & (kEpiAdd | kEpiAddRelu)) != 0;
        float* my_stg = stg + (warp - 2) * nstg * kSlabStgFloats;
        float rmax = 0.0f;
        int it = 0;
        if (p.qout) slab_rowq_epilogue<SL>(p, accfull, tmem_base, s_ws, s_bias, q, h, lane, m, row_ok, sa, mt, ng, nch, s_qfail);
        for (int g = h; !p.qout && quarter_live && g < nch; g += 2, ++it) {
            const int n = n0 + g * 32;
            const int nv = p.N - n < 32 ? p.N - n : 32;     // valid columns of the chunk
            // the residual row segment goes out before the accumulator wait
            float rv[32];
            if (has_res) {
                const float* rr = p.res + (long long)m * p.ldr + n;
                if (row_ok && nv == 32 && p.vec_ok) {
                    #pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float4 t = *reinterpret_cast<const float4*>(rr + 4 * c);
                        rv[4 * c] = t.x; rv[4 * c + 1] = t.y; rv[4 * c + 2] = t.z; rv[4 * c + 3] = t.w;
                    }
                } else {
                    #pragma unroll
                    for (int e = 0; e < 32; ++e) rv[e] = (row_ok && e < nv) ? rr[e] : 0.0f;
                }
            }
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(&accfull[(g * 32) / SL], 0))) break;
            tc_fence_after();
            uint32_t acc[32];
            tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + g * 32, acc);
            tmem_ld_wait();
            float v[32];
            #pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 w4 = *reinterpret_cast<const float4*>(s_ws + g * 32 + 4 * c);
                const float4 b4 = *reinterpret_cast<const float4*>(s_bias + g * 32 + 4 * c);
                const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
                #pragma unroll
                for (int e = 0; e < 4; ++e)
                    v[4 * c + e] = __fmaf_rn(__fmul_rn(__int2float_rn(static_cast<int32_t>(acc[4 * c + e])), wv[e]),
                                             sa, bv[e]);
            }
            if (mode & kEpiRelu) {                                       // tcpu::relu (eltwise.cpp:213-214)
                #pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = v[e] < 0.0f ? 0.0f : v[e];
            }
            if (mode & kEpiAdd) {                                        // x[i] += y[i]
                #pragma unroll
                for (int e = 0; e < 32; ++e) v[e] = __fadd_rn(rv[e], v[e]);
            }
            if (mode & kEpiAddRelu) {                                    // resnet_backbone.cpp:293-295
                #pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const float t = __fadd_rn(v[e], rv[e]);
                    v[e] = t > 0.0f ? t : 0.0f;
                }
            }
            if (p.amax) {
                #pragma unroll
                for (int e = 0; e < 32; ++e) rmax = fmaxf(rmax, e < nv ? fabsf(v[e]) : 0.0f);
            }
            // staging tile: its previous TMA store must have finished reading it
            float* sb = my_stg + (it % nstg) * kSlabStgFloats;
            if (it >= nstg) {
                if (lane == 0) {
                    if (nstg == 2) bulk_wait_read<1>();
                    else bulk_wait_read<0>();
                }
                __syncwarp();
            }
            // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
            #pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<float4*>(sb + lane * 32 + ((c ^ (lane & 7)) << 2)) =
                    make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (p.conv_bw) tma_store_4d(&tmap_out, sb, n, st_x, st_y, st_f);
                else tma_store_2d(&tmap_out, sb, n, st_y);
                bulk_commit();
            }
        }
        if (lane == 0) bulk_wait_read<0>();   // the staging tiles must outlive the stores' reads
        __syncwarp();
        if (p.amax && quarter_live) {
            // one atomic per warp when its rows share a slot, else one per row
            const unsigned key = row_ok ? static_cast<unsigned>(m / p.amax_rows) : 0xFFFFFFFFu;
            const unsigned k0 = __shfl_sync(0xFFFFFFFFu, key, 0);      // lane 0's row is always live
            if (__all_sync(0xFFFFFFFFu, key == k0 || key == 0xFFFFFFFFu)) {
                float wm = row_ok ? rmax : 0.0f;
                #pragma unroll
                for (int off = 16; off > 0; off >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xFFFFFFFFu, wm, off));
                if (lane == 0) atomicMax(&p.amax[k0], __float_as_uint(wm));
            } else if (row_ok) {
                atomicMax(&p.amax[key], __float_as_uint(rmax));
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        // never leave the CTA with TMA writes still landing in its shared memory
        for (int j = *s_bdone; j < b_issued; ++j)
            if (!mbar_wait(&bfull[j % stages], (j / stages) & 1)) break;
        if (a_issued && !*s_adone)
            for (int kb = 0; kb < nkb; ++kb)
                if (!mbar_wait(&afull[kb], 0)) break;
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, tcols);
    }
}
