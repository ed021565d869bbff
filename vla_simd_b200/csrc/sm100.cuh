// Thin inline-PTX layer for the sm_100a features the kernels use: mbarriers,
// TMA tile loads (each CTA loads its own tiles), tcgen05 MMA /
// TMEM allocation / TMEM loads, and bounded waits.
//
// Every wait on an mbarrier is bounded by wall time (%globaltimer). A wait that
// runs out records a code in the device status word `g_vsb_status` and returns
// false; callers then skip the rest of their work (never __trap()), so a stuck
// pipeline ends the kernel with an error the host can read instead of hanging a
// shared GPU.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace vsb {

// Device status word, read by vsb_device_status() on the host. 0 == OK.
enum : int {
    kStatusOK = 0,
    kStatusWaitTimeout = 1,   // an mbarrier wait exceeded kWaitLimitNs
    kStatusBadShape = 2,      // a kernel saw a shape its launcher should have rejected
};

// Defined here: every kernel of the library is compiled in one translation
// unit (kernels.cu includes the .cu files), so there is exactly one copy.
__device__ int g_vsb_status = 0;

// 2 s: orders of magnitude above any legitimate wait in these kernels.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_status(int code) {
    atomicCAS(&g_vsb_status, 0, code);
}

// ------------------------------------------------------- exact conversions
// Small-range int <-> float conversions as two fma-pipe / integer operations
// instead of the conversion unit (the int8 quantizers round every element).
// Both are exact: adding 1.5 * 2^23 to a float rounds it to the nearest (even)
// integer, and an integer placed in the low mantissa bits of 1.5 * 2^23 reads
// back exactly.
constexpr float kRoundConst = 12582912.0f;   // 1.5 * 2^23, bits 0x4B400000

// round-to-nearest-even float -> int, for |x| <= 2^22 (callers clamp first)
__device__ __forceinline__ int f2i_rn_small(float x) {
    return __float_as_int(__fadd_rn(x, kRoundConst)) - 0x4B400000;
}

// small non-negative or signed int (|x| < 2^22) -> float, exact
__device__ __forceinline__ float i2f_small(int x) {
    return __fsub_rn(__int_as_float(x + 0x4B400000), kRoundConst);
}

// ------------------------------------------------ programmatic dependent launch
// Every kernel of the library is launched with programmatic stream
// serialization (launch.cuh): it may start while the previous kernel in the
// stream is still running. pdl_wait() blocks the calling thread until that
// kernel has completed and its memory is visible; each kernel calls it before
// touching anything a predecessor writes or reads (only constant weights and
// on-chip setup come before it). pdl_trigger() lets the next kernel be
// scheduled; it is safe anywhere, since a dependent only starts once every CTA
// of this grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ----------------------------------------------------------------- mbarrier --

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Wait for the phase with the given parity to complete, for at most
// kWaitLimitNs. Returns false (and records kStatusWaitTimeout) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        #pragma unroll 1
        for (int i = 0; i < 32; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            record_status(kStatusWaitTimeout);
            return false;
        }
    }
}

// The error path's wait: for a phase to complete or %globaltimer to pass
// deadline_ns, whichever comes first (nothing more is recorded). Used to let a
// CTA's own copies land before it leaves after another wait gave up.
__device__ __forceinline__ void mbar_wait_until(uint64_t* bar, uint32_t parity, uint64_t deadline_ns) {
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() > deadline_ns) return;
}

// ---------------------------------------------------------------------- TMA --

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tile load global -> this CTA's shared memory, completion counted in bytes
// on `bar`. x (innermost) must be a multiple of 16 bytes; callers pass k-block
// offsets that are multiples of 128.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
           "r"(x), "r"(y)
        : "memory");
}

// 3D tile load; x (innermost) a multiple of 16 bytes. y and z may start
// outside the tensor (those rows read zeros).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
           "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 4D tile load (implicit convolution: box {channels, W, H, 1} of an NHWC
// tensor); x = channel offset, a multiple of 16 bytes. Coordinates past the
// tensor (conv padding) read zeros.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z, int32_t w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];"
        :: "r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)),
           "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

// 2D tile store shared::cta -> global through a tensor map, tracked in this
// thread's bulk async-group. x (innermost) must be a multiple of 16 bytes and
// both coordinates non-negative; rows / columns past the tensor are not written.
// Every thread that wrote the source tile must have executed
// fence_proxy_async_smem() (and synchronized with the issuing thread) first.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y) : "memory");
}

// 4D tile store (an NHWC fp32 output: {channels, W, H, frame}); the same rules.
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int32_t x, int32_t y,
                                             int32_t z, int32_t w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Wait until at most N of this thread's committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(N) : "memory");
}

// Wait until every committed bulk group of this thread has completed (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Barrier over the `nthreads` threads (whole warps) that use named barrier `id` (1..15).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ tcgen05 --

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to *smem_slot. Whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(smem_slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (what a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes):
// rows of 128 bytes, 8-row atoms 1024 bytes apart (SBO), LBO unused (encoded 1),
// descriptor version 1, layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4)
         | (static_cast<uint64_t>(1u) << 16)
         | (static_cast<uint64_t>(1024u >> 4) << 32)
         | (static_cast<uint64_t>(1u) << 46)
         | (static_cast<uint64_t>(2u) << 61);
}

// The same for the 64-byte swizzle (CU_TENSOR_MAP_SWIZZLE_64B): rows of 64
// bytes, 8-row atoms 512 bytes apart, layout type 4 = SWIZZLE_64B.
__device__ __forceinline__ uint64_t sw64_kmajor_desc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4)
         | (static_cast<uint64_t>(1u) << 16)
         | (static_cast<uint64_t>(512u >> 4) << 32)
         | (static_cast<uint64_t>(1u) << 46)
         | (static_cast<uint64_t>(4u) << 61);
}

// Instruction descriptor, kind::i8: signed A and B, int32 accumulator, both
// operands K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_s8s8_s32(int M, int N) {
    return (2u << 4)                              // D format: S32
         | (1u << 7)                              // A: signed 8-bit
         | (1u << 10)                             // B: signed 8-bit
         | (static_cast<uint32_t>(N >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24); // M / 16
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_s8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive once on `bar` when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets TMEM lane
// (taddr.lane + i), columns [taddr.col, taddr.col + 32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---- thread-block clusters: distributed shared memory between the CTAs of a
// cluster (all of them are resident together by construction)
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// the shared-memory address `saddr` of this CTA, as seen in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

__device__ __forceinline__ int4 dsmem_ld_v4(uint32_t caddr) {
    int4 v;
    asm volatile("ld.shared::cluster.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(caddr) : "memory");
    return v;
}

}  // namespace vsb
