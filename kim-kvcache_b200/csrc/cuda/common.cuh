// Device-side helpers shared by the sm_100a kernels: PTX wrappers for
// mbarriers, TMA (cp.async.bulk / cp.async.bulk.tensor, never with
// .multicast), tcgen05 (TMEM alloc, MMA, commit, loads), thread-block
// clusters and programmatic dependent launch, plus bounded waits.
//
// Every wait in these kernels is bounded: a wait that exceeds its poll budget
// records an error code in the module's status word and returns false, so a
// kernel can never spin forever on a barrier that will not complete.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace kk {

// Error codes written into a module status word (first error wins).
enum DeviceError : unsigned int {
    kErrNone = 0,
    kErrWaitTimeout = 1,      // an mbarrier wait ran out of polls
    kErrBadDescriptor = 2,    // a page descriptor pointed outside its pool
    kErrBadArgument = 3,
};

// A wait gives up after this much wall time (read from %globaltimer) or this
// many polls, whichever comes first.
constexpr std::uint64_t kWaitLimitNs = 2000000000ull;
constexpr std::uint32_t kMaxWaitPolls = 1u << 26;

__device__ __forceinline__ std::uint32_t smem_u32(void const* p)
{
    return static_cast<std::uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void pdl_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void pdl_launch_dependents()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(std::uint64_t* bar, std::uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(std::uint64_t* bar, std::uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(std::uint64_t* bar, std::uint32_t phase)
{
    std::uint32_t done = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ std::uint64_t global_ns()
{
    std::uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// 16-byte read-only global load issued where it stands in the program (a
// plain __ldg of constant data may be sunk by the compiler to its first
// use, which puts its latency after any wait in between).
__device__ __forceinline__ uint4 ldg_u4_now(void const* p)
{
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

#ifdef KK_TRACE
// Phase trace, compiled only into instrumented builds (-DKK_TRACE): each CTA
// of an instrumented kernel fills one record with %globaltimer stamps of its
// phases. Each translation unit keeps its own record array and exports a
// reader (kk_trace_read_*).
struct TraceRec {
    std::uint32_t tag;    // kernel kind and layer
    std::uint32_t block;  // blockIdx.y << 16 | blockIdx.x
    std::uint32_t smid;
    std::uint32_t aux;
    std::uint64_t t[16];
};
constexpr std::uint32_t kTraceCap = 1u << 16;

__device__ __forceinline__ std::uint32_t sm_id()
{
    std::uint32_t r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
#endif

// Potentially suspending test of an mbarrier phase: the thread sleeps in
// hardware until the phase completes or a short system time limit passes,
// instead of spinning through issue slots.
__device__ __forceinline__ bool mbar_try_wait_suspend(std::uint64_t* bar, std::uint32_t phase)
{
    std::uint32_t done = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return done != 0;
}

// The poll of the bounded pipeline waits: suspending by default; the
// KK_MBAR_SPIN tuning variant polls without suspending.
__device__ __forceinline__ bool mbar_poll(std::uint64_t* bar, std::uint32_t phase)
{
#ifdef KK_MBAR_SPIN
    return mbar_try_wait(bar, phase);
#else
    return mbar_try_wait_suspend(bar, phase);
#endif
}

// Bounded wait on an mbarrier phase (polls limited by wall time and poll
// count). Returns false, and records the error, when it gives up.
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, std::uint32_t phase,
    unsigned int* status)
{
    if (mbar_poll(bar, phase)) {
        return true;
    }
    std::uint64_t const t0 = global_ns();
    for (std::uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        if (mbar_poll(bar, phase)) {
            return true;
        }
        if (global_ns() - t0 > kWaitLimitNs) {
            break;
        }
    }
    if (status != nullptr) {
        atomicCAS(status, kErrNone, kErrWaitTimeout);
    }
    return false;
}

// The same bounded wait polling without suspending the thread, for a wait
// that is expected to end within a few hundred nanoseconds and sits on the
// critical path (a suspended thread wakes up late).
__device__ __forceinline__ bool mbar_wait_spin(std::uint64_t* bar, std::uint32_t phase,
    unsigned int* status)
{
    if (mbar_try_wait(bar, phase)) {
        return true;
    }
    std::uint64_t const t0 = global_ns();
    for (std::uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        if (mbar_try_wait(bar, phase)) {
            return true;
        }
        if ((i & 255u) == 255u && global_ns() - t0 > kWaitLimitNs) {
            break;
        }
    }
    if (status != nullptr) {
        atomicCAS(status, kErrNone, kErrWaitTimeout);
    }
    return false;
}

// ---- TMA (no multicast anywhere) -------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, CUtensorMap const* map,
    std::uint64_t* bar, int x, int y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(smem_u32(bar)),
        "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, CUtensorMap const* map,
    std::uint64_t* bar, int x, int y, std::uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(smem_u32(bar)),
        "r"(x), "r"(y), "l"(policy)
        : "memory");
}

// Untiled bulk copy global -> shared (no multicast): size and both addresses
// must be multiples of 16 bytes.
__device__ __forceinline__ void bulk_load_hint(void* dst, void const* src, std::uint32_t bytes,
    std::uint64_t* bar, std::uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(src)), "r"(bytes),
        "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ std::uint64_t l2_policy_evict_first()
{
    std::uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
    return policy;
}

// Asks L2 to fetch [src, src + bytes) from DRAM: no shared-memory destination
// and nothing to wait for. src and bytes are multiples of 16.
__device__ __forceinline__ void l2_prefetch_bulk(void const* src, std::uint32_t bytes)
{
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;"
                 ::"l"(reinterpret_cast<std::uint64_t>(src)), "r"(bytes)
                 : "memory");
}

// One CTA's share of an L2 prefetch of a byte range that a later kernel of
// the step reads (weights of a projection that is still a few kernels away).
// The range is cut into `parts` contiguous 16-byte-aligned shares; issue()
// requests the next piece of this share.
struct L2PrefetchShare {
    std::uint8_t const* cur;
    std::uint8_t const* end;

    __device__ __forceinline__ void init(void const* base, std::uint64_t bytes, std::uint32_t part,
        std::uint32_t parts)
    {
        std::uint64_t const units = bytes / 16u;
        std::uint8_t const* b = static_cast<std::uint8_t const*>(base);
        cur = b + units * part / parts * 16u;
        end = b + units * (part + 1u) / parts * 16u;
        if (base == nullptr) {
            cur = end = nullptr;
        }
    }
    __device__ __forceinline__ bool issue(std::uint32_t max_bytes)
    {
        if (cur >= end) {
            return false;
        }
        std::uint64_t const left = static_cast<std::uint64_t>(end - cur);
        std::uint32_t const n = left < max_bytes ? static_cast<std::uint32_t>(left) : max_bytes;
        l2_prefetch_bulk(cur, n);
        cur += n;
        return true;
    }
};

__device__ __forceinline__ void prefetch_tensormap(CUtensorMap const* map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<std::uint64_t>(map))
                 : "memory");
}

// ---- tcgen05 ----------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(std::uint32_t* dst_smem, std::uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(cols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(std::uint32_t taddr, std::uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16, one CTA.
__device__ __forceinline__ void tc_mma_f16(std::uint32_t tmem_d, std::uint64_t a_desc,
    std::uint64_t b_desc, std::uint32_t idesc, std::uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on a CTA-local mbarrier once all previously issued MMAs completed.
__device__ __forceinline__ void tc_commit(std::uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar))
                 : "memory");
}

// Warp-collective: 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(std::uint32_t taddr, float (&v)[16])
{
    std::uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32"
        " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v[i] = __uint_as_float(r[i]);
    }
}

// K-major operand tile in shared memory, 128-byte rows with the 128B swizzle
// written by TMA (8-row / 1024-byte swizzle atoms stacked along M or N).
__device__ __forceinline__ std::uint64_t umma_desc_k_sw128(void const* smem_tile)
{
    std::uint64_t const start = (smem_u32(smem_tile) & 0x3FFFFu) >> 4;
    std::uint64_t desc = 0;
    desc |= start;                        // bits 0-13  start address >> 4
    desc |= std::uint64_t(1) << 16;       // bits 16-29 leading byte offset (unused, 1)
    desc |= std::uint64_t(1024 >> 4) << 32;  // bits 32-45 stride between 8-row atoms
    desc |= std::uint64_t(1) << 46;       // bits 46-47 descriptor version (sm_100)
    desc |= std::uint64_t(2) << 61;       // bits 61-63 swizzle mode: 128B
    return desc;
}

// Instruction descriptor: FP16 A/B, FP32 accumulate, both K-major, M x N.
__host__ __device__ constexpr std::uint32_t umma_idesc_f16_f32(int m, int n)
{
    return (1u << 4)                                   // D format F32
        | (0u << 7) | (0u << 10)                       // A, B format F16
        | (0u << 15) | (0u << 16)                      // A, B K-major
        | (static_cast<std::uint32_t>(n >> 3) << 17)   // N / 8
        | (static_cast<std::uint32_t>(m >> 4) << 24);  // M / 16
}

// ---- clusters ---------------------------------------------------------------

__device__ __forceinline__ std::uint32_t cluster_rank()
{
    std::uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ std::uint32_t cluster_map(void const* p, std::uint32_t rank)
{
    std::uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

__device__ __forceinline__ float ld_cluster_f32(std::uint32_t addr)
{
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// ---- streaming global loads ---------------------------------------------------

__device__ __forceinline__ uint4 ld_stream_v4(void const* p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

} // namespace kk
