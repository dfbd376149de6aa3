// K4/K5 — weight-streaming tensor-core GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
// Y[n][m] = sum_k W[m][k] X[n][k]: W is a decoder weight ([out][in] FP16,
// streamed from HBM exactly once per step), X holds the batch's activations
// (N <= 64 rows). This replaces the reference's cublasGemmEx projections
// (src/cuda/model/runner_support.cpp:196-274) and the elementwise kernels that
// follow them (RoPE, KV write, SwiGLU, residual add, argmax; src/cuda/model/
// kernels.cu, src/cuda/attention/paged_decode_kernels.cu:65-99).
//
// Weights come in one of two layouts:
//  * row-major [M][K]: 128x64 W tiles are fetched with 2-D TMA tensor loads
//    (128 rows of 128 bytes, K*2 bytes apart);
//  * packed (kk_gemm_pack_weight): every 128x64 tile is one contiguous 16 KB
//    block, already in the 128-byte-swizzled K-major arrangement the MMA
//    reads, and the K blocks of a row tile follow each other. A tile is then
//    one 16 KB untiled bulk copy and a CTA's K range one sequential stream,
//    which keeps DRAM pages open instead of touching 128 rows per tile.
//
// Structure of one CTA (128 threads; more with a fused RMSNorm, below):
//  * warp 0 / lane 0 issues the W tile loads and TMA loads of BNx64 X tiles
//    (128-byte swizzle) into an NS-stage mbarrier ring; W tiles for the first
//    stages are requested before griddepcontrol.wait, and every CTA triggers
//    its dependents as soon as it starts, so under programmatic dependent
//    launch the next kernel's weight stream starts while this one finishes;
//  * warp 1 / lane 0 issues tcgen05.mma (M=128, N=BN, K=16, FP16 in, FP32
//    accumulate in TMEM) and releases stages with tcgen05.commit;
//  * all 4 warps drain TMEM with tcgen05.ld.
// The K dimension is split across the CTAs of a thread-block cluster (up to 8);
// each CTA owns a disjoint subset of the batch columns. After a cluster
// barrier every CTA pushes each owner's columns of its FP32 partial tile into
// the owner's receive buffer with one bulk shared::cluster copy per owner
// (completion counted on the owner's mbarrier), so the reduction reads only
// local shared memory, in rank order (deterministic), and then runs the fused
// epilogue for those columns. Epilogue inputs (residual rows, RoPE positions,
// KV slots) are requested right after the dependency wait, while the tile
// streams.
// No TMA multicast is used anywhere.
#include "../../../include/kk_kernels.h"
#include "kernels_internal.h"
#include "launch.cuh"

#include <cfloat>
#include <mutex>

namespace kk {

__device__ unsigned int g_gemm_status;
#ifdef KK_TRACE
__device__ TraceRec g_gemm_trace[kTraceCap];
__device__ unsigned int g_gemm_trace_n;
#define KK_GEMM_STAMP(i) \
    if (tid == 0) {     \
        tr[i] = global_ns(); \
    }
#else
#define KK_GEMM_STAMP(i)
#endif

namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;                  // FP16 elements in one 128-byte swizzle row
constexpr int kThreads = 128;
// With a fused RMSNorm, KK_XNORM_WARPS warps starting at warp 2 normalise the
// activation tiles (8 by default: warps 2-9, two per SM sub-partition, so the
// CTA has 320 threads), and only warps 0-3 run the epilogue (one TMEM lane
// quarter and 32 rows each). Measured on the decode step: 8 normalising warps
// beat 4 (c4 -0.8 %, c5 -3.2 %), 4 beat 2 (-2.5 %); 16 (576 threads) made
// the step 30 % slower.
#ifndef KK_XNORM_WARPS
#define KK_XNORM_WARPS 8
#endif
static_assert(KK_XNORM_WARPS == 2 || KK_XNORM_WARPS == 4 || KK_XNORM_WARPS == 8,
    "the normalising warps cover 8, 16 or 32 tile rows per pass");
#ifndef KK_XNORM_WARPS_QKV
#define KK_XNORM_WARPS_QKV KK_XNORM_WARPS
#endif
static_assert(KK_XNORM_WARPS_QKV == 2 || KK_XNORM_WARPS_QKV == 4 || KK_XNORM_WARPS_QKV == 8,
    "the normalising warps cover 8, 16 or 32 tile rows per pass");
// Normalising threads of a projection with epilogue `epi` (the QKV one may
// use fewer, KK_XNORM_WARPS_QKV).
constexpr std::uint32_t xnThreadsFor(int epi)
{
    return (epi == KK_EPI_QKV_ROPE ? KK_XNORM_WARPS_QKV : KK_XNORM_WARPS) * 32u;
}
constexpr int kThreadsXnorm = 64 + (KK_XNORM_WARPS > KK_XNORM_WARPS_QKV ? KK_XNORM_WARPS : KK_XNORM_WARPS_QKV) * 32;
constexpr std::uint32_t kTileWBytes = kBM * kBK * 2;
constexpr std::uint32_t kSqStride = 64;  // columns per row of a sums-of-squares array
// Four W+X stages: with the split-K receive buffer about 99 KB at N <= 32,
// so an attention CTA or a second projection CTA fits beside this one on an
// SM and can start (and prefetch its weights under programmatic dependent
// launch) while this kernel drains. Measured on the decode step, 4 beats 3
// and 5. At BN = 64 (64-lane decode, prefill chunks) three stages keep a CTA
// at ~107 KB, two per SM; four (~131 KB, one per SM; build variant
// KK_GEMM_STAGES_N64=4) made the 64-lane decode step 39 % slower and c3 5 %
// slower. The epilogue's partial and
// reduced tiles reuse the ring (at most 66 KB, BN = 64).
template <int BN>
constexpr int stagesFor()
{
#ifdef KK_GEMM_STAGES
    return KK_GEMM_STAGES;
#elif defined(KK_GEMM_STAGES_N64)
    return BN >= 64 ? KK_GEMM_STAGES_N64 : 4;
#else
    return BN >= 64 ? 3 : 4;
#endif
}

// The QKV epilogue's host inputs for the CTA's (at most 8) columns, staged
// in shared memory at kernel start.
struct QkvStage {
    std::uint32_t pos[8];
    kk_kv_slot slot[8];
    float2 cs[8][32];
};

struct EpiArgs {
    std::uint32_t kind;
    void* out;
    std::uint32_t out_stride;
    // KK_EPI_QKV_ROPE
    std::uint32_t const* positions;
    kk_kv_slot const* slots;
    __half* micro;
    __half* extent;
    std::uint64_t micro_page;
    std::uint64_t extent_page;
    std::uint32_t micro_slots;
    std::uint32_t extent_slots;
    std::uint32_t micro_cap;     // tokens per micro page
    std::uint32_t kv_row;        // kv_heads * head_dim
    std::uint32_t layer;
    std::uint32_t q_rows;
    std::uint32_t kv_rows;
    float theta;
    float2 const* rope_cs;       // [positions][32] (cos, sin), or null: computed here
    std::uint32_t rope_positions;
    // KK_EPI_ARGMAX
    std::uint32_t* tokens;
    float* part_val;
    std::uint32_t* part_idx;
    std::uint32_t* counter;
    std::uint32_t num_m_tiles;
};

struct GemmArgs {
    std::uint8_t const* w_packed;   // packed weight tiles, or null for row-major + TMA
    std::uint32_t M;
    std::uint32_t K;
    std::uint32_t N;
    std::uint32_t split;
    std::uint32_t kb_total;
    __half const* norm_x;           // RMS-normalise the X rows by the rows of norm_x (or null)
    std::uint32_t norm_stride;
    float norm_eps;
    __half const* norm_w;           // RMSNorm weight [K] applied with the factor (null: 1)
    // L2 prefetch of bytes that a later kernel of the step reads (or null):
    // every CTA requests its share after the dependency wait, while this
    // kernel's own weights are already on chip.
    void const* l2_pf;
    std::uint64_t l2_pf_bytes;
    // Runner path of the fused RMSNorm: column n's factor comes from per-row-
    // tile sums of squares, rsqrt(sum_t sq_in[t * kSqStride + n] / K + eps),
    // written by the kernel that produced the rows (null: reduce norm_x rows).
    float const* sq_in;
    std::uint32_t sq_tiles;
    // KK_EPI_RESIDUAL: sums of squares of the new FP16 rows over this tile,
    // sq_out[m_tile * kSqStride + n] (or null).
    float* sq_out;
    unsigned int* status;           // error word of the launch (null: the module's word)
    EpiArgs epi;
};

// Generic-proxy writes to shared memory, made visible to bulk copies that
// read it afterwards (async proxy).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk copy of `bytes` from this CTA's shared memory into another CTA of the
// cluster (dst and bar are shared::cluster addresses from mapa); completion
// is counted on the destination CTA's mbarrier.
__device__ __forceinline__ void bulk_copy_to_peer(std::uint32_t dst, void const* src, std::uint32_t bytes,
    std::uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "r"(smem_u32(src)), "r"(bytes), "r"(bar)
        : "memory");
}

// Barrier of `count` threads (multiple of 32) on hardware barrier `id` (id 0
// is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(std::uint32_t id, std::uint32_t count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Named barrier that also ANDs a predicate over the participating threads,
// so that all of them take the same branch afterwards.
__device__ __forceinline__ bool named_barrier_and(std::uint32_t id, std::uint32_t count, bool pred)
{
    std::uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<std::uint32_t>(pred)), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void cluster_arrive()
{
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

// Arrive without release semantics: for a barrier phase that orders nothing
// in memory (the data it guards was handed over through mbarriers).
__device__ __forceinline__ void cluster_arrive_relaxed()
{
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait()
{
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// RoPE cos / sin of a position and pair index when the caller gives no
// factor table: kept out of line so that the QKV epilogue's own code (run
// once per launch, its instruction fetches on the critical path) stays small.
__device__ __noinline__ float2 ropeFactors(float theta, std::uint32_t position, std::uint32_t pair)
{
    float const inv_freq = powf(theta, -2.0f * static_cast<float>(pair) / 64.0f);
    float2 cs;
    sincosf(static_cast<float>(position) * inv_freq, &cs.y, &cs.x);
    return cs;
}

__device__ __forceinline__ bool better(float v, std::uint32_t i, float bv, std::uint32_t bi)
{
    return v > bv || (v == bv && i < bi);
}

template <int BN>
constexpr std::uint32_t tmemCols()
{
    return BN <= 32 ? 32u : (BN <= 64 ? 64u : (BN <= 128 ? 128u : 256u));
}

// Receive buffer of the split-K reduction, outside the ring so that peers
// can push into it while this CTA's MMAs still read the ring: one slot of
// ceil(N/S) FP32 columns per source rank, S * ceil(N/S) <= recvCols columns
// in all (the planner lowers S until that holds). BN + 1 at BN <= 32, so
// that a CTA (98.5 KB at BN = 32) and an attention CTA share an SM, which
// admits S = 3 at N = 32; BN + 2 above, which admits S = 3 at N = 64 (the
// gate/up projection's 88 row tiles then run 264 CTAs instead of 176) and
// keeps two 107 KB CTAs per SM.
constexpr std::uint32_t recvCols(std::uint32_t bn)
{
    return bn <= 32u ? bn + 1u : bn + 2u;
}

template <int BN>
constexpr std::size_t recvBytes()
{
    return std::size_t(recvCols(BN)) * kBM * 4;
}

template <int BN>
constexpr std::size_t smemBytes()
{
    return 1024 /* alignment slack */ + stagesFor<BN>() * (kTileWBytes + BN * 128) + recvBytes<BN>()
        + 1024 /* barriers + scratch */;
}

// One instance per (N tile, epilogue kind): each instance carries only its
// own epilogue, which keeps the code that runs after the main loop small
// (instruction fetches after the main loop are on the critical path).
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreadsXnorm, 1) gemm_tc_kernel(
    const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
    GemmArgs args)
{
    constexpr int kStages = stagesFor<BN>();
    constexpr std::uint32_t kXnThreads = xnThreadsFor(EPI);  // normalising threads (fused RMSNorm)
    extern __shared__ std::uint8_t smem_raw[];
    std::uint32_t const pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    std::uint8_t* smem = smem_raw + pad;
    std::uint8_t* w_stage = smem;
    std::uint8_t* x_stage = smem + kStages * kTileWBytes;
    float* recv = reinterpret_cast<float*>(x_stage + kStages * BN * 128);
    std::uint64_t* full = reinterpret_cast<std::uint64_t*>(reinterpret_cast<std::uint8_t*>(recv) + recvBytes<BN>());
    std::uint64_t* empty = full + kStages;
    std::uint64_t* accum = empty + kStages;
    std::uint64_t* rbar = accum + 1;  // this CTA's receive buffer is complete
    std::uint32_t* tmem_slot = reinterpret_cast<std::uint32_t*>(rbar + 1);
    int* flag = reinterpret_cast<int*>(tmem_slot + 4);
    float* rnorm = reinterpret_cast<float*>(flag + 4);  // [BN] per-column RMS factors
    // With a fused RMSNorm the X tile of stage s lands on xfull[s] and full[s]
    // completes only once the normalising warps rewrote it in place.
    std::uint64_t* xfull = reinterpret_cast<std::uint64_t*>(rnorm + BN);

    std::uint32_t const tid = threadIdx.x;
    std::uint32_t const warp = tid / 32;
    std::uint32_t const lane = tid % 32;
    unsigned int* const st = args.status != nullptr ? args.status : &g_gemm_status;
#ifdef KK_TRACE
    std::uint64_t tr[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
    // Stamps of other threads (0: not reached): 9 the first stages normalised
    // and released, 10 the RMS factors ready, 11 the first X tile seen landed,
    // 12 the first stages' transforms done, 13 the first MMA issued, 14 the
    // first stage's transform done, 15 the last prefetched X tile seen landed.
    __shared__ std::uint64_t s_xstamp[7];
    if (tid < 7) {
        s_xstamp[tid] = 0;
    }
#endif
    KK_GEMM_STAMP(0)
    std::uint32_t const S = args.split;
    std::uint32_t const rank = S > 1 ? cluster_rank() : 0;
    std::uint32_t const m_tile = blockIdx.y;
    std::uint32_t const kb_begin = rank * args.kb_total / S;
    std::uint32_t const nk = (rank + 1) * args.kb_total / S - kb_begin;
    constexpr std::uint32_t kStageBytes = kTileWBytes + BN * 128;
    // Fused RMSNorm: X tiles are normalised in shared memory before the MMA
    // reads them, X'[n][k] = half(x[n][k] * r[n] * g[k]), the rounding point
    // of the reference's rmsNormBatchKernel (its output is FP16).
    bool const xnorm = args.norm_x != nullptr;
    std::uint32_t const w_expect = xnorm ? kTileWBytes : kStageBytes;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], xnorm ? 2 : 1);  // producer (+ the normalising warps)
            mbar_init(&empty[s], 1);
            mbar_init(&xfull[s], 1);
        }
        mbar_init(accum, 1);
        mbar_init(rbar, 1);
        if (S > 1) {
            // Armed now: peers may push as soon as their own partial is ready.
            mbar_arrive_expect_tx(rbar, ((rank + 1) * args.N / S - rank * args.N / S) * S * kBM * 4u);
        }
        fence_barrier_init();
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_x);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, tmemCols<BN>());
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (S > 1) {
        // Cluster barrier phase 1, arrive: this CTA's barriers are initialised
        // and armed. The matching wait comes just before the first push.
        cluster_arrive();
    }
    std::uint32_t const tmem = *tmem_slot;
    // Dependents may launch now: they only prefetch weights before their own
    // griddepcontrol.wait, which returns once this grid has completed.
    pdl_launch_dependents();

    // QKV epilogue inputs that come from the host (positions, KV slots, RoPE
    // factors of the CTA's columns): staged in shared memory now, before the
    // dependency wait, so the epilogue reads them there (they are not held
    // in registers across the main loop).
    constexpr std::uint32_t kPre = 8;
    std::uint32_t const pn0 = rank * args.N / S;
    std::uint32_t const pcols = (rank + 1) * args.N / S - pn0;
    bool const prefetched = pcols <= kPre;
    [[maybe_unused]] QkvStage* qs = nullptr;
    if constexpr (EPI == KK_EPI_QKV_ROPE) {
        __shared__ QkvStage s_qkv;
        qs = &s_qkv;
        for (std::uint32_t idx = tid; prefetched && idx < pcols * 32u && tid < kBM; idx += kBM) {
            std::uint32_t const j = idx / 32u;
            std::uint32_t const d = idx % 32u;
            std::uint32_t const p = args.epi.positions[pn0 + j];
            if (d == 0) {
                s_qkv.pos[j] = p;
                s_qkv.slot[j] = args.epi.slots[pn0 + j];
            }
            s_qkv.cs[j][d] = args.epi.rope_cs != nullptr && p < args.epi.rope_positions
                ? args.epi.rope_cs[std::uint64_t(p) * 32u + d] : make_float2(1.f, 0.f);
        }
    }

    if (warp == 0 && lane == 0) {
        // Producer. Weights never depend on the previous kernel: request them
        // before waiting for it; activations only after.
        std::uint32_t const pre = nk < kStages ? nk : kStages;
        std::uint64_t const policy = l2_policy_evict_first();
        std::uint8_t const* wp = args.w_packed == nullptr ? nullptr
            : args.w_packed + (std::uint64_t(m_tile) * args.kb_total + kb_begin) * kTileWBytes;
        auto load_w = [&](std::uint32_t s, std::uint32_t i) {
            if (wp != nullptr) {
                bulk_load_hint(w_stage + s * kTileWBytes, wp + std::uint64_t(i) * kTileWBytes,
                    kTileWBytes, &full[s], policy);
            } else {
                tma_load_2d_hint(w_stage + s * kTileWBytes, &tm_w, &full[s],
                    static_cast<int>((kb_begin + i) * kBK), static_cast<int>(m_tile * kBM), policy);
            }
        };
        // X tile i of the CTA: into full[] directly, or into xfull[] for the
        // normalising warps.
        auto load_x = [&](std::uint32_t s, std::uint32_t i) {
            std::uint64_t* bar = &full[s];
            if (xnorm) {
                bar = &xfull[s];
                mbar_arrive_expect_tx(bar, BN * 128u);
            }
            tma_load_2d(x_stage + s * BN * 128, &tm_x, bar, static_cast<int>((kb_begin + i) * kBK), 0);
        };
        for (std::uint32_t i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], w_expect);
            load_w(i, i);
        }
        pdl_wait();
        KK_GEMM_STAMP(1)
        for (std::uint32_t i = 0; i < pre; ++i) {
            load_x(i, i);
        }
        if (args.l2_pf != nullptr) {
            L2PrefetchShare pf;
            pf.init(args.l2_pf, args.l2_pf_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
            while (pf.issue(32768u)) {
            }
        }
        for (std::uint32_t i = pre; i < nk; ++i) {
            std::uint32_t const s = i % kStages;
            if (!mbar_wait(&empty[s], ((i / kStages) - 1) & 1u, st)) {
                break;
            }
            mbar_arrive_expect_tx(&full[s], w_expect);
            load_w(s, i);
            load_x(s, i);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer.
        std::uint32_t const idesc = umma_idesc_f16_f32(kBM, BN);
        for (std::uint32_t i = 0; i < nk; ++i) {
            std::uint32_t const s = i % kStages;
            if (!mbar_wait(&full[s], (i / kStages) & 1u, st)) {
                break;
            }
            tc_fence_after();
#ifdef KK_TRACE
            if (i == 0) {
                s_xstamp[4] = global_ns();
            }
#endif
            std::uint64_t const a = umma_desc_k_sw128(w_stage + s * kTileWBytes);
            std::uint64_t const b = umma_desc_k_sw128(x_stage + s * BN * 128);
#pragma unroll
            for (std::uint32_t k = 0; k < kBK / 16; ++k) {
                // +32 bytes along K inside the 128-byte swizzle row: +2 in addr>>4 units.
                tc_mma_f16(tmem, a + 2 * k, b + 2 * k, idesc, (i | k) != 0 ? 1u : 0u);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(accum);
    }
    // Lanes 1-31 of the producer and MMA warps park here (not in a polling
    // loop) until their lane 0 has finished its role.
    __syncwarp();
    pdl_wait();
    // Epilogue inputs of this CTA's columns, requested now so that they are
    // in registers when the reduced tile is ready: the residual rows (written
    // by the previous kernel, hence after the wait); the QKV epilogue's
    // positions, KV slots and RoPE factors were requested at kernel start.
    std::uint32_t const pm = m_tile * kBM + tid;
    __half resid[kPre];
#pragma unroll
    for (std::uint32_t j = 0; j < kPre; ++j) {
        resid[j] = __float2half_rn(0.f);
        if (EPI == KK_EPI_RESIDUAL && prefetched && j < pcols && tid < kBM && pm < args.M) {
            resid[j] = static_cast<__half const*>(args.epi.out)[std::uint64_t(pn0 + j) * args.epi.out_stride + pm];
        }
    }
    if (xnorm && warp >= 2 && warp < 2u + kXnThreads / 32u) {
        // The normalising warps: the RMS factor of every batch row, then each X tile
        // normalised in place as it lands.
        std::uint32_t const t = tid - 64u;
        std::uint32_t const c = t & 7u;
        // This thread's 8 norm weights of stage i (FP16 ones without a
        // weight), issued in program order: those of the first stages go out
        // together with the sums of squares below.
        auto norm_chunk = [&](std::uint32_t i) {
            std::uint32_t const k0 = (kb_begin + i) * kBK + c * 8u;
            uint4 g = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);  // FP16 1.0 x 8
            if (args.norm_w != nullptr && i < nk && k0 < args.K) {
                g = ldg_u4_now(args.norm_w + k0);
            }
            return g;
        };
        std::uint32_t const first = nk < static_cast<std::uint32_t>(kStages) ? nk : kStages;
        uint4 gfirst[kStages];
#pragma unroll
        for (int j = 0; j < kStages; ++j) {
            gfirst[j] = norm_chunk(j);
        }
        uint4 g_next = norm_chunk(first);
        if (args.sq_in != nullptr) {
            // From the producing kernel's per-tile sums of squares, one thread
            // per row, every partial requested at once and summed in tile order.
            for (std::uint32_t n = t; n < static_cast<std::uint32_t>(BN); n += kXnThreads) {
                float sum = 0.f;
                for (std::uint32_t t0 = 0; n < args.N && t0 < args.sq_tiles; t0 += 16u) {
                    float v[16];
#pragma unroll
                    for (std::uint32_t q = 0; q < 16u; ++q) {
                        v[q] = t0 + q < args.sq_tiles ? args.sq_in[(t0 + q) * kSqStride + n] : 0.f;
                    }
#pragma unroll
                    for (std::uint32_t q = 0; q < 16u; ++q) {
                        sum += v[q];
                    }
                }
                rnorm[n] = n < args.N ? 1.0f / sqrtf(sum / static_cast<float>(args.K) + args.norm_eps) : 0.f;
            }
        } else {
            // From the rows themselves, one warp per row.
            for (std::uint32_t n = warp - 2u; n < static_cast<std::uint32_t>(BN); n += kXnThreads / 32u) {
                float sum = 0.f;
                __half const* xr = args.norm_x + std::uint64_t(n) * args.norm_stride;
                for (std::uint32_t k = lane * 8u; n < args.N && k < args.K; k += 256u) {
                    uint4 const raw = *reinterpret_cast<uint4 const*>(xr + k);
                    __half const* h = reinterpret_cast<__half const*>(&raw);
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        float const f = __half2float(h[e]);
                        sum += f * f;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    sum += __shfl_xor_sync(0xffffffffu, sum, o);
                }
                if (lane == 0) {
                    rnorm[n] = n < args.N ? 1.0f / sqrtf(sum / static_cast<float>(args.K) + args.norm_eps) : 0.f;
                }
            }
        }
        named_barrier_sync(1, kXnThreads);
#ifdef KK_TRACE
        if (t == 0) {
            s_xstamp[1] = global_ns();
        }
#endif
        // Thread t owns 16-byte chunk t % 8 (dims 8c .. 8c+7 of the tile's 64)
        // of rows t / 8, t / 8 + kXnThreads / 8, ...; the tile is [BN rows][128 bytes] with
        // the 128-byte swizzle, chunk c of row n at n*128 + ((c ^ n%8) * 16).
        // One stage in place: x' = half((x * r) * g) per element, FP32
        // products rounded once (packed conversions, two elements each).
        auto transform = [&](std::uint32_t s, uint4 graw) {
            float2 gv[4];
            __half2 const* gh = reinterpret_cast<__half2 const*>(&graw);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                gv[e] = __half22float2(gh[e]);
            }
            std::uint8_t* xs = x_stage + s * BN * 128;
            // The thread's rows (t / 8, t / 8 + kRowStep, ...): every load
            // first, then the math and the stores, so the loads overlap. With
            // more threads than the tile has row chunks (BN < kRowStep) the
            // threads past the last row have none.
            constexpr std::uint32_t kRowStep = kXnThreads / 8u;
            constexpr std::uint32_t kRows = (static_cast<std::uint32_t>(BN) + kRowStep - 1u) / kRowStep;
            if (static_cast<std::uint32_t>(BN) < kRowStep && (t >> 3) >= static_cast<std::uint32_t>(BN)) {
                return;
            }
            uint4 raw[kRows];
            float rr[kRows];
#pragma unroll
            for (std::uint32_t q = 0; q < kRows; ++q) {
                std::uint32_t const n = (t >> 3) + kRowStep * q;
                raw[q] = *reinterpret_cast<uint4 const*>(xs + n * 128u + ((c ^ (n & 7u)) << 4));
                rr[q] = rnorm[n];
            }
#pragma unroll
            for (std::uint32_t q = 0; q < kRows; ++q) {
                std::uint32_t const n = (t >> 3) + kRowStep * q;
                __half2* h = reinterpret_cast<__half2*>(&raw[q]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    float2 const f = __half22float2(h[e]);
                    h[e] = __floats2half2_rn(f.x * rr[q] * gv[e].x, f.y * rr[q] * gv[e].y);
                }
                *reinterpret_cast<uint4*>(xs + n * 128u + ((c ^ (n & 7u)) << 4)) = raw[q];
            }
        };
        // The stages requested right after the dependency wait land together:
        // they are normalised as one batch behind one proxy fence and one
        // barrier, so the MMA of the prefetched weights starts after one
        // hand-over instead of one per stage. Later stages go one by one
        // (their weights stream from HBM meanwhile). Later norm weights are
        // requested one stage ahead.
        bool got = true;
#pragma unroll
        for (int j = 0; j < kStages; ++j) {
            if (got && static_cast<std::uint32_t>(j) < first) {
                got = mbar_wait_spin(&xfull[j], 0u, st);
#ifdef KK_TRACE
                if (j == 0 && t == 0) {
                    s_xstamp[2] = global_ns();
                }
                if (static_cast<std::uint32_t>(j) + 1u == first && t == 0) {
                    s_xstamp[6] = global_ns();
                }
#endif
                if (got) {
                    transform(j, gfirst[j]);
                }
#ifdef KK_TRACE
                if (j == 0 && t == 0) {
                    s_xstamp[5] = global_ns();
                }
#endif
            }
        }
#ifdef KK_TRACE
        if (t == 0) {
            s_xstamp[3] = global_ns();
        }
#endif
        // Generic-proxy writes, read next by the tensor cores (async proxy).
        // A wait that gave up stops every normalising thread at the same
        // point (the MMA warp's own bounded wait then ends the tile).
        fence_proxy_async_smem();
        bool ok = named_barrier_and(1, kXnThreads, got);
        if (t == 0 && ok) {
            for (std::uint32_t j = 0; j < first; ++j) {
                mbar_arrive(&full[j]);
            }
#ifdef KK_TRACE
            s_xstamp[0] = global_ns();
#endif
        }
        for (std::uint32_t i = first; ok && i < nk; ++i) {
            std::uint32_t const s = i % kStages;
            uint4 const graw = g_next;
            g_next = norm_chunk(i + 1);
            got = mbar_wait_spin(&xfull[s], (i / kStages) & 1u, st);
            if (got) {
                transform(s, graw);
            }
            fence_proxy_async_smem();
            ok = named_barrier_and(1, kXnThreads, got);
            if (t == 0 && ok) {
                mbar_arrive(&full[s]);
            }
        }
    }
    // The epilogue: warps 0-3, one TMEM lane quarter and 32 rows each (their
    // barriers count 128 threads). Warps 4 and up of a fused-RMSNorm CTA only
    // take part in the cluster barrier's phases.
    if (tid < kBM) {
        bool const have_acc = mbar_wait(accum, 0, st);
        tc_fence_after();
        KK_GEMM_STAMP(2)

        // TMEM -> this CTA's FP32 partial tile, column-major [BN][128] (aliases the
        // W stages: every MMA that read them has completed).
        float* part = reinterpret_cast<float*>(smem);
        std::uint32_t const row = tid;
#pragma unroll
        for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
            tmem_ld16(tmem + ((warp * 32u) << 16) + static_cast<std::uint32_t>(c0), v);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                part[(c0 + j) * kBM + row] = have_acc && nk != 0 ? v[j] : 0.f;
            }
        }
        std::uint32_t const n0 = rank * args.N / S;
        std::uint32_t const n1 = (rank + 1) * args.N / S;
        std::uint32_t const cols = n1 - n0;
        std::uint32_t const m = m_tile * kBM + row;
        EpiArgs const& e = args.epi;
        // The receive buffer holds one slot of up to cw columns per source rank;
        // the reduced columns and the argmax scratch follow the partial in the
        // (now idle) ring.
        std::uint32_t const cw = (args.N + S - 1) / S;
        float* red = part + BN * kBM;
        float* amax_v = red + (S > 1 ? cw : static_cast<std::uint32_t>(BN)) * kBM;  // [4][BN]
        std::uint32_t* amax_i = reinterpret_cast<std::uint32_t*>(amax_v + 4 * BN);  // [4][BN]
        if (S > 1) {
            fence_proxy_async_smem();
        }
        tc_fence_before();
        named_barrier_sync(2, kBM);
        KK_GEMM_STAMP(3)
        if (S > 1) {
            // The partial is written; every peer's receive buffer is armed (phase
            // 1 of the cluster barrier, long complete by now). Thread r pushes
            // owner r's columns.
            cluster_wait();
            KK_GEMM_STAMP(4)
            if (tid < S) {
                std::uint32_t const r0 = tid * args.N / S;
                std::uint32_t const r1 = (tid + 1) * args.N / S;
                if (r1 > r0) {
                    bulk_copy_to_peer(cluster_map(recv + rank * cw * kBM, tid), part + r0 * kBM,
                        (r1 - r0) * kBM * 4u, cluster_map(rbar, tid));
                }
            }
            bool const got = mbar_wait(rbar, 0, st);
            KK_GEMM_STAMP(5)
            // Sum over the K slices in rank order (deterministic), four
            // columns at a time so that their shared-memory loads overlap.
            for (std::uint32_t j = 0; j < cols; j += 4u) {
                float acc0 = 0.f;
                float acc1 = 0.f;
                float acc2 = 0.f;
                float acc3 = 0.f;
                for (std::uint32_t r = 0; r < S; ++r) {
                    float const* src = recv + (r * cw + j) * kBM + row;
                    acc0 += got ? src[0] : 0.f;
                    acc1 += got && j + 1u < cols ? src[kBM] : 0.f;
                    acc2 += got && j + 2u < cols ? src[2u * kBM] : 0.f;
                    acc3 += got && j + 3u < cols ? src[3u * kBM] : 0.f;
                }
                red[j * kBM + row] = acc0;
                if (j + 1u < cols) {
                    red[(j + 1u) * kBM + row] = acc1;
                }
                if (j + 2u < cols) {
                    red[(j + 2u) * kBM + row] = acc2;
                }
                if (j + 3u < cols) {
                    red[(j + 3u) * kBM + row] = acc3;
                }
            }
            // Cluster barrier phase 2, arrive: this CTA has received everything
            // (the receive mbarrier completed), so the senders' partials may go.
            // Relaxed: no memory needs ordering here, and a release arrive waits
            // for this CTA's outstanding memory operations.
            cluster_arrive_relaxed();
        } else {
            for (std::uint32_t j = 0; j < cols; ++j) {
                red[j * kBM + row] = part[(n0 + j) * kBM + row];
            }
        }
        named_barrier_sync(2, kBM);
        KK_GEMM_STAMP(6)

        switch (EPI) {
        case KK_EPI_STORE_F16:
            if (m < args.M) {
                for (std::uint32_t j = 0; j < cols; ++j) {
                    static_cast<__half*>(e.out)[std::uint64_t(n0 + j) * e.out_stride + m] =
                        __float2half_rn(red[j * kBM + row]);
                }
            }
            break;
        case KK_EPI_STORE_F32:
            if (m < args.M) {
                for (std::uint32_t j = 0; j < cols; ++j) {
                    static_cast<float*>(e.out)[std::uint64_t(n0 + j) * e.out_stride + m] = red[j * kBM + row];
                }
            }
            break;
        case KK_EPI_RESIDUAL: {
            // New rows h = half(resid + half(acc)); with sq_out, also the tile's
            // sum of h^2 per column (the next RMSNorm's statistics), reduced in a
            // fixed order: lanes by shuffles, then the four warps in turn.
            float* wsq = amax_v;  // [4][BN], idle in this epilogue
            bool const want_sq = args.sq_out != nullptr;
            if (prefetched) {
#pragma unroll
                for (std::uint32_t j = 0; j < kPre; ++j) {
                    if (j < cols) {
                        __half const h = __hadd(resid[j], __float2half_rn(red[j * kBM + row]));
                        if (m < args.M) {
                            static_cast<__half*>(e.out)[std::uint64_t(n0 + j) * e.out_stride + m] = h;
                        }
                        if (want_sq) {
                            float const f = m < args.M ? __half2float(h) : 0.f;
                            float q = f * f;
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                q += __shfl_xor_sync(0xffffffffu, q, o);
                            }
                            if (lane == 0) {
                                wsq[warp * BN + j] = q;
                            }
                        }
                    }
                }
            } else {
                for (std::uint32_t j = 0; j < cols; ++j) {
                    float f = 0.f;
                    if (m < args.M) {
                        __half* hp = static_cast<__half*>(e.out) + std::uint64_t(n0 + j) * e.out_stride + m;
                        __half const h = __hadd(*hp, __float2half_rn(red[j * kBM + row]));
                        *hp = h;
                        f = __half2float(h);
                    }
                    if (want_sq) {
                        float q = f * f;
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            q += __shfl_xor_sync(0xffffffffu, q, o);
                        }
                        if (lane == 0) {
                            wsq[warp * BN + j] = q;
                        }
                    }
                }
            }
            if (want_sq) {
                named_barrier_sync(2, kBM);
                if (tid < cols) {
                    args.sq_out[m_tile * kSqStride + n0 + tid] =
                        ((wsq[tid] + wsq[BN + tid]) + wsq[2 * BN + tid]) + wsq[3 * BN + tid];
                }
            }
            break;
        }
        case KK_EPI_SILU_PAIRS: {
            // Rows 2i / 2i+1 hold gate_i / up_i; the pair's two threads take
            // alternate columns (thread 2i the even ones, 2i+1 the odd ones).
            std::uint32_t const pr = row & ~1u;
            std::uint32_t const mp = m_tile * kBM + pr;
            if (mp < args.M) {
                for (std::uint32_t j = row & 1u; j < cols; j += 2u) {
                    float const g = __half2float(__float2half_rn(red[j * kBM + pr]));
                    float const u = __half2float(__float2half_rn(red[j * kBM + pr + 1u]));
                    static_cast<__half*>(e.out)[std::uint64_t(n0 + j) * e.out_stride + mp / 2] =
                        __float2half_rn(g / (1.0f + expf(-g)) * u);
                }
            }
            break;
        }
        case KK_EPI_QKV_ROPE: {
            std::uint32_t const kv_end = e.q_rows + 2 * e.kv_rows;
            if (m >= args.M || m >= kv_end) {
                break;
            }
            // RoPE pairs dims d and d+32 of a head: rows row and row^32 of the tile.
            bool const is_v = m >= e.q_rows + e.kv_rows;
            std::uint32_t const idx = m < e.q_rows ? m : (is_v ? m - e.q_rows - e.kv_rows : m - e.q_rows);
            std::uint32_t const d = idx & 63u;
            // The rotation's first product minus (or plus) the second, each
            // rounded on its own (no fused multiply-add), as the reference's
            // host model computes it.
#pragma unroll 1
            for (std::uint32_t j = 0; j < cols; ++j) {
                std::uint32_t const n = n0 + j;
                // Staged values when the CTA owns at most kPre columns.
                std::uint32_t position = 0;
                kk_kv_slot slot_rec{0, 0, 0, 0};
                float2 cs = make_float2(1.f, 0.f);
                if (prefetched) {
                    position = qs->pos[j];
                    slot_rec = qs->slot[j];
                    cs = qs->cs[j][d & 31u];
                } else {
                    position = e.positions[n];
                    slot_rec = e.slots[n];
                    if (e.rope_cs != nullptr && position < e.rope_positions) {
                        cs = e.rope_cs[std::uint64_t(position) * 32u + (d & 31u)];
                    }
                }
                float const mine = __half2float(__float2half_rn(red[j * kBM + row]));
                float out = mine;
                if (!is_v) {
                    float const other = __half2float(__float2half_rn(red[j * kBM + (row ^ 32u)]));
                    if (e.rope_cs == nullptr) {
                        cs = ropeFactors(e.theta, position, d & 31u);
                    }
                    float const a = __fmul_rn(mine, cs.x);
                    float const b = __fmul_rn(other, cs.y);
                    out = d < 32u ? __fsub_rn(a, b) : __fadd_rn(a, b);
                }
                __half const hv = __float2half_rn(out);
                if (m < e.q_rows) {
                    static_cast<__half*>(e.out)[std::uint64_t(n) * e.out_stride + idx] = hv;
                } else {
                    kk_kv_slot const sl = slot_rec;
                    bool const micro = sl.kind == 0;
                    std::uint32_t const cap = micro ? e.micro_cap : 64u;
                    if (sl.active && sl.page_token < cap
                        && (micro ? sl.slot < e.micro_slots : sl.slot < e.extent_slots)) {
                        __half* page = micro ? e.micro + std::uint64_t(sl.slot) * e.micro_page
                                             : e.extent + std::uint64_t(sl.slot) * e.extent_page;
                        std::uint64_t const off = ((std::uint64_t(e.layer) * 2u + (is_v ? 1u : 0u)) * cap
                            + sl.page_token) * e.kv_row + idx;
                        page[off] = hv;
                    } else if (sl.active) {
                        atomicCAS(st, kErrNone, kErrBadDescriptor);
                    }
                }
            }
            break;
        }
        case KK_EPI_ARGMAX: {
            bool const valid = m < args.M;
            if (valid && e.out != nullptr) {
                for (std::uint32_t j = 0; j < cols; ++j) {
                    static_cast<float*>(e.out)[std::uint64_t(n0 + j) * e.out_stride + m] = red[j * kBM + row];
                }
            }
            // Per warp, every column's winner over its 32 rows; then per column
            // over the 4 warps. Ties keep the lowest index.
            for (std::uint32_t j = 0; j < cols; ++j) {
                float bv = valid ? red[j * kBM + row] : -INFINITY;
                std::uint32_t bi = valid ? m : 0xffffffffu;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    float const ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    std::uint32_t const oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (better(ov, oi, bv, bi)) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    amax_v[warp * BN + j] = bv;
                    amax_i[warp * BN + j] = bi;
                }
            }
            named_barrier_sync(2, kBM);
            if (tid < cols) {
                float bv = amax_v[tid];
                std::uint32_t bi = amax_i[tid];
                for (int w = 1; w < 4; ++w) {
                    if (better(amax_v[w * BN + tid], amax_i[w * BN + tid], bv, bi)) {
                        bv = amax_v[w * BN + tid];
                        bi = amax_i[w * BN + tid];
                    }
                }
                e.part_val[std::uint64_t(m_tile) * args.N + n0 + tid] = bv;
                e.part_idx[std::uint64_t(m_tile) * args.N + n0 + tid] = bi;
            }
            break;
        }
        default:
            break;
        }

        if (EPI == KK_EPI_ARGMAX) {
            // The last CTA of the launch folds the per-tile winners of every column.
            __threadfence();
            named_barrier_sync(2, kBM);
            if (tid == 0) {
                std::uint32_t const done = atomicAdd(e.counter, 1u);
                *flag = done + 1 == e.num_m_tiles * S;
            }
            named_barrier_sync(2, kBM);
            if (*flag) {
                __threadfence();
                for (std::uint32_t n = tid; n < args.N; n += kThreads) {
                    float bv = -FLT_MAX;     // same starting point as the reference reduction
                    std::uint32_t bi = 0;
                    for (std::uint32_t t = 0; t < e.num_m_tiles; ++t) {
                        float const v = __ldcg(e.part_val + std::uint64_t(t) * args.N + n);
                        std::uint32_t const i = __ldcg(e.part_idx + std::uint64_t(t) * args.N + n);
                        if (better(v, i, bv, bi)) {
                            bv = v;
                            bi = i;
                        }
                    }
                    e.tokens[n] = bi;
                }
                if (tid == 0) {
                    *e.counter = 0;
                }
            }
        }

        KK_GEMM_STAMP(7)
        if (S > 1) {
            cluster_wait();  // this CTA's partial stays alive until every owner has received it
        }
    } else if (S > 1) {
        cluster_wait();
        cluster_arrive_relaxed();
        cluster_wait();
    }
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, tmemCols<BN>());
    }
#ifdef KK_TRACE
    if (tid == 0) {
        tr[8] = global_ns();
        for (int i = 0; i < 7; ++i) {
            tr[9 + i] = s_xstamp[i];
        }
        std::uint32_t const slot = atomicAdd(&g_gemm_trace_n, 1u);
        if (slot < kTraceCap) {
            TraceRec& r = g_gemm_trace[slot];
            r.tag = (static_cast<std::uint32_t>(EPI) << 16) | args.epi.layer;
            r.block = (blockIdx.y << 16) | blockIdx.x;
            r.smid = sm_id();
            r.aux = args.K;
            for (int i = 0; i < 16; ++i) {
                r.t[i] = tr[i];
            }
        }
    }
#endif
}

// Packs W [M][K] (row-major, K % 8 == 0) into 128x64 tiles, tile (t, b) at
// ((t * kb_total + b) * 16 KB): row r, 16-byte chunk c of the tile lands at
// r * 128 + ((c ^ (r % 8)) * 16), the 128-byte swizzle the MMA descriptors
// expect; rows >= M and columns >= K are zero. One thread per 16-byte chunk.
__global__ void pack_weight_kernel(std::uint16_t const* __restrict__ w, std::uint32_t M,
    std::uint32_t K, std::uint32_t kb_total, std::uint64_t chunks, uint4* __restrict__ out,
    __half const* __restrict__ col_scale)
{
    std::uint64_t const i = std::uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= chunks) {
        return;
    }
    std::uint64_t const block = i / 1024u;      // (tile, kb) block
    std::uint32_t const within = static_cast<std::uint32_t>(i % 1024u);
    std::uint32_t const r = within / 8u;
    std::uint32_t const c = within % 8u;
    std::uint64_t const t = block / kb_total;
    std::uint32_t const b = static_cast<std::uint32_t>(block % kb_total);
    std::uint64_t const row = t * kBM + r;
    std::uint32_t const col = b * kBK + c * 8u;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < M && col < K) {
        v = *reinterpret_cast<uint4 const*>(w + row * K + col);
        if (col_scale != nullptr) {
            // W[m][k] * g[k], rounded once to FP16 (an RMSNorm weight folded in).
            uint4 const gs = *reinterpret_cast<uint4 const*>(col_scale + col);
            __half* hv = reinterpret_cast<__half*>(&v);
            __half const* hg = reinterpret_cast<__half const*>(&gs);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                hv[e] = __float2half_rn(__half2float(hv[e]) * __half2float(hg[e]));
            }
        }
    }
    out[block * 1024u + r * 8u + (c ^ (r & 7u))] = v;
}

// ---- host side ------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
    cuuint64_t const*, cuuint64_t const*, cuuint32_t const*, cuuint32_t const*,
    CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeFn()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q)
                == cudaSuccess && q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    return fn;
}

// 2D FP16 tensor [rows][cols] (row stride in elements), box 64 x box_rows, 128B swizzle.
bool makeMap(CUtensorMap* map, void const* base, std::uint64_t cols, std::uint64_t rows,
    std::uint64_t stride_elems, std::uint32_t box_rows)
{
    EncodeTiledFn const fn = encodeFn();
    if (fn == nullptr) {
        return false;
    }
    cuuint64_t const dims[2] = {cols, rows};
    cuuint64_t const strides[1] = {stride_elems * 2};
    cuuint32_t const box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
    cuuint32_t const elem_strides[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
               elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
        == CUDA_SUCCESS;
}

int g_sms = 0;

int numSms()
{
    if (g_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms <= 0) {
            g_sms = 148;
        }
    }
    return g_sms;
}

template <int BN, int EPI>
cudaError_t configureOne()
{
    static cudaError_t status = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smemBytes<BN>()));
    return status;
}

template <int BN>
cudaError_t configure(std::uint32_t epi)
{
    switch (epi) {
    case KK_EPI_STORE_F16: return configureOne<BN, KK_EPI_STORE_F16>();
    case KK_EPI_STORE_F32: return configureOne<BN, KK_EPI_STORE_F32>();
    case KK_EPI_RESIDUAL: return configureOne<BN, KK_EPI_RESIDUAL>();
    case KK_EPI_SILU_PAIRS: return configureOne<BN, KK_EPI_SILU_PAIRS>();
    case KK_EPI_QKV_ROPE: return configureOne<BN, KK_EPI_QKV_ROPE>();
    default: return configureOne<BN, KK_EPI_ARGMAX>();
    }
}

} // namespace

struct GemmPlan {
    CUtensorMap tm_w;
    CUtensorMap tm_x;
    GemmArgs args;
    std::uint32_t tiles;
    int bn;
};

void GemmPlanDeleter::operator()(GemmPlan* p) const noexcept { delete p; }

namespace {

int buildArgs(kk_gemm_desc const* d, GemmArgs& args)
{
    if (d == nullptr || d->weight == nullptr || d->x == nullptr || d->M == 0 || d->K == 0
        || d->K % 8 != 0 || d->N == 0 || d->N > 64 || d->x_rows < d->N || d->x_stride < d->K
        || d->x_stride % 8 != 0 || d->epilogue > KK_EPI_ARGMAX
        || (reinterpret_cast<std::uintptr_t>(d->weight) & 15u) != 0
        || (reinterpret_cast<std::uintptr_t>(d->x) & 15u) != 0) {
        return KK_EINVAL;
    }
    if (d->weight_layout > KK_W_PACKED) {
        return KK_EINVAL;
    }
    args = GemmArgs{};
    args.w_packed = d->weight_layout == KK_W_PACKED ? reinterpret_cast<std::uint8_t const*>(d->weight)
                                                    : nullptr;
    args.M = d->M;
    args.K = d->K;
    args.N = d->N;
    args.kb_total = (d->K + kBK - 1) / kBK;
    if (d->norm_input != nullptr) {
        if (d->norm_stride < d->K || d->norm_stride % 8 != 0 || d->K % 8 != 0
            || (reinterpret_cast<std::uintptr_t>(d->norm_input) & 15u) != 0 || !(d->norm_eps >= 0.f)) {
            return KK_EINVAL;
        }
        args.norm_x = reinterpret_cast<__half const*>(d->norm_input);
        args.norm_stride = d->norm_stride;
        args.norm_eps = d->norm_eps;
        if ((reinterpret_cast<std::uintptr_t>(d->norm_weight) & 15u) != 0) {
            return KK_EINVAL;
        }
        args.norm_w = reinterpret_cast<__half const*>(d->norm_weight);
    }
    EpiArgs& e = args.epi;
    e.kind = d->epilogue;
    e.layer = d->layer;
    e.out = d->out;
    e.out_stride = d->out_stride;
    if (d->epilogue != KK_EPI_ARGMAX && d->out == nullptr) {
        return KK_EINVAL;
    }
    if (d->epilogue == KK_EPI_SILU_PAIRS && d->M % 2 != 0) {
        return KK_EINVAL;
    }
    if (d->epilogue == KK_EPI_QKV_ROPE) {
        kk_kv_pools const& p = d->pools;
        if (d->head_dim != 64 || p.head_dim != 64 || d->positions == nullptr || !microPageTokensValid(p)
            || d->slots == nullptr || d->q_rows % 64 != 0 || d->kv_rows % 64 != 0
            || d->kv_rows != p.kv_heads * p.head_dim || d->layer >= p.layers
            || d->M != d->q_rows + 2 * d->kv_rows || !(d->rope_theta > 0.f)) {
            return KK_EINVAL;
        }
        e.positions = d->positions;
        e.slots = d->slots;
        e.micro = static_cast<__half*>(p.micro);
        e.extent = static_cast<__half*>(p.extent);
        e.kv_row = p.kv_heads * p.head_dim;
        e.micro_cap = microPageTokens(p);
        e.micro_page = std::uint64_t(p.layers) * 2u * e.micro_cap * e.kv_row;
        e.extent_page = std::uint64_t(p.layers) * 2u * 64u * e.kv_row;
        e.micro_slots = p.micro == nullptr ? 0 : p.micro_capacity;
        e.extent_slots = p.extent == nullptr ? 0 : p.extent_capacity;
        e.layer = d->layer;
        e.q_rows = d->q_rows;
        e.kv_rows = d->kv_rows;
        e.theta = d->rope_theta;
        if (d->rope_cos_sin != nullptr) {
            if ((reinterpret_cast<std::uintptr_t>(d->rope_cos_sin) & 7u) != 0 || d->rope_positions == 0) {
                return KK_EINVAL;
            }
            e.rope_cs = reinterpret_cast<float2 const*>(d->rope_cos_sin);
            e.rope_positions = d->rope_positions;
        }
    }
    if (d->epilogue == KK_EPI_ARGMAX) {
        if (d->tokens == nullptr || d->argmax_workspace == nullptr) {
            return KK_EINVAL;
        }
        std::uint64_t const tiles = (d->M + 127u) / 128u;
        char* ws = static_cast<char*>(d->argmax_workspace);
        e.counter = reinterpret_cast<std::uint32_t*>(ws);
        e.part_val = reinterpret_cast<float*>(ws + 256);
        e.part_idx = reinterpret_cast<std::uint32_t*>(ws + 256 + tiles * d->N * 4u);
        e.tokens = d->tokens;
    }
    return 0;
}

template <int BN, int EPI>
int runGemmOne(GemmPlan const& plan, cudaStream_t stream)
{
    cudaError_t const c = configureOne<BN, EPI>();
    if (c != cudaSuccess) {
        return static_cast<int>(c);
    }
    return static_cast<int>(launch(gemm_tc_kernel<BN, EPI>, dim3(plan.args.split, plan.tiles),
        dim3(plan.args.norm_x != nullptr ? 64u + xnThreadsFor(EPI) : static_cast<unsigned>(kThreads)),
        smemBytes<BN>(), stream, plan.args.split,
        plan.tm_w, plan.tm_x, plan.args));
}

template <int BN>
int runGemm(GemmPlan const& plan, cudaStream_t stream)
{
    switch (plan.args.epi.kind) {
    case KK_EPI_STORE_F16: return runGemmOne<BN, KK_EPI_STORE_F16>(plan, stream);
    case KK_EPI_STORE_F32: return runGemmOne<BN, KK_EPI_STORE_F32>(plan, stream);
    case KK_EPI_RESIDUAL: return runGemmOne<BN, KK_EPI_RESIDUAL>(plan, stream);
    case KK_EPI_SILU_PAIRS: return runGemmOne<BN, KK_EPI_SILU_PAIRS>(plan, stream);
    case KK_EPI_QKV_ROPE: return runGemmOne<BN, KK_EPI_QKV_ROPE>(plan, stream);
    default: return runGemmOne<BN, KK_EPI_ARGMAX>(plan, stream);
    }
}

} // namespace
} // namespace kk

extern "C" {

uint64_t kk_gemm_packed_bytes(uint32_t M, uint32_t K)
{
    std::uint64_t const tiles = (std::uint64_t(M) + kk::kBM - 1) / kk::kBM;
    std::uint64_t const kb = (std::uint64_t(K) + kk::kBK - 1) / kk::kBK;
    return tiles * kb * kk::kTileWBytes;
}

int kk_gemm_pack_weight(const uint16_t* weight, uint32_t M, uint32_t K, uint16_t* packed,
    void* stream)
{
    return kk_gemm_pack_weight_scaled(weight, M, K, nullptr, packed, stream);
}

int kk_gemm_pack_weight_scaled(const uint16_t* weight, uint32_t M, uint32_t K,
    const uint16_t* col_scale, uint16_t* packed, void* stream)
{
    if (weight == nullptr || packed == nullptr || M == 0 || K == 0 || K % 8 != 0
        || (reinterpret_cast<std::uintptr_t>(weight) & 15u) != 0
        || (reinterpret_cast<std::uintptr_t>(packed) & 15u) != 0
        || (reinterpret_cast<std::uintptr_t>(col_scale) & 15u) != 0) {
        return KK_EINVAL;
    }
    std::uint32_t const kb = (K + kk::kBK - 1) / kk::kBK;
    std::uint64_t const chunks = kk_gemm_packed_bytes(M, K) / 16u;
    std::uint64_t const blocks = (chunks + 255u) / 256u;
    kk::pack_weight_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        weight, M, K, kb, chunks, reinterpret_cast<uint4*>(packed),
        reinterpret_cast<__half const*>(col_scale));
    return static_cast<int>(cudaGetLastError());
}

uint64_t kk_argmax_workspace_bytes(uint32_t M, uint32_t N)
{
    std::uint64_t const tiles = (M + 127u) / 128u;
    return 256u + tiles * N * 8u;
}

int kk_gemm(const kk_gemm_desc* d, void* stream)
{
    int rc = 0;
    kk::GemmPlanPtr const plan = kk::gemmPlan(*d, rc);
    return plan ? kk::gemmRun(*plan, static_cast<cudaStream_t>(stream)) : rc;
}

} // extern "C"

namespace kk {
int gemmStatus(cudaStream_t stream) { return readStatus(&g_gemm_status, stream); }

GemmPlanPtr gemmPlan(kk_gemm_desc const& d, int& rc)
{
    GemmPlanPtr plan(new GemmPlan{});
    rc = buildArgs(&d, plan->args);
    if (rc != 0) {
        return nullptr;
    }
    plan->bn = d.N <= 16 ? 16 : (d.N <= 32 ? 32 : 64);
    if ((d.weight_layout == KK_W_ROW_MAJOR && !makeMap(&plan->tm_w, d.weight, d.K, d.M, d.K, kBM))
        || !makeMap(&plan->tm_x, d.x, d.K, d.x_rows, d.x_stride, static_cast<std::uint32_t>(plan->bn))) {
        rc = KK_EINVAL;
        return nullptr;
    }
    cudaError_t const configured = plan->bn == 16 ? configure<16>(d.epilogue)
        : (plan->bn == 32 ? configure<32>(d.epilogue) : configure<64>(d.epilogue));
    if (configured != cudaSuccess) {
        rc = static_cast<int>(configured);
        return nullptr;
    }
    plan->tiles = (d.M + kBM - 1) / kBM;
    std::uint32_t split = d.split_k;
    if (split == 0) {
        split = 2u * static_cast<std::uint32_t>(numSms()) / plan->tiles;  // ~2 CTAs per SM
    }
    std::uint32_t const max_split = plan->args.kb_total < 8u ? plan->args.kb_total : 8u;
    split = split < 1u ? 1u : (split > max_split ? max_split : split);
    while (split > 1u && split * ((d.N + split - 1u) / split) > recvCols(plan->bn)) {
        --split;
    }
    plan->args.split = split;
    plan->args.epi.num_m_tiles = plan->tiles;
    return plan;
}

bool gemmSetNormPartials(GemmPlan& plan, float const* sq_in, std::uint32_t tiles)
{
    if (plan.args.norm_x == nullptr || sq_in == nullptr || tiles == 0
        || (reinterpret_cast<std::uintptr_t>(sq_in) & 3u) != 0) {
        return false;
    }
    plan.args.sq_in = sq_in;
    plan.args.sq_tiles = tiles;
    return true;
}

bool gemmSetSumSquaresOut(GemmPlan& plan, float* sq_out)
{
    if (plan.args.epi.kind != KK_EPI_RESIDUAL || sq_out == nullptr) {
        return false;
    }
    plan.args.sq_out = sq_out;
    return true;
}

void gemmSetStatus(GemmPlan& plan, unsigned int* status) { plan.args.status = status; }

void gemmSetL2Prefetch(GemmPlan& plan, void const* ptr, std::uint64_t bytes)
{
    bool const ok = ptr != nullptr && (reinterpret_cast<std::uintptr_t>(ptr) & 15u) == 0 && bytes >= 16;
    plan.args.l2_pf = ok ? ptr : nullptr;
    plan.args.l2_pf_bytes = ok ? bytes & ~std::uint64_t(15) : 0;
}

#ifdef KK_TRACE
extern "C" KK_KAPI std::uint32_t kk_trace_read_gemm(void* host, std::uint32_t cap, int reset)
{
    unsigned int n = 0;
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(&n, g_gemm_trace_n, sizeof(n));
    n = n < kTraceCap ? n : kTraceCap;
    n = n < cap ? n : cap;
    if (host != nullptr && n != 0) {
        cudaMemcpyFromSymbol(host, g_gemm_trace, n * sizeof(TraceRec));
    }
    if (reset != 0) {
        unsigned int const zero = 0;
        cudaMemcpyToSymbol(g_gemm_trace_n, &zero, sizeof(zero));
    }
    return n;
}
#endif

int gemmRun(GemmPlan const& plan, cudaStream_t stream)
{
    switch (plan.bn) {
    case 16: return runGemm<16>(plan, stream);
    case 32: return runGemm<32>(plan, stream);
    default: return runGemm<64>(plan, stream);
    }
}
} // namespace kk
