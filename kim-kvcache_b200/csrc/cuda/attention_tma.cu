// K1 (TMA variant) — persistent, TMA-fed GQA paged decode attention for sm_100a.
//
// Same numerics as the direct-load kernel in attention.cu (one pass: QK^T,
// online softmax in FP32, PV, split-KV with a last-CTA combine), organised so
// that every SM streams K/V at close to the HBM read rate:
//
//  * Warp-specialised CTA of 288 threads, one per SM: warp 8 is the producer
//    (the whole warp walks the descriptors in lock step, lane 0 issues the
//    copies), warps 0-7 are consumers.
//  * A stage holds Ts = min(64, 128 / kv_heads) tokens of every KV head, K
//    then V, each laid out [kv_head][token][64 dims] with the 128-byte swizzle
//    (32 KB per stage, 3 stages). An extent page fills a stage with ONE tensor
//    load for K and one for V: the extent tensor map views the pool as
//    [slot][layer*2+kv][kv_head][token][dim] (strides permuted, so the box
//    lands head-major), box 64 dims x Ts tokens x kv_heads. A micro page
//    occupies one 8-token group of a stage and is loaded per head.
//  * Consumer warp w owns KV head w % kv_heads and the 16-token slice
//    w / kv_heads of each stage; its GQA query heads are the rows of m16n8k16
//    tiles (ldmatrix for K as the B operand of QK^T, ldmatrix.trans for V as
//    the B operand of PV), conflict-free thanks to the swizzle.
//  * Work items may span lanes (kk_attention_plan_balanced cuts the batch's
//    token stream into one equal run per SM): a stage never mixes lanes, the
//    producer flags the last stage of each lane segment, and consumers merge
//    and store (or park a partial for the split combine) at that point, then
//    continue with the next lane. A lane's segments use partial slots
//    2*item (first lane of the item) and 2*item+1 (last lane).
//  * Work lists (items, lanes, descriptors) are read before
//    griddepcontrol.wait: under the runner's programmatic dependent launch
//    they come from host copies that precede the whole step. K/V pages and
//    queries are only touched after it.
//  * Every wait is bounded and abort-aware, the consumers' own barrier
//    included (an mbarrier, not a named barrier): a wait that runs out of
//    time records kErrWaitTimeout and raises a CTA-wide abort flag, after
//    which every wait returns at once and all warps run to the end.
#include "../../../include/kk_kernels.h"
#include "kernels_internal.h"
#include "launch.cuh"

#include <cmath>
#include <mutex>
#include <vector>

namespace kk {

__device__ unsigned int g_attn_tma_status;
// Test hook (kk_debug_attention_fault): CTA 0 of every launch drops stage
// g_attn_fault_stage (no copy, no arrival), so its consumers' bounded wait
// runs out; waits give up after g_attn_wait_limit_ns. Defaults: no stage
// dropped, the production limit.
__device__ std::uint32_t g_attn_fault_stage = 0xffffffffu;
__device__ std::uint64_t g_attn_wait_limit_ns = kWaitLimitNs;
#ifdef KK_TRACE
__device__ TraceRec g_attn_trace[kTraceCap];
__device__ unsigned int g_attn_trace_n;
#endif

namespace {

constexpr int kHeadDim = 64;
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
#ifdef KK_ATTN_STAGES
constexpr int kStages = KK_ATTN_STAGES;
#else
constexpr int kStages = 3;
#endif
constexpr std::uint32_t kStageBytes = 32768;           // K 16 KB + V 16 KB
constexpr std::uint32_t kRowBytes = kHeadDim * 2;      // one head x one token
constexpr std::uint32_t kORow = kHeadDim + 4;          // padded merge row (floats)
// Partials a combining thread requests at once: a lane of the balanced plan
// spans about 5-6 items, so all of them arrive in one L2 round trip.
constexpr std::uint32_t kCombineBatch = 8;

constexpr std::uint32_t kSegEnd = 1u;    // last stage of a lane segment
constexpr std::uint32_t kItemEnd = 2u;   // last stage of the item
// The stage holds micro pages loaded whole ([head][8 tokens] per page, page
// n at rows n*kv_heads*8): one load for K and one for V per page.
constexpr std::uint32_t kMicroStage = 4u;
// With kMicroStage: the pages are 16-token pages of a fixed-page pool (page n
// at rows n*kv_heads*16, [head][16 tokens] each), so a 16-token slice is one
// page and its second 8 tokens follow its first within the head's block.
constexpr std::uint32_t kPage16 = 8u;

struct StageMeta {
    // Valid tokens of each 8-token group slot, one byte per slot (0 = empty
    // slot). Packed in one word so neither side indexes an array with a
    // runtime index (that would place it in local memory).
    std::uint64_t valid;
    std::uint32_t lane;     // lane whose tokens the stage holds
    std::uint32_t flags;    // kSegEnd | kItemEnd
    std::uint32_t next_lane;  // lane of the item's next segment (kSegEnd without kItemEnd)
    std::uint32_t pad[3];
};

// One lane segment of a work item, published by the producer with the
// segment's query row.
struct SegInfo {
    std::uint32_t lane;
    std::uint32_t query_row;
    std::uint32_t item_offset;  // the lane's items (split-KV combine)
    std::uint32_t item_count;
    std::uint32_t first_sub;    // 1: the lane's first item wrote its second slot
    std::uint32_t part_slot;    // partial slot this segment writes when split
};

struct TmaArgs {
    std::uint32_t micro_slots;
    std::uint32_t extent_slots;
    std::uint32_t layer;
    std::uint32_t kv_heads;
    std::uint32_t group;          // query heads per KV head
    std::uint32_t q_heads;
    std::uint32_t ts;             // tokens per stage
    std::uint32_t extent_per_head;  // 1: the extent map has per-head boxes (fallback)
    std::uint32_t micro_per_head;   // 1: the micro map has per-head boxes
    std::uint32_t micro_cap;        // tokens per micro page (8, or 16/32/64 for a fixed-page pool)
    std::uint32_t micro_box;        // tokens per micro-map box when micro pages are loaded in chunks
    std::uint32_t micro_packed;     // 1: several whole micro pages share a stage (8- and 16-token pages)
    kk_page_desc const* descs;
    kk_attn_lane const* lanes;
    std::uint32_t num_lanes;
    kk_attn_item const* items;
    std::uint32_t num_items;
    std::uint32_t const* num_items_dev;
    __half const* query;
    std::uint32_t query_stride;
    __half* output;
    std::uint32_t output_stride;
    float scale_log2;
    std::uint32_t* counters;
    float* part_o;
    float* part_ml;
    unsigned int* status;  // error word of this launch (null: the module's word)
};

__device__ __forceinline__ void tma_load_5d_hint(void* dst, CUtensorMap const* map, std::uint64_t* bar,
    int c0, int c1, int c2, int c3, int c4, std::uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2], %8;"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(smem_u32(bar)),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, CUtensorMap const* map, std::uint64_t* bar,
    int c0, int c1, int c2, int c3, int c4)
{
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(map)), "r"(smem_u32(bar)),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
        : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, void const* src, std::uint32_t bytes, std::uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<std::uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(std::uint64_t* bar, std::uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4(std::uint32_t addr, std::uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_t(std::uint32_t addr, std::uint32_t (&r)[4])
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void mma16816(float (&d)[4], std::uint32_t a0, std::uint32_t a1,
    std::uint32_t a2, std::uint32_t a3, std::uint32_t b0, std::uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ std::uint32_t pack_half2(float lo, float hi)
{
    __half2 const h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<std::uint32_t const*>(&h);
}

// Bounded wait (suspending polls, wall-time limit) that also gives up as soon
// as another warp raised the CTA's abort flag.
__device__ __forceinline__ bool wait_or_abort(std::uint64_t* bar, std::uint32_t phase,
    int volatile* abort, unsigned int* status)
{
    if (mbar_poll(bar, phase)) {
        return true;
    }
    std::uint64_t const t0 = global_ns();
    std::uint64_t const limit = *static_cast<std::uint64_t volatile*>(&g_attn_wait_limit_ns);
    for (std::uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        if (mbar_poll(bar, phase)) {
            return true;
        }
        if (*abort) {
            return false;
        }
        if (global_ns() - t0 > limit) {
            break;
        }
    }
    *abort = 1;
    atomicCAS(status, kErrNone, kErrWaitTimeout);
    return false;
}

// Bounded wait that ignores the abort flag: used after an abort to let the
// copies this CTA issued land before it exits.
__device__ __forceinline__ bool wait_bounded(std::uint64_t* bar, std::uint32_t phase)
{
    std::uint64_t const t0 = global_ns();
    for (std::uint32_t i = 0; i < kMaxWaitPolls; ++i) {
        if (mbar_try_wait_suspend(bar, phase)) {
            return true;
        }
        if (global_ns() - t0 > kWaitLimitNs) {
            break;
        }
    }
    return false;
}

__device__ __forceinline__ std::uint32_t atom_add_acq_rel_gpu(std::uint32_t* p, std::uint32_t v)
{
    std::uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void store_row8(__half* out, float const (&acc)[8], float inv)
{
    __align__(16) __half vals[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        vals[e] = __float2half_rn(acc[e] * inv);
    }
    *reinterpret_cast<uint4*>(out) = *reinterpret_cast<uint4 const*>(vals);
}

__device__ __forceinline__ std::uint32_t lane_desc_end(kk_attn_lane const& ln)
{
    return ln.desc_offset + ln.desc_count;
}

// The GQA group's queries as m16n8k16 B fragments of Q^T (k = dim, n = query
// head): n-tile nt holds heads nt*8 .. nt*8+7 of KV head `head`; thread
// (g = lane/4, c = lane%4) holds dims 2c, 2c+1 and 2c+8, 2c+9 of each 16-dim
// k step for head nt*8+g. Heads past the group are zero.
__device__ __forceinline__ std::uint32_t transpose8x8(std::uint32_t x)
{
    std::uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1) paged_attention_tma_kernel(
    const __grid_constant__ CUtensorMap tm_micro, const __grid_constant__ CUtensorMap tm_extent,
    TmaArgs a)
{
    extern __shared__ std::uint8_t smem_raw[];
    // The 128-byte swizzle pattern repeats every 1 KB: align the ring to 1 KB.
    std::uint32_t const pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
    std::uint8_t* ring = smem_raw + pad;
    std::uint32_t const q_bytes = a.q_heads * kRowBytes;  // one query row, all heads
    std::uint8_t* qbuf = ring + kStages * kStageBytes;     // [q_bytes], the current lane segment
    std::uint64_t* full = reinterpret_cast<std::uint64_t*>(qbuf + q_bytes);
    std::uint64_t* empty = full + kStages;
    std::uint64_t* q_full = empty + kStages;   // query row + SegInfo landed
    std::uint64_t* q_empty = q_full + 1;       // every consumer warp took its query
    // Barrier of the consumer threads (the producer never joins). An mbarrier
    // rather than a named barrier, so that its waits are bounded too.
    std::uint64_t* cbar = q_empty + 1;
    StageMeta* meta = reinterpret_cast<StageMeta*>(cbar + 1);
    SegInfo* seg = reinterpret_cast<SegInfo*>(meta + kStages);
    float* s_m = reinterpret_cast<float*>(seg + 1);             // [warp][16]
    float* s_l = s_m + kConsumerWarps * 16;                      // [warp][16]
    float* s_o = s_l + kConsumerWarps * 16;                      // [warp][8*NT][kORow]
    int* s_last = reinterpret_cast<int*>(s_o + kConsumerWarps * 8 * NT * kORow);
    int volatile* s_abort = s_last + 1;

    std::uint32_t const warp = threadIdx.x / 32;
    std::uint32_t const lane = threadIdx.x % 32;
    unsigned int* const st = a.status != nullptr ? a.status : &g_attn_tma_status;
#ifdef KK_TRACE
    __shared__ TraceRec* s_tr;
    if (threadIdx.x == 0) {
        std::uint32_t const slot = atomicAdd(&g_attn_trace_n, 1u);
        s_tr = slot < kTraceCap ? &g_attn_trace[slot] : nullptr;
        if (s_tr != nullptr) {
            s_tr->tag = (0xA0u << 16) | a.layer;
            s_tr->block = blockIdx.x;
            s_tr->smid = sm_id();
            s_tr->aux = 0;
            s_tr->t[0] = global_ns();
        }
    }
#define KK_ATTN_STAMP(i)                 \
    if (s_tr != nullptr) {               \
        s_tr->t[i] = global_ns();        \
    }
#else
#define KK_ATTN_STAMP(i)
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, kConsumerWarps);
        mbar_init(cbar, kConsumerWarps * 32);
        *s_abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();  // dependents only prefetch weights before their own wait
    std::uint32_t num_items = a.num_items;
    if (a.num_items_dev != nullptr && *a.num_items_dev < num_items) {
        num_items = *a.num_items_dev;
    }
    std::uint32_t const Hkv = a.kv_heads;
    std::uint32_t const Ts = a.ts;
    std::uint32_t const groups_per_stage = Ts / 8u;
    std::uint32_t const v_offset = Hkv * Ts * kRowBytes;  // V half of a stage

    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            prefetch_tensormap(&tm_micro);
            prefetch_tensormap(&tm_extent);
        }
        // K/V of a layer is read once per step: first to go from L2. Measured
        // on the c4 step, this keeps the small data that the other kernels
        // re-read (activations, partials, norm statistics, descriptors) in L2
        // (the step is ~3% slower with default priority), although a replay
        // of attention alone is ~1.5% faster without it.
        std::uint64_t const kv_policy = l2_policy_evict_first();
        bool waited = false;
        std::uint32_t stage = 0;
        std::uint32_t qk = 0;  // lane segments started by this CTA
        // Stage that the test hook drops in CTA 0 (none by default).
        std::uint32_t const fault_stage =
            blockIdx.x == 0 ? *static_cast<std::uint32_t volatile*>(&g_attn_fault_stage) : 0xffffffffu;
        // Publishes lane segment qk to the consumers: its bookkeeping in seg
        // and its query row (all heads) copied into qbuf by one bulk copy,
        // both covered by q_full, once the consumers took segment qk - 1's
        // query (q_empty). Consumers only read shared memory, so a new
        // segment costs them no global round trip.
        auto start_segment = [&](kk_attn_lane const& L, std::uint32_t lane_b, std::uint32_t part_slot) -> bool {
            bool const ready = qk == 0u || wait_or_abort(q_empty, (qk - 1u) & 1u, s_abort, st);
            if (!__all_sync(0xffffffffu, ready)) {
                return false;
            }
            if (lane == 0) {
                *seg = SegInfo{lane_b, L.query_row, L.item_offset, L.item_count, L.first_item_shared ? 1u : 0u,
                    part_slot};
                mbar_expect_tx(q_full, q_bytes);
                bulk_load(qbuf, a.query + static_cast<std::uint64_t>(L.query_row) * a.query_stride, q_bytes,
                    q_full);
                mbar_arrive(q_full);  // releases seg; the phase ends when the row lands
            }
            ++qk;
            return true;
        };
        // Before the producer exits: lets the copies this CTA may still have
        // in flight (the last kStages stages, the last query row) land, so
        // that none outlives the CTA when the consumers gave up early.
        auto drain = [&]() {
            if (lane == 0) {
                for (std::uint32_t j = stage > kStages ? stage - kStages : 0u; j < stage; ++j) {
                    if (j != fault_stage) {
                        wait_bounded(&full[j % kStages], (j / kStages) & 1u);
                    }
                }
                if (qk != 0u) {
                    wait_bounded(q_full, (qk - 1u) & 1u);
                }
            }
            __syncwarp();
        };
        for (std::uint32_t it = blockIdx.x; it < num_items; it += gridDim.x) {

            kk_attn_item const item = a.items[it];
            // A half-extent cut: the item's first descriptor starts at token
            // skip0, its last one ends at token limit_last (0: valid count).
            std::uint32_t const skip0 = KK_ATTN_ITEM_SKIP(item.reserved);
            std::uint32_t const limit_last = KK_ATTN_ITEM_LIMIT(item.reserved);
            std::uint32_t b = item.lane;
            if (b >= a.num_lanes) {
                if (lane == 0) {
                    atomicCAS(st, kErrNone, kErrBadArgument);
                }
                b = 0;
            }
            // Lane records are read before griddepcontrol.wait (host data),
            // and the next lane's record is requested one segment ahead.
            kk_attn_lane cur_lane = a.lanes[b];
            kk_attn_lane next_lane = a.lanes[b + 1 < a.num_lanes ? b + 1 : b];
            std::uint32_t seg_end = lane_desc_end(cur_lane);
            seg_end = seg_end < item.desc_end ? seg_end : item.desc_end;
            // 32 descriptors at a time, one per lane, broadcast with shuffles.
            std::uint32_t win = item.desc_begin;
            std::uint32_t w_slot = 0, w_word = 0;
            auto load_window = [&]() {
                std::uint32_t const i = win + lane;
                if (i < item.desc_end) {
                    std::uint32_t const* d = reinterpret_cast<std::uint32_t const*>(a.descs + i);
                    w_slot = d[0];
                    w_word = d[2];
                } else {
                    w_slot = 0;
                    w_word = 0;
                }
            };
            load_window();
            // Cursor over the segment's non-empty, in-bounds descriptors. A
            // descriptor outside its pool or over its page capacity
            // contributes nothing and is reported.
            std::uint32_t e = item.desc_begin;
            std::uint32_t vt = 0, tok = 0;
            int slot = 0;
            bool micro = true;
            bool have = false;
            auto seek = [&]() {
                have = false;
                for (; e < seg_end; ++e) {
                    if (e >= win + 32u) {
                        win += 32u;
                        load_window();
                    }
                    std::uint32_t const j = e - win;
                    std::uint32_t const d_slot = __shfl_sync(0xffffffffu, w_slot, j);
                    std::uint32_t const d_word = __shfl_sync(0xffffffffu, w_word, j);
                    std::uint32_t const valid = d_word & 0xffffu;
                    bool const m = ((d_word >> 16) & 0xffu) == 0;
                    bool const ok = (m ? d_slot < a.micro_slots : d_slot < a.extent_slots)
                        && valid <= (m ? a.micro_cap : 64u);
                    if (!ok) {
                        if (lane == 0) {
                            atomicCAS(st, kErrNone, kErrBadDescriptor);
                        }
                        continue;
                    }
                    std::uint32_t const first = e == item.desc_begin ? skip0 : 0u;
                    std::uint32_t const last = e + 1u == item.desc_end && limit_last != 0u && limit_last < valid
                        ? limit_last : valid;
                    if (m && (first != 0u || last != valid)) {
                        // Only extent pages are cut (a micro page is one box).
                        if (lane == 0) {
                            atomicCAS(st, kErrNone, kErrBadDescriptor);
                        }
                        continue;
                    }
                    if (first < last) {
                        vt = last;
                        tok = first;
                        slot = static_cast<int>(d_slot);
                        micro = m;
                        have = true;
                        return;
                    }
                }
            };
            seek();
            if (!waited) {
                pdl_wait();  // K/V pages and queries are written by the previous kernel
                waited = true;
                if (lane == 0) {
                    KK_ATTN_STAMP(1)
                }
            }
            if (!start_segment(cur_lane, b, 2u * it)) {
                drain();
                return;
            }
            for (;;) {
                std::uint32_t const s = stage % kStages;
                bool const ready = stage < kStages
                    || wait_or_abort(&empty[s], ((stage / kStages) - 1u) & 1u, s_abort, st);
                if (!__all_sync(0xffffffffu, ready)) {
                    drain();
                    return;
                }
                bool const issue = lane == 0 && stage != fault_stage;
                StageMeta m{};
                m.lane = b;
                std::uint8_t* base = ring + s * kStageBytes;
                std::uint32_t const kv = a.layer * 2u;
                std::uint32_t n = 0;
                while (have && n < groups_per_stage) {
                    if (!micro || a.micro_packed == 0) {
                        // A chunk of up to Ts tokens of one page: an extent
                        // page, or a page of a fixed-page micro pool (16-64
                        // tokens; a page shorter than a stage fills the first
                        // rows of each head's block, per-head boxes).
                        if (n != 0) {
                            break;  // a chunk always starts a fresh stage
                        }
                        CUtensorMap const* map = micro ? &tm_micro : &tm_extent;
                        bool const per_head = micro ? a.micro_per_head != 0 : a.extent_per_head != 0;
                        std::uint32_t const bt = micro ? a.micro_box : Ts;
#pragma unroll
                        for (std::uint32_t j = 0; j < 8; ++j) {
                            std::uint32_t const first = tok + 8u * j;
                            std::uint32_t const left = j < groups_per_stage && first < vt ? vt - first : 0u;
                            m.valid |= std::uint64_t(left < 8u ? left : 8u) << (8u * j);
                        }
                        if (issue) {
                            mbar_expect_tx(&full[s], 2u * Hkv * bt * kRowBytes);
                            if (!per_head) {
                                tma_load_5d_hint(base, map, &full[s], 0, static_cast<int>(tok), 0,
                                    static_cast<int>(kv), slot, kv_policy);
                                tma_load_5d_hint(base + v_offset, map, &full[s], 0, static_cast<int>(tok),
                                    0, static_cast<int>(kv + 1), slot, kv_policy);
                            } else {
                                for (std::uint32_t h = 0; h < Hkv; ++h) {
                                    std::uint8_t* dst = base + h * Ts * kRowBytes;
                                    tma_load_5d_hint(dst, map, &full[s], 0, static_cast<int>(h),
                                        static_cast<int>(tok), static_cast<int>(kv), slot, kv_policy);
                                    tma_load_5d_hint(dst + v_offset, map, &full[s], 0, static_cast<int>(h),
                                        static_cast<int>(tok), static_cast<int>(kv + 1), slot, kv_policy);
                                }
                            }
                        }
                        n = groups_per_stage;
                        tok += Ts;
                        if (tok >= vt) {
                            ++e;
                            seek();
                        }
                    } else if (a.micro_cap == 16u) {
                        // A whole 16-token page (two groups) per box; pages
                        // of this pool start at even groups.
                        std::uint32_t const lo = vt < 8u ? vt : 8u;
                        m.valid |= (std::uint64_t(lo) << (8u * n)) | (std::uint64_t(vt - lo) << (8u * (n + 1u)));
                        m.flags |= kMicroStage | kPage16;
                        if (issue) {
                            mbar_expect_tx(&full[s], 2u * Hkv * 16u * kRowBytes);
                            std::uint8_t* dst = base + n * Hkv * 8u * kRowBytes;
                            tma_load_5d_hint(dst, &tm_micro, &full[s], 0, 0, 0, static_cast<int>(kv), slot, kv_policy);
                            tma_load_5d_hint(dst + v_offset, &tm_micro, &full[s], 0, 0, 0,
                                static_cast<int>(kv + 1), slot, kv_policy);
                        }
                        n += 2u;
                        ++e;
                        seek();
                    } else {
                        m.valid |= std::uint64_t(vt) << (8u * n);
                        if (a.micro_per_head == 0) {
                            m.flags |= kMicroStage;
                            if (issue) {
                                mbar_expect_tx(&full[s], 2u * Hkv * 8u * kRowBytes);
                                std::uint8_t* dst = base + n * Hkv * 8u * kRowBytes;
                                tma_load_5d_hint(dst, &tm_micro, &full[s], 0, 0, 0, static_cast<int>(kv), slot, kv_policy);
                                tma_load_5d_hint(dst + v_offset, &tm_micro, &full[s], 0, 0, 0,
                                    static_cast<int>(kv + 1), slot, kv_policy);
                            }
                        } else if (issue) {
                            mbar_expect_tx(&full[s], 2u * Hkv * 8u * kRowBytes);
                            for (std::uint32_t h = 0; h < Hkv; ++h) {
                                std::uint8_t* dst = base + (h * Ts + n * 8u) * kRowBytes;
                                tma_load_5d_hint(dst, &tm_micro, &full[s], 0, static_cast<int>(h), 0,
                                    static_cast<int>(kv), slot, kv_policy);
                                tma_load_5d_hint(dst + v_offset, &tm_micro, &full[s], 0, static_cast<int>(h), 0,
                                    static_cast<int>(kv + 1), slot, kv_policy);
                            }
                        }
                        ++n;
                        ++e;
                        seek();
                    }
                }
                bool item_done = false;
                bool next_segment = false;
                if (!have) {
                    // This lane's segment is exhausted: the next one starts at
                    // the next lane with descriptors (lanes are contiguous in
                    // the descriptor array inside a multi-lane item).
                    m.flags |= kSegEnd;
                    e = seg_end;
                    if (e >= item.desc_end) {
                        m.flags |= kItemEnd;
                        item_done = true;
                    } else {
                        std::uint32_t nb = b + 1;
                        if (nb < a.num_lanes) {
                            cur_lane = next_lane;  // lanes[b + 1], requested a segment ago
                            while (cur_lane.desc_count == 0 && ++nb < a.num_lanes) {
                                cur_lane = a.lanes[nb];
                            }
                        }
                        if (nb >= a.num_lanes || cur_lane.desc_offset != e) {
                            if (lane == 0) {
                                atomicCAS(st, kErrNone, kErrBadArgument);
                            }
                            m.flags |= kItemEnd;
                            item_done = true;
                        } else {
                            b = nb;
                            m.next_lane = b;
                            next_lane = a.lanes[b + 1 < a.num_lanes ? b + 1 : b];
                            seg_end = lane_desc_end(cur_lane);
                            seg_end = seg_end < item.desc_end ? seg_end : item.desc_end;
                            next_segment = true;
                        }
                    }
                }
                if (issue) {
                    meta[s] = m;
                    mbar_arrive(&full[s]);  // releases meta[s]; the phase ends when the bytes land
                }
                ++stage;
                if (item_done) {
                    break;
                }
                if (next_segment && !start_segment(cur_lane, b, 2u * it + 1u)) {
                    drain();
                    return;
                }
                if (!have) {
                    seek();
                }
            }
        }
        if (lane == 0) {
            KK_ATTN_STAMP(2)
        }
        // No CTA exits with its own copies in flight, also when the
        // consumers gave up on an earlier stage.
        drain();
        return;
    }

    // ------------------------------ consumers ------------------------------
    // Scores are computed transposed, S^T = K Q^T (rows = 16 tokens of the
    // slice, columns = up to 8*NT query heads), and the output as
    // O^T = V^T P^T (rows = 16 dims per m-tile, columns = query heads), so no
    // MMA row is spent on padding when a GQA group has 8 heads.
    std::uint32_t const g = lane >> 2;   // token (or dim) row within an 8-row block
    std::uint32_t const c4 = lane & 3;
    std::uint32_t const head = warp % Hkv;
    std::uint32_t const chunk = warp / Hkv;  // 16-token slice of each stage
    bool const active = chunk * 16u < Ts;
    std::uint32_t const warps_per_head = kConsumerWarps / Hkv;
    std::uint32_t const G = a.group;
    std::uint32_t const tid = threadIdx.x;  // 0 .. 255
    float const kNegInf = -INFINITY;
    std::uint32_t const ring_base = smem_u32(ring);
    std::uint32_t const mi = lane >> 3;  // ldmatrix: which 8x8 matrix this lane addresses
    std::uint32_t const r8 = lane & 7;
    std::uint32_t stage = 0;
    std::uint32_t ck = 0;  // lane segments consumed
    std::uint32_t cphase = 0;
    auto consumer_sync = [&]() {
        mbar_arrive(cbar);
        wait_or_abort(cbar, cphase, s_abort, st);
        cphase ^= 1u;
    };
    // Takes lane segment ck from the producer: its bookkeeping and this
    // warp's query fragments (B operand of S^T = K Q^T), then hands the query
    // buffer back.
    std::uint32_t qf[NT][4][2];
    SegInfo si{};
    auto begin_segment = [&]() -> bool {
        if (*s_abort || !wait_or_abort(q_full, ck & 1u, s_abort, st)) {
            return false;
        }
        si = *seg;
        std::uint8_t const* q = qbuf + head * G * kRowBytes;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            std::uint32_t const qh = nt * 8u + g;
#pragma unroll
            for (int k16 = 0; k16 < 4; ++k16) {
#pragma unroll
                for (int hi = 0; hi < 2; ++hi) {
                    std::uint32_t const col = k16 * 16 + hi * 8 + c4 * 2;
                    qf[nt][k16][hi] = qh < G
                        ? *reinterpret_cast<std::uint32_t const*>(q + qh * kRowBytes + col * 2u) : 0u;
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(q_empty);
        }
        ++ck;
        return true;
    };
    // A split lane's completion count is taken at its segment end, but the
    // answer (was this CTA the lane's last?) is read only at the next segment
    // end or at the end of the CTA's work, so the atomic's round trip is off
    // the critical path. The combine runs when the answer is read.
    bool pending = false;
    SegInfo pend{};
    std::uint32_t pend_done = 0;  // meaningful in thread 0
    std::uint32_t pend_stage = 0;
    auto combine = [&](SegInfo const& sg) {
        // Every partial of lane sg.lane: item j = item_offset + i wrote slot
        // 2j, except the lane's first item, which wrote slot 2j + 1 when it
        // started with an earlier lane. Loads of kCombineBatch items are
        // issued together and folded with an online rescale, so a combine
        // costs one L2 round trip for the lanes of the balanced plan.
        std::uint32_t const first = sg.item_offset;
        std::uint32_t const count = sg.item_count;
        for (std::uint32_t idx = tid; idx < a.q_heads * 8u; idx += kConsumerWarps * 32) {
            std::uint32_t const qh = idx / 8u;
            std::uint32_t const d0 = (idx % 8u) * 8u;
            float M = kNegInf;
            float L = 0.f;
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (std::uint32_t i0 = 0; i0 < count; i0 += kCombineBatch) {
                float2 ml[kCombineBatch];
                float4 lo[kCombineBatch], hi[kCombineBatch];
#pragma unroll
                for (std::uint32_t k = 0; k < kCombineBatch; ++k) {
                    std::uint32_t const i = i0 + k;
                    if (i < count) {
                        std::uint64_t const sl = 2ull * (first + i) + (i == 0 ? sg.first_sub : 0u);
                        std::uint64_t const prow = sl * a.q_heads + qh;
                        ml[k] = __ldcg(reinterpret_cast<float2 const*>(a.part_ml) + prow);
                        float4 const* po = reinterpret_cast<float4 const*>(a.part_o + prow * kHeadDim + d0);
                        lo[k] = __ldcg(po);
                        hi[k] = __ldcg(po + 1);
                    } else {
                        ml[k] = make_float2(kNegInf, 0.f);
                        lo[k] = hi[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
#pragma unroll
                for (std::uint32_t k = 0; k < kCombineBatch; ++k) {
                    float const m_new = fmaxf(M, ml[k].x);
                    float const m_use = m_new == kNegInf ? 0.f : m_new;
                    float const fo = exp2f(M - m_use);       // rescale of what is folded so far
                    float const fk = exp2f(ml[k].x - m_use);  // weight of partial k
                    L = L * fo + ml[k].y * fk;
                    acc[0] = acc[0] * fo + lo[k].x * fk;
                    acc[1] = acc[1] * fo + lo[k].y * fk;
                    acc[2] = acc[2] * fo + lo[k].z * fk;
                    acc[3] = acc[3] * fo + lo[k].w * fk;
                    acc[4] = acc[4] * fo + hi[k].x * fk;
                    acc[5] = acc[5] * fo + hi[k].y * fk;
                    acc[6] = acc[6] * fo + hi[k].z * fk;
                    acc[7] = acc[7] * fo + hi[k].w * fk;
                    M = m_new;
                }
            }
            store_row8(a.output + static_cast<std::uint64_t>(sg.query_row) * a.output_stride
                    + qh * kHeadDim + d0, acc, 1.f / L);
        }
        if (tid == 0) {
            a.counters[sg.lane] = 0;  // ready for the next launch
        }
    };
    // Reads the pending lane's answer (thread 0 wrote s_last before calling)
    // and combines it if this CTA was the lane's last.
    auto resolve_pending = [&]() {
        consumer_sync();  // thread 0's acquire reaches the other consumers through this barrier
        if (*s_last) {
            combine(pend);
        }
        pending = false;
    };

    for (std::uint32_t it = blockIdx.x; it < num_items; it += gridDim.x) {
        if (!begin_segment()) {
            break;
        }
        // Per query head (nt*8 + 2*c4 + e): running max (same in all 8 g-lanes)
        // and this lane's share of the softmax denominator.
        float mrow[NT][2], lrow[NT][2];
        float o[NT][4][4];  // [nt][dim m-tile][dim g|g+8 x head e]
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            mrow[nt][0] = mrow[nt][1] = kNegInf;
            lrow[nt][0] = lrow[nt][1] = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.f;
            }
        }
        for (;;) {

            std::uint32_t const s = stage % kStages;
            if (*s_abort || !wait_or_abort(&full[s], (stage / kStages) & 1u, s_abort, st)) {
                break;
            }
#ifdef KK_TRACE
            if (stage == 0 && threadIdx.x == 0) {
                KK_ATTN_STAMP(3)
            }
#endif
            StageMeta const m = meta[s];
            std::uint32_t const pair =
                chunk < 4u ? static_cast<std::uint32_t>(m.valid >> (16u * chunk)) & 0xffffu : 0u;
            std::uint32_t const v0 = active ? (pair & 0xffu) : 0u;
            std::uint32_t const v1 = active ? (pair >> 8) : 0u;
            if (v0 + v1 != 0) {
                // Row of slice token r: r itself in an extent stage; in a
                // micro stage token r lives in page 2*chunk + r/8, whose
                // [head][8 tokens] block starts every kv_heads*8 rows.
                std::uint32_t const step8 = (m.flags & kMicroStage) ? Hkv * 8u : 8u;
                std::uint32_t const gstep = (m.flags & kPage16) ? 8u : step8;  // second 8 tokens of the slice
                std::uint32_t const hrows = (m.flags & kMicroStage) ? ((m.flags & kPage16) ? 16u : 8u) : Ts;
                std::uint32_t const kbase = ring_base + s * kStageBytes
                    + (head * hrows + chunk * 2u * step8) * kRowBytes;
                std::uint32_t const vbase = kbase + v_offset;
                // S^T = K Q^T over the slice's 16 tokens: K rows are the A operand.
                float st[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    st[nt][0] = st[nt][1] = st[nt][2] = st[nt][3] = 0.f;
                }
#pragma unroll
                for (std::uint32_t k16 = 0; k16 < 4; ++k16) {
                    std::uint32_t const row = (mi & 1u) * gstep + r8;
                    std::uint32_t const ch = 2u * k16 + (mi >> 1);
                    std::uint32_t ka[4];
                    ldsm_x4(kbase + row * kRowBytes + ((ch ^ r8) << 4), ka);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816(st[nt], ka[0], ka[1], ka[2], ka[3], qf[nt][k16][0], qf[nt][k16][1]);
                    }
                }
                bool const tg = g < v0;       // token g of the slice
                bool const tg8 = g < v1;      // token g + 8
                // V^T rows are the A operand of O^T += V^T P^T. V halves of
                // masked tokens are zeroed: bytes past a page's valid tokens
                // are never trusted (0 * NaN would be NaN).
                std::uint32_t const mask0 = (2 * c4 < v0 ? 0x0000ffffu : 0u) | (2 * c4 + 1 < v0 ? 0xffff0000u : 0u);
                std::uint32_t const mask1 = (2 * c4 < v1 ? 0x0000ffffu : 0u) | (2 * c4 + 1 < v1 ? 0xffff0000u : 0u);
                // P is handed to the FP16 PV product as hi + lo halves
                // (p = hi + lo to ~2^-22 relative), so the weights keep FP32
                // precision as in the reference's softmax (which multiplies
                // FP32 probabilities into V, paged_decode_kernels.cu:420-470).
                std::uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float p[4];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float const xa = tg ? st[nt][e] * a.scale_log2 : kNegInf;
                        float const xb = tg8 ? st[nt][2 + e] * a.scale_log2 : kNegInf;
                        float mx = fmaxf(xa, xb);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        float const m_new = fmaxf(mrow[nt][e], mx);
                        float const m_use = m_new == kNegInf ? 0.f : m_new;
                        float const alpha = exp2f(mrow[nt][e] - m_use);
                        p[e] = exp2f(xa - m_use);
                        p[2 + e] = exp2f(xb - m_use);
                        lrow[nt][e] = lrow[nt][e] * alpha + p[e] + p[2 + e];
                        mrow[nt][e] = m_new;
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            o[nt][j][e] *= alpha;
                            o[nt][j][2 + e] *= alpha;
                        }
                    }
                    // P^T fragments (token rows, head columns) transposed into
                    // the B layout of the PV product (k = token, n = head).
                    __half2 const h01 = __floats2half2_rn(p[0], p[1]);
                    __half2 const h23 = __floats2half2_rn(p[2], p[3]);
                    pb[nt][0] = transpose8x8(*reinterpret_cast<std::uint32_t const*>(&h01));
                    pb[nt][1] = transpose8x8(*reinterpret_cast<std::uint32_t const*>(&h23));
                    pl[nt][0] = transpose8x8(pack_half2(p[0] - __low2float(h01), p[1] - __high2float(h01)));
                    pl[nt][1] = transpose8x8(pack_half2(p[2] - __low2float(h23), p[3] - __high2float(h23)));
                }
#pragma unroll
                for (std::uint32_t j = 0; j < 4; ++j) {
                    std::uint32_t const row = (mi >> 1) * gstep + r8;
                    std::uint32_t const ch = 2u * j + (mi & 1u);
                    std::uint32_t va[4];
                    ldsm_x4_t(vbase + row * kRowBytes + ((ch ^ r8) << 4), va);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma16816(o[nt][j], va[0] & mask0, va[1] & mask0, va[2] & mask1, va[3] & mask1,
                            pb[nt][0], pb[nt][1]);
                        mma16816(o[nt][j], va[0] & mask0, va[1] & mask0, va[2] & mask1, va[3] & mask1,
                            pl[nt][0], pl[nt][1]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[s]);
            }
            ++stage;
            if ((m.flags & kSegEnd) == 0) {
                // Two stages after a split lane's completion count was taken
                // its answer has arrived: combine now, while the producer
                // keeps the ring full, rather than at the next segment end.
                if (pending && stage == pend_stage + 2u) {
                    if (tid == 0) {
                        *s_last = pend_done + 1 == pend.item_count;
                    }
                    resolve_pending();
                }
                continue;
            }

            // ---- end of lane b's segment: merge the warps of each KV head ----
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float l = lrow[nt][e];
                    l += __shfl_xor_sync(0xffffffffu, l, 4);
                    l += __shfl_xor_sync(0xffffffffu, l, 8);
                    l += __shfl_xor_sync(0xffffffffu, l, 16);
                    std::uint32_t const qh = nt * 8u + 2u * c4 + e;
                    if (g == 0) {
                        s_m[warp * 16 + qh] = mrow[nt][e];
                        s_l[warp * 16 + qh] = l;
                    }
                    float* dst = s_o + (warp * 8 * NT + qh) * kORow;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        dst[16 * j + g] = o[nt][j][e];
                        dst[16 * j + 8 + g] = o[nt][j][2 + e];
                    }
                }
            }
            consumer_sync();
            // A split lane needs the caller's workspace; without one it is
            // reported and its partial is dropped.
            bool const split = si.item_count > 1 && a.part_o != nullptr;
            if (si.item_count > 1 && a.part_o == nullptr && tid == 0) {
                atomicCAS(st, kErrNone, kErrBadArgument);
            }
            bool const keep = si.item_count <= 1 || split;
            for (std::uint32_t idx = tid; idx < a.q_heads * 8u; idx += kConsumerWarps * 32) {
                std::uint32_t const qh = idx / 8u;
                std::uint32_t const d0 = (idx % 8u) * 8u;
                std::uint32_t const h = qh / G;
                std::uint32_t const gq = qh % G;
                float M = kNegInf;
                for (std::uint32_t sub = 0; sub < warps_per_head; ++sub) {
                    M = fmaxf(M, s_m[(sub * Hkv + h) * 16 + gq]);
                }
                float const m_use = M == kNegInf ? 0.f : M;
                float L = 0.f;
                float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                for (std::uint32_t sub = 0; sub < warps_per_head; ++sub) {
                    std::uint32_t const w = sub * Hkv + h;
                    float const f = exp2f(s_m[w * 16 + gq] - m_use);
                    L += s_l[w * 16 + gq] * f;
                    float const* src = s_o + (w * 8 * NT + gq) * kORow + d0;
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        acc[e] += src[e] * f;
                    }
                }
                if (!split) {
                    if (keep) {
                        store_row8(a.output + static_cast<std::uint64_t>(si.query_row) * a.output_stride
                                + qh * kHeadDim + d0, acc, 1.f / L);
                    }
                } else {
                    std::uint64_t const prow = std::uint64_t(si.part_slot) * a.q_heads + qh;
                    float4* po = reinterpret_cast<float4*>(a.part_o + prow * kHeadDim + d0);
                    po[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
                    po[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
                    if (d0 == 0) {
                        reinterpret_cast<float2*>(a.part_ml)[prow] = make_float2(M, L);
                    }
                }
            }
            // This segment's partial is written (CTA scope) and s_m / s_l / s_o
            // are free for the next segment once every consumer is here.
            consumer_sync();
            if (tid == 0) {
                if (pending) {
                    *s_last = pend_done + 1 == pend.item_count;
                }
                if (split) {
                    // Release (cumulative over the partial stores of every
                    // consumer thread, ordered before this one by the
                    // consumer barrier) and acquire in one atomic: the CTA
                    // that counts last also sees every other partial.
                    pend_done = atom_add_acq_rel_gpu(&a.counters[si.lane], 1u);
                }
            }
            if (pending) {
                resolve_pending();
            }
            if (split) {
                pending = true;
                pend = si;
                pend_stage = stage;
            }
            if (m.flags & kItemEnd) {
                break;
            }
            // Next lane of this item.
            if (!begin_segment()) {
                break;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                mrow[nt][0] = mrow[nt][1] = kNegInf;
                lrow[nt][0] = lrow[nt][1] = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    o[nt][j][0] = o[nt][j][1] = o[nt][j][2] = o[nt][j][3] = 0.f;
                }
            }
        }
        if (*s_abort) {
            break;
        }
    }
#ifdef KK_TRACE
    if (tid == 0) {
        KK_ATTN_STAMP(4)
    }
#endif
    if (pending && !*s_abort) {
        if (tid == 0) {
            *s_last = pend_done + 1 == pend.item_count;
        }
        resolve_pending();
    }
#ifdef KK_TRACE
    if (tid == 0) {
        KK_ATTN_STAMP(5)
        if (s_tr != nullptr) {
            s_tr->aux = (pending ? 0x80000000u : 0u) | stage;
        }
    }
#endif
}

// About 122 KB with NT = 1 at 32 query heads: small enough that a
// projection CTA (99 KB) of the neighbouring kernels fits on the same SM, so
// programmatic dependent launch can overlap their prologues and tails with
// this kernel.
template <int NT>
constexpr std::size_t smemBytes(std::uint32_t q_heads)
{
    return 1024 + kStages * kStageBytes + std::size_t(q_heads) * kRowBytes
        + (2 * kStages + 3) * 8 + kStages * sizeof(StageMeta) + sizeof(SegInfo)
        + 2 * kConsumerWarps * 16 * 4 + kConsumerWarps * 8 * NT * kORow * 4 + 8;
}
static_assert(smemBytes<2>(128) <= 227 * 1024, "shared memory budget");

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
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess
            && q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiledFn>(p);
        }
    });
    return fn;
}

bool encode(CUtensorMap* map, void const* base, cuuint64_t const (&dims)[5],
    cuuint64_t const (&strides)[4], cuuint32_t const (&box)[5])
{
    EncodeTiledFn const fn = encodeFn();
    cuuint32_t const elem[5] = {1, 1, 1, 1, 1};
    return fn != nullptr
        && fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE)
        == CUDA_SUCCESS;
}

// Natural view [slot][layer*2+kv][token][kv_head][dim] of a pool of `cap`-token
// pages, box = one head x box_tokens tokens.
bool encodePerHead(CUtensorMap* map, void const* base, std::uint32_t pages, std::uint32_t cap,
    std::uint32_t layers, std::uint32_t heads, std::uint32_t box_tokens)
{
    cuuint64_t const row = kRowBytes;
    cuuint64_t const dims[5] = {kHeadDim, heads, cap, 2ull * layers, pages};
    cuuint64_t const strides[4] = {row, row * heads, row * heads * cap, row * heads * cap * 2ull * layers};
    cuuint32_t const box[5] = {kHeadDim, 1, box_tokens, 1, 1};
    return encode(map, base, dims, strides, box);
}

// Head-major view [slot][layer*2+kv][kv_head][token][dim] of a pool of
// `cap`-token pages (token and head strides swapped), box = all heads x
// box_tokens tokens, so that one load lands [head][token][dim] in shared
// memory.
bool encodeHeadMajor(CUtensorMap* map, void const* base, std::uint32_t pages, std::uint32_t cap,
    std::uint32_t layers, std::uint32_t heads, std::uint32_t box_tokens)
{
    cuuint64_t const row = kRowBytes;
    cuuint64_t const dims[5] = {kHeadDim, cap, heads, 2ull * layers, pages};
    cuuint64_t const strides[4] = {row * heads, row, row * heads * cap, row * heads * cap * 2ull * layers};
    cuuint32_t const box[5] = {kHeadDim, box_tokens, heads, 1, 1};
    return encode(map, base, dims, strides, box);
}

struct PoolMaps {
    kk_kv_pools pools;
    int device;
    CUtensorMap micro;
    CUtensorMap extent;
    bool extent_per_head;
    bool micro_per_head;
    std::uint32_t micro_box;
    bool micro_packed;
};

std::uint32_t stageTokens(std::uint32_t kv_heads)
{
    std::uint32_t const t = 128u / kv_heads;
    return t < 64u ? t : 64u;
}

// Tensor maps are encoded once per (device, pool set) and reused.
bool poolMaps(kk_kv_pools const& p, PoolMaps& out)
{
    static std::mutex mutex;
    static std::vector<PoolMaps> cache;
    int device = 0;
    cudaGetDevice(&device);
    std::lock_guard<std::mutex> lock(mutex);
    for (PoolMaps const& e : cache) {
        if (e.device == device && e.pools.micro == p.micro && e.pools.extent == p.extent
            && e.pools.micro_capacity == p.micro_capacity
            && e.pools.extent_capacity == p.extent_capacity && e.pools.layers == p.layers
            && e.pools.kv_heads == p.kv_heads && e.pools.micro_page_tokens == p.micro_page_tokens) {
            out = e;
            return true;
        }
    }
    PoolMaps e{p, device, {}, {}, false, false, 8, false};
    std::uint32_t const ts = stageTokens(p.kv_heads);
    std::uint32_t const mcap = microPageTokens(p);
    if (mcap == 16u && ts > 16u
        && encodeHeadMajor(&e.micro, p.micro, p.micro_capacity, 16, p.layers, p.kv_heads, 16)) {
        // 16-token pages packed whole, several per stage (like 8-token pages).
        e.micro_per_head = false;
        e.micro_packed = true;
        e.micro_box = 16;
    } else if (mcap != 8u) {
        // Pages of a fixed-page pool, loaded in chunks like extent pages:
        // one box per stage when a page fills a stage, per-head boxes of the
        // whole page otherwise.
        e.micro_box = mcap < ts ? mcap : ts;
        if (e.micro_box == ts
            && encodeHeadMajor(&e.micro, p.micro, p.micro_capacity, mcap, p.layers, p.kv_heads, ts)) {
            e.micro_per_head = false;
        } else if (encodePerHead(&e.micro, p.micro, p.micro_capacity, mcap, p.layers, p.kv_heads, e.micro_box)) {
            e.micro_per_head = true;
        } else {
            return false;
        }
    } else if (encodeHeadMajor(&e.micro, p.micro, p.micro_capacity, 8, p.layers, p.kv_heads, 8)) {
        e.micro_per_head = false;
        e.micro_packed = true;
    } else if (encodePerHead(&e.micro, p.micro, p.micro_capacity, 8, p.layers, p.kv_heads, 8)) {
        e.micro_per_head = true;
        e.micro_packed = true;
    } else {
        return false;
    }
    if (p.extent == nullptr || p.extent_capacity == 0) {
        // No descriptor can select the extent map (extent_slots is 0).
        e.extent = e.micro;
        e.extent_per_head = true;
    } else if (encodeHeadMajor(&e.extent, p.extent, p.extent_capacity, 64, p.layers, p.kv_heads, ts)) {
        e.extent_per_head = false;
    } else if (encodePerHead(&e.extent, p.extent, p.extent_capacity, 64, p.layers, p.kv_heads, ts)) {
        e.extent_per_head = true;
    } else {
        return false;
    }
    if (cache.size() >= 64) {
        cache.erase(cache.begin());
    }
    cache.push_back(e);
    out = e;
    return true;
}

int smCount()
{
    int device = 0;
    int sms = 0;
    cudaGetDevice(&device);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    return sms > 0 ? sms : 148;
}

} // namespace

bool attentionTmaSupported(kk_kv_pools const* pools, std::uint32_t q_heads)
{
    return pools != nullptr && pools->head_dim == kHeadDim && pools->micro != nullptr
        && pools->micro_capacity != 0 && microPageTokensValid(*pools)
        && (pools->kv_heads == 1 || pools->kv_heads == 2 || pools->kv_heads == 4 || pools->kv_heads == 8)
        && q_heads % pools->kv_heads == 0 && q_heads / pools->kv_heads <= 16;
}

int attentionTmaLaunch(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint32_t const* num_items_dev,
    std::uint16_t const* query, std::uint32_t query_stride, std::uint16_t* output,
    std::uint32_t output_stride, float scale, std::uint32_t* counters, float* part_o, float* part_ml,
    unsigned int* status, cudaStream_t stream)
{
    PoolMaps maps{};
    if (!poolMaps(*pools, maps)) {
        return KK_EINVAL;
    }
    static cudaError_t const attr1 = cudaFuncSetAttribute(paged_attention_tma_kernel<1>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smemBytes<1>(128)));
    static cudaError_t const attr2 = cudaFuncSetAttribute(paged_attention_tma_kernel<2>,
        cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smemBytes<2>(128)));
    if (attr1 != cudaSuccess || attr2 != cudaSuccess) {
        return static_cast<int>(attr1 != cudaSuccess ? attr1 : attr2);
    }
    TmaArgs a{};
    a.micro_slots = pools->micro_capacity;
    a.extent_slots = pools->extent == nullptr ? 0 : pools->extent_capacity;
    a.layer = layer;
    a.kv_heads = pools->kv_heads;
    a.group = q_heads / pools->kv_heads;
    a.q_heads = q_heads;
    a.ts = stageTokens(pools->kv_heads);
    a.extent_per_head = maps.extent_per_head ? 1u : 0u;
    a.micro_per_head = maps.micro_per_head ? 1u : 0u;
    a.micro_cap = microPageTokens(*pools);
    a.micro_box = maps.micro_box;
    a.micro_packed = maps.micro_packed ? 1u : 0u;
    a.descs = descs;
    a.lanes = lanes;
    a.num_lanes = num_lanes;
    a.items = items;
    a.num_items = num_items;
    a.num_items_dev = num_items_dev;
    a.query = reinterpret_cast<__half const*>(query);
    a.query_stride = query_stride;
    a.output = reinterpret_cast<__half*>(output);
    a.output_stride = output_stride;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.counters = counters;
    a.part_o = part_o;
    a.part_ml = part_ml;
    a.status = status;
    static int const sms = smCount();
    unsigned const grid = num_items < unsigned(sms) ? num_items : unsigned(sms);
    bool const narrow = a.group <= 8;
    auto const kernel = narrow ? paged_attention_tma_kernel<1> : paged_attention_tma_kernel<2>;
    std::size_t const smem = narrow ? smemBytes<1>(q_heads) : smemBytes<2>(q_heads);
    return static_cast<int>(launch(kernel, dim3(grid), dim3(kThreads), smem, stream, 1,
        maps.micro, maps.extent, a));
}

int attentionTmaStatus(cudaStream_t stream) { return readStatus(&g_attn_tma_status, stream); }

} // namespace kk

extern "C" int kk_debug_attention_fault(uint32_t stage, uint64_t wait_limit_ns)
{
    cudaError_t e = cudaMemcpyToSymbol(kk::g_attn_fault_stage, &stage, sizeof(stage));
    if (e == cudaSuccess) {
        std::uint64_t const limit = wait_limit_ns == 0 ? kk::kWaitLimitNs : wait_limit_ns;
        e = cudaMemcpyToSymbol(kk::g_attn_wait_limit_ns, &limit, sizeof(limit));
    }
    return static_cast<int>(e);
}

namespace kk {

#ifdef KK_TRACE
extern "C" KK_KAPI std::uint32_t kk_trace_read_attn(void* host, std::uint32_t cap, int reset)
{
    unsigned int n = 0;
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(&n, g_attn_trace_n, sizeof(n));
    n = n < kTraceCap ? n : kTraceCap;
    n = n < cap ? n : cap;
    if (host != nullptr && n != 0) {
        cudaMemcpyFromSymbol(host, g_attn_trace, n * sizeof(TraceRec));
    }
    if (reset != 0) {
        unsigned int const zero = 0;
        cudaMemcpyToSymbol(g_attn_trace_n, &zero, sizeof(zero));
    }
    return n;
}
#endif

} // namespace kk
