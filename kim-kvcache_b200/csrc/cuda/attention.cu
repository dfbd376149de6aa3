// K1 — fused GQA paged decode attention for sm_100a.
//
// Replaces the reference's two-kernel split (scores, then softmax+PV, with a
// per-token linear descriptor scan: src/cuda/attention/paged_decode_kernels.cu
// :132-474) by one pass per layer over all lanes:
//
//  * Work items are runs of a lane's block-table entries (micro or extent
//    pages) of roughly equal token count (kk_attention_plan); a persistent
//    grid walks them.
//  * A CTA has 8 warps; each warp owns one KV head and a strided subset of the
//    item's 8-token groups. The 8 query heads of the GQA group form the rows of
//    an m16n8k16 tensor-core tile, so K/V are read once per group.
//  * Each quad of a warp loads one 128-byte token-head row of K (and of V)
//    straight from HBM into registers: K is already a B fragment once the
//    head dimension is permuted consistently in Q and K; V is transposed in
//    registers with movmatrix. No shared-memory staging, no bank conflicts.
//  * Online softmax in FP32 (exp2 with the scale folded in), PV accumulated in
//    FP32; the warps of a head merge in shared memory; lanes split over several
//    items are combined by the last CTA to finish (completion counter), which
//    writes the FP16 output.
#include "../../../include/kk_kernels.h"
#include "kernels_internal.h"
#include "launch.cuh"

#include <atomic>
#include <cmath>
#include <mutex>
#include <vector>

namespace kk {

__device__ unsigned int g_attn_status;

// Cost model of the balanced plan, in tokens: every token, plus a fixed
// charge per lane for what a CTA spends at the end of each lane segment
// (merge, partial write, completion count and combine), measured at about
// four and a half 32-token stages on B200.
#ifdef KK_PLAN_SEGMENT_COST
constexpr std::uint64_t kPlanSegmentCost = KK_PLAN_SEGMENT_COST;
#else
constexpr std::uint64_t kPlanSegmentCost = 144;
#endif

// Kernel choice for kk_paged_decode_attention (KK_ATTN_*), process-wide.
std::atomic<int> g_attention_variant{KK_ATTN_AUTO};

// Scratch of kk_paged_decode_attention_noalloc: the per-lane completion
// counters and partial softmax states live in this fixed device array (one
// per device, created with the module) instead of in caller memory.
static __device__ __align__(256) unsigned char g_attn_scratch[KK_ATTN_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_attn_scratch on the device that owns `stream`, looked
// up once per device (the first call on a device does the lookup, with that
// device made current for it).
int scratchAddress(cudaStream_t stream, void** out)
{
    int current = 0;
    cudaError_t e = cudaGetDevice(&current);
    int device = current;
    if (e == cudaSuccess && stream != nullptr) {
        e = cudaStreamGetDevice(stream, &device);
    }
    if (e != cudaSuccess) {
        return static_cast<int>(e);
    }
    if (device < 0 || device >= kMaxDevices) {
        return KK_EINVAL;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (g_scratch_address[device] == nullptr) {
        if (device != current && (e = cudaSetDevice(device)) != cudaSuccess) {
            return static_cast<int>(e);
        }
        void* address = nullptr;
        e = cudaGetSymbolAddress(&address, g_attn_scratch);
        if (device != current) {
            cudaSetDevice(current);
        }
        if (e != cudaSuccess) {
            return static_cast<int>(e);
        }
        g_scratch_address[device] = address;
    }
    *out = g_scratch_address[device];
    return 0;
}

} // namespace

namespace {

constexpr int kHeadDim = 64;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMicroTokens = 8;
constexpr int kExtentTokens = 64;

struct AttnArgs {
    __half const* micro;
    __half const* extent;
    std::uint64_t micro_page;        // elements per micro page
    std::uint64_t extent_page;
    std::uint32_t micro_slots;       // pool capacities (pages), for bounds checks
    std::uint32_t extent_slots;
    std::uint32_t micro_cap;         // tokens per micro page
    std::uint32_t layer;
    std::uint32_t kv_heads;
    std::uint32_t group;             // query heads per KV head
    std::uint32_t q_heads;
    kk_page_desc const* descs;
    kk_attn_lane const* lanes;
    kk_attn_item const* items;
    std::uint32_t num_items;
    std::uint32_t const* num_items_dev;  // when set, the item count is read from here
    __half const* query;
    std::uint32_t query_stride;
    __half* output;
    std::uint32_t output_stride;
    float scale_log2;                // softmax scale * log2(e)
    std::uint32_t* counters;         // [lanes] completion counters
    float* part_o;                   // [items][q_heads][64]
    float* part_ml;                  // [items][q_heads][2]
    unsigned int* status;            // error word of this launch (never null in the kernel)
};

__device__ __forceinline__ void mma16816(float (&d)[4], std::uint32_t a0, std::uint32_t a1,
    std::uint32_t a2, std::uint32_t a3, std::uint32_t b0, std::uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ std::uint32_t transpose8x8(std::uint32_t x)
{
    std::uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ std::uint32_t pack_half2(float lo, float hi)
{
    __half2 const h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<std::uint32_t const*>(&h);
}

// Position inside an item: descriptor index + 8-token group within it.
struct Cursor {
    std::uint32_t entry;
    std::uint32_t group;
};

__device__ __forceinline__ std::uint32_t groups_of(kk_page_desc const& d)
{
    return (static_cast<std::uint32_t>(d.valid_tokens) + 7u) / 8u;
}

__device__ __forceinline__ void advance(Cursor& c, std::uint32_t n, kk_page_desc const* descs,
    std::uint32_t end)
{
    while (n != 0 && c.entry < end) {
        std::uint32_t const left = groups_of(descs[c.entry]) - c.group;
        if (n < left) {
            c.group += n;
            return;
        }
        n -= left;
        ++c.entry;
        c.group = 0;
    }
}

// The 16-byte K and V chunks one thread streams for one 8-token group.
struct GroupRegs {
    uint4 k[2];
    uint4 v[2];
    std::uint32_t count;  // valid tokens in the group (0 = no group)
};

__device__ __forceinline__ void load_group(GroupRegs& g, AttnArgs const& a, Cursor c,
    std::uint32_t end, std::uint32_t head, std::uint32_t quad, std::uint32_t lane4)
{
    g.count = 0;
    g.k[0] = g.k[1] = g.v[0] = g.v[1] = make_uint4(0, 0, 0, 0);
    if (c.entry >= end) {
        return;
    }
    kk_page_desc const d = a.descs[c.entry];
    bool const micro = d.kind == 0;
    std::uint32_t const cap = micro ? a.micro_cap : kExtentTokens;
    if ((micro ? d.slot >= a.micro_slots : d.slot >= a.extent_slots)
        || d.valid_tokens > cap) {
        atomicCAS(a.status, kErrNone, kErrBadDescriptor);
        return;
    }
    std::uint32_t const first = c.group * 8u;
    std::uint32_t const left = d.valid_tokens - first;
    g.count = left < 8u ? left : 8u;
    if (quad >= g.count) {
        return;  // this quad's token is past the end of the page: stays zero
    }
    std::uint64_t const row = static_cast<std::uint64_t>(a.kv_heads) * kHeadDim;
    __half const* page = micro ? a.micro + static_cast<std::uint64_t>(d.slot) * a.micro_page
                               : a.extent + static_cast<std::uint64_t>(d.slot) * a.extent_page;
    __half const* kblock = page + static_cast<std::uint64_t>(a.layer) * 2u * cap * row;
    std::uint64_t const offset = (first + quad) * row + head * kHeadDim + lane4 * 16u;
    __half const* kp = kblock + offset;
    __half const* vp = kblock + cap * row + offset;
    g.k[0] = ld_stream_v4(kp);
    g.k[1] = ld_stream_v4(kp + 8);
    g.v[0] = ld_stream_v4(vp);
    g.v[1] = ld_stream_v4(vp + 8);
}

__device__ __forceinline__ std::uint32_t word(uint4 const (&w)[2], int i)
{
    uint4 const& v = w[i >> 2];
    switch (i & 3) {
    case 0: return v.x;
    case 1: return v.y;
    case 2: return v.z;
    default: return v.w;
    }
}

__global__ void __launch_bounds__(kThreads, 1) paged_decode_attention_kernel(AttnArgs a)
{
    pdl_launch_dependents();  // dependents only prefetch weights before their own wait
    pdl_wait();
    __shared__ float s_m[kWarps][16];
    __shared__ float s_l[kWarps][16];
    __shared__ float s_o[kWarps][16][kHeadDim + 4];  // +4: fewer bank conflicts
    __shared__ int s_last;

    std::uint32_t const warp = threadIdx.x / 32;
    std::uint32_t const lane = threadIdx.x % 32;
    std::uint32_t const quad = lane >> 2;
    std::uint32_t const c4 = lane & 3;
    std::uint32_t const warps_per_head = kWarps / a.kv_heads;
    std::uint32_t const head = warp / warps_per_head;
    std::uint32_t const sub = warp % warps_per_head;
    std::uint32_t const G = a.group;
    float const kNegInf = -INFINITY;

    std::uint32_t const num_items = a.num_items_dev != nullptr
        ? (*a.num_items_dev < a.num_items ? *a.num_items_dev : a.num_items) : a.num_items;
    for (std::uint32_t it = blockIdx.x; it < num_items; it += gridDim.x) {
        kk_attn_item const item = a.items[it];
        if (item.reserved & KK_ATTN_ITEM_MULTI_LANE) {
            // Items that may span lanes are served by the TMA kernel only.
            if (threadIdx.x == 0) {
                atomicCAS(a.status, kErrNone, kErrBadArgument);
            }
            continue;
        }
        kk_attn_lane const ln = a.lanes[item.lane];

        // Q rows quad and quad+8 of this head's GQA group, dims 16*c4 .. +15.
        uint4 qa[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        uint4 qb[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
        __half const* qrow = a.query + static_cast<std::uint64_t>(ln.query_row) * a.query_stride
            + static_cast<std::uint64_t>(head * G) * kHeadDim + c4 * 16u;
        if (quad < G) {
            qa[0] = *reinterpret_cast<uint4 const*>(qrow + quad * kHeadDim);
            qa[1] = *reinterpret_cast<uint4 const*>(qrow + quad * kHeadDim + 8);
        }
        if (quad + 8 < G) {
            qb[0] = *reinterpret_cast<uint4 const*>(qrow + (quad + 8) * kHeadDim);
            qb[1] = *reinterpret_cast<uint4 const*>(qrow + (quad + 8) * kHeadDim + 8);
        }

        float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
        float o[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        }

        Cursor cur{item.desc_begin, 0};
        advance(cur, 2 * sub, a.descs, item.desc_end);
        GroupRegs ga, gb;
        load_group(ga, a, cur, item.desc_end, head, quad, c4);
        {
            Cursor nb = cur;
            advance(nb, 1, a.descs, item.desc_end);
            load_group(gb, a, nb, item.desc_end, head, quad, c4);
        }
        while (ga.count != 0) {
            // Prefetch the next pair of groups of this warp.
            Cursor next = cur;
            advance(next, 2 * warps_per_head, a.descs, item.desc_end);
            GroupRegs na, nb;
            load_group(na, a, next, item.desc_end, head, quad, c4);
            {
                Cursor n2 = next;
                advance(n2, 1, a.descs, item.desc_end);
                load_group(nb, a, n2, item.desc_end, head, quad, c4);
            }

            // S = Q K^T for the two 8-token tiles.
            float s0[4] = {0.f, 0.f, 0.f, 0.f};
            float s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                std::uint32_t const a0 = word(qa, 2 * j), a2 = word(qa, 2 * j + 1);
                std::uint32_t const a1 = word(qb, 2 * j), a3 = word(qb, 2 * j + 1);
                mma16816(s0, a0, a1, a2, a3, word(ga.k, 2 * j), word(ga.k, 2 * j + 1));
                mma16816(s1, a0, a1, a2, a3, word(gb.k, 2 * j), word(gb.k, 2 * j + 1));
            }
            bool const v00 = 2 * c4 < ga.count, v01 = 2 * c4 + 1 < ga.count;
            bool const v10 = 2 * c4 < gb.count, v11 = 2 * c4 + 1 < gb.count;
            float x[2][4];
            x[0][0] = v00 ? s0[0] * a.scale_log2 : kNegInf;
            x[0][1] = v01 ? s0[1] * a.scale_log2 : kNegInf;
            x[0][2] = v10 ? s1[0] * a.scale_log2 : kNegInf;
            x[0][3] = v11 ? s1[1] * a.scale_log2 : kNegInf;
            x[1][0] = v00 ? s0[2] * a.scale_log2 : kNegInf;
            x[1][1] = v01 ? s0[3] * a.scale_log2 : kNegInf;
            x[1][2] = v10 ? s1[2] * a.scale_log2 : kNegInf;
            x[1][3] = v11 ? s1[3] * a.scale_log2 : kNegInf;

            float p[2][4];
            float alpha[2];
            float* mrow[2] = {&m0, &m1};
            float* lrow[2] = {&l0, &l1};
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float mx = fmaxf(fmaxf(x[r][0], x[r][1]), fmaxf(x[r][2], x[r][3]));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
                float const m_new = fmaxf(*mrow[r], mx);
                float const m_use = m_new == kNegInf ? 0.f : m_new;
                alpha[r] = exp2f(*mrow[r] - m_use);
                float sum = 0.f;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    p[r][t] = exp2f(x[r][t] - m_use);
                    sum += p[r][t];
                }
                *lrow[r] = *lrow[r] * alpha[r] + sum;
                *mrow[r] = m_new;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                o[j][0] *= alpha[0];
                o[j][1] *= alpha[0];
                o[j][2] *= alpha[1];
                o[j][3] *= alpha[1];
            }
            std::uint32_t const pa0 = pack_half2(p[0][0], p[0][1]);
            std::uint32_t const pa1 = pack_half2(p[1][0], p[1][1]);
            std::uint32_t const pa2 = pack_half2(p[0][2], p[0][3]);
            std::uint32_t const pa3 = pack_half2(p[1][2], p[1][3]);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                std::uint32_t const b0 = transpose8x8(word(ga.v, j));
                std::uint32_t const b1 = transpose8x8(word(gb.v, j));
                mma16816(o[j], pa0, pa1, pa2, pa3, b0, b1);
            }

            ga = na;
            gb = nb;
            cur = next;
        }
        l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
        l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
        l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

        // Per-warp state -> shared memory (row quad, and quad+8 when G > 8).
        if (c4 == 0) {
            s_m[warp][quad] = m0;
            s_l[warp][quad] = l0;
            s_m[warp][quad + 8] = m1;
            s_l[warp][quad + 8] = l1;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            s_o[warp][quad][c4 * 16 + 2 * j] = o[j][0];
            s_o[warp][quad][c4 * 16 + 2 * j + 1] = o[j][1];
            s_o[warp][quad + 8][c4 * 16 + 2 * j] = o[j][2];
            s_o[warp][quad + 8][c4 * 16 + 2 * j + 1] = o[j][3];
        }
        __syncthreads();

        // Merge the warps of each head: thread -> (query head, 8 dims).
        bool const split = ln.item_count > 1;
        for (std::uint32_t idx = threadIdx.x; idx < a.q_heads * 8u; idx += kThreads) {
            std::uint32_t const qh = idx / 8u;
            std::uint32_t const d0 = (idx % 8u) * 8u;
            std::uint32_t const h = qh / G;
            std::uint32_t const g = qh % G;
            float M = kNegInf;
            for (std::uint32_t s = 0; s < warps_per_head; ++s) {
                M = fmaxf(M, s_m[h * warps_per_head + s][g]);
            }
            float const m_use = M == kNegInf ? 0.f : M;
            float L = 0.f;
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (std::uint32_t s = 0; s < warps_per_head; ++s) {
                std::uint32_t const w = h * warps_per_head + s;
                float const f = exp2f(s_m[w][g] - m_use);
                L += s_l[w][g] * f;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    acc[e] += s_o[w][g][d0 + e] * f;
                }
            }
            if (!split) {
                __half* out = a.output + static_cast<std::uint64_t>(ln.query_row) * a.output_stride
                    + qh * kHeadDim + d0;
                float const inv = 1.f / L;
                __align__(16) __half vals[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    vals[e] = __float2half_rn(acc[e] * inv);
                }
                *reinterpret_cast<uint4*>(out) = *reinterpret_cast<uint4 const*>(vals);
            } else {
                float* po = a.part_o + (static_cast<std::uint64_t>(it) * a.q_heads + qh) * kHeadDim
                    + d0;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    po[e] = acc[e];
                }
                if (d0 == 0) {
                    float* pml = a.part_ml + (static_cast<std::uint64_t>(it) * a.q_heads + qh) * 2;
                    pml[0] = M;
                    pml[1] = L;
                }
            }
        }
        if (split) {
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                std::uint32_t const done = atomicAdd(&a.counters[item.lane], 1u);
                s_last = done + 1 == ln.item_count;
            }
            __syncthreads();
            if (s_last) {
                __threadfence();
                for (std::uint32_t idx = threadIdx.x; idx < a.q_heads * 8u; idx += kThreads) {
                    std::uint32_t const qh = idx / 8u;
                    std::uint32_t const d0 = (idx % 8u) * 8u;
                    float M = kNegInf;
                    for (std::uint32_t i = 0; i < ln.item_count; ++i) {
                        std::uint64_t const row = (ln.item_offset + i) * static_cast<std::uint64_t>(a.q_heads) + qh;
                        M = fmaxf(M, __ldcg(a.part_ml + row * 2));
                    }
                    float const m_use = M == kNegInf ? 0.f : M;
                    float L = 0.f;
                    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    for (std::uint32_t i = 0; i < ln.item_count; ++i) {
                        std::uint64_t const row = (ln.item_offset + i) * static_cast<std::uint64_t>(a.q_heads) + qh;
                        float const f = exp2f(__ldcg(a.part_ml + row * 2) - m_use);
                        L += __ldcg(a.part_ml + row * 2 + 1) * f;
                        float const* po = a.part_o + row * kHeadDim + d0;
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            acc[e] += __ldcg(po + e) * f;
                        }
                    }
                    __half* out = a.output + static_cast<std::uint64_t>(ln.query_row) * a.output_stride
                        + qh * kHeadDim + d0;
                    float const inv = 1.f / L;
                    __align__(16) __half vals[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        vals[e] = __float2half_rn(acc[e] * inv);
                    }
                    *reinterpret_cast<uint4*>(out) = *reinterpret_cast<uint4 const*>(vals);
                }
                if (threadIdx.x == 0) {
                    a.counters[item.lane] = 0;  // ready for the next launch
                }
            }
        }
        __syncthreads();
    }
}

constexpr std::uint64_t align256(std::uint64_t x) { return (x + 255u) & ~std::uint64_t(255); }

int g_num_sms = 0;

int numSms()
{
    if (g_num_sms == 0) {
        int device = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, device);
        if (g_num_sms <= 0) {
            g_num_sms = 148;
        }
    }
    return g_num_sms;
}

} // namespace
} // namespace kk

namespace {
// Argument checks of kk_paged_decode_attention other than the workspace:
// nothing is launched (and nothing is written to the device) when they fail.
bool attentionShapeValid(const kk_kv_pools* pools, uint32_t layer, uint32_t q_heads,
    const kk_page_desc* descs, const kk_attn_lane* lanes, const kk_attn_item* items,
    const uint16_t* query, uint32_t query_stride, const uint16_t* output, uint32_t output_stride,
    float scale)
{
    using namespace kk;
    return !(pools == nullptr || pools->head_dim != kHeadDim || layer >= pools->layers
        || (pools->kv_heads != 1 && pools->kv_heads != 2 && pools->kv_heads != 4
            && pools->kv_heads != 8)
        || q_heads % pools->kv_heads != 0 || q_heads / pools->kv_heads > 16
        || q_heads / pools->kv_heads == 0 || !(scale > 0.f) || query == nullptr
        || output == nullptr || descs == nullptr || lanes == nullptr || items == nullptr
        || query_stride % 8 != 0 || output_stride % 8 != 0 || !microPageTokensValid(*pools));
}

// attentionShapeValid plus the workspace: the completion counters and
// partial states are only touched when some lane is split over several
// items; partial states are read and written as float2/float4.
bool attentionArgsValid(const kk_kv_pools* pools, uint32_t layer, uint32_t q_heads,
    const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, const uint16_t* query, uint32_t query_stride,
    const uint16_t* output, uint32_t output_stride, float scale, const void* workspace,
    uint64_t workspace_bytes)
{
    using kk::kHeadDim;
    if (!attentionShapeValid(pools, layer, q_heads, descs, lanes, items, query, query_stride, output,
            output_stride, scale)) {
        return false;
    }
    if (num_items > num_lanes
        && (workspace == nullptr
            || workspace_bytes < kk_attention_workspace_bytes(num_lanes, num_items, q_heads, kHeadDim))) {
        return false;
    }
    return reinterpret_cast<std::uintptr_t>(workspace) % 16u == 0;
}

int launchAttention(const kk_kv_pools* pools, uint32_t layer, uint32_t q_heads,
    const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, std::uint32_t const* num_items_dev,
    const uint16_t* query, uint32_t query_stride,
    uint16_t* output, uint32_t output_stride, float scale, void* workspace,
    uint64_t workspace_bytes, int variant, unsigned int* status, cudaStream_t stream)
{
    using namespace kk;
    if (!attentionArgsValid(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items, query,
            query_stride, output, output_stride, scale, workspace, workspace_bytes)) {
        return KK_EINVAL;
    }
    if (num_items == 0) {
        return 0;
    }
    AttnArgs a{};
    a.micro = static_cast<__half const*>(pools->micro);
    a.extent = static_cast<__half const*>(pools->extent);
    std::uint64_t const row = std::uint64_t(pools->kv_heads) * kHeadDim;
    a.micro_cap = microPageTokens(*pools);
    a.micro_page = std::uint64_t(pools->layers) * 2u * a.micro_cap * row;
    a.extent_page = std::uint64_t(pools->layers) * 2u * kExtentTokens * row;
    a.micro_slots = pools->micro == nullptr ? 0 : pools->micro_capacity;
    a.extent_slots = pools->extent == nullptr ? 0 : pools->extent_capacity;
    a.layer = layer;
    a.kv_heads = pools->kv_heads;
    a.group = q_heads / pools->kv_heads;
    a.q_heads = q_heads;
    a.descs = descs;
    a.lanes = lanes;
    a.items = items;
    a.num_items = num_items;
    a.num_items_dev = num_items_dev;
    a.query = reinterpret_cast<__half const*>(query);
    a.query_stride = query_stride;
    a.output = reinterpret_cast<__half*>(output);
    a.output_stride = output_stride;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.status = status;
    if (a.status == nullptr) {
        cudaError_t const e = cudaGetSymbolAddress(reinterpret_cast<void**>(&a.status), g_attn_status);
        if (e != cudaSuccess) {
            return static_cast<int>(e);
        }
    }
    // Without a workspace the kernels see null partial pointers: a lane that
    // turns out to be split is then reported (bad argument), never written.
    if (workspace != nullptr) {
        char* ws = static_cast<char*>(workspace);
        a.counters = reinterpret_cast<std::uint32_t*>(ws);
        ws += align256(std::uint64_t(num_lanes) * 4u);
        a.part_o = reinterpret_cast<float*>(ws);
        ws += align256(2ull * num_items * q_heads * kHeadDim * 4u);
        a.part_ml = reinterpret_cast<float*>(ws);
    }
    // The TMA kernel copies each query row with one bulk copy (16-byte aligned source).
    bool const tma_ok = attentionTmaSupported(pools, q_heads)
        && reinterpret_cast<std::uintptr_t>(query) % 16u == 0;
    if (variant == KK_ATTN_TMA && !tma_ok) {
        return KK_EINVAL;
    }
    if (tma_ok && variant != KK_ATTN_DIRECT) {
        return attentionTmaLaunch(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items,
            num_items_dev, query, query_stride, output, output_stride, scale, a.counters, a.part_o,
            a.part_ml, status, stream);
    }
    unsigned const grid = num_items < unsigned(numSms()) ? num_items : unsigned(numSms());
    return static_cast<int>(launch(paged_decode_attention_kernel, dim3(grid), dim3(kThreads), 0,
        stream, 1, a));
}

} // namespace

extern "C" {

uint32_t kk_attention_plan(const kk_page_desc* descs, kk_attn_lane* lanes, uint32_t num_lanes,
    uint32_t target_tokens, kk_attn_item* items, uint32_t max_items)
{
    if (target_tokens == 0) {
        target_tokens = 256;
    }
    std::uint32_t count = 0;
    for (std::uint32_t b = 0; b < num_lanes; ++b) {
        kk_attn_lane& ln = lanes[b];
        ln.item_offset = count;
        ln.item_count = 0;
        ln.first_item_shared = 0;
        std::uint32_t begin = ln.desc_offset;
        std::uint32_t tokens = 0;
        std::uint32_t const end = ln.desc_offset + ln.desc_count;
        for (std::uint32_t e = ln.desc_offset; e < end; ++e) {
            tokens += descs[e].valid_tokens;
            bool const last = e + 1 == end;
            if (tokens >= target_tokens || last) {
                if (count < max_items) {
                    items[count] = kk_attn_item{b, begin, e + 1, 0};
                }
                ++count;
                ++ln.item_count;
                begin = e + 1;
                tokens = 0;
            }
        }
    }
    return count;
}

uint32_t kk_attention_plan_balanced(const kk_page_desc* descs, kk_attn_lane* lanes,
    uint32_t num_lanes, uint32_t num_parts, kk_attn_item* items, uint32_t max_items)
{
    if (num_parts == 0) {
        num_parts = 1;
    }
    constexpr std::uint64_t kSegmentCost = kk::kPlanSegmentCost;
    // A page occupies whole 8-token groups of a stage whatever its valid
    // count, so it costs its valid tokens rounded up to a group.
    auto cost = [](kk_page_desc const& d) -> std::uint64_t { return (d.valid_tokens + 7u) & ~7u; };
    std::uint64_t total = 0;
    for (std::uint32_t b = 0; b < num_lanes; ++b) {
        if (lanes[b].desc_count != 0) {
            total += kSegmentCost;
        }
        for (std::uint32_t e = lanes[b].desc_offset; e < lanes[b].desc_offset + lanes[b].desc_count; ++e) {
            total += cost(descs[e]);
        }
    }
    // Cut k of num_parts - 1 lands on the unit boundary nearest to
    // k * total / num_parts, where a unit is a page, or half of a full
    // 64-token extent page (a stage's worth: the two halves stream as two
    // stages), so the runs are equal to within a quarter of an extent.
    std::uint64_t const whole = total / num_parts;
    std::uint64_t const rest = total % num_parts;
    auto target = [&](std::uint64_t k) { return whole * k + rest * k / num_parts; };
    std::uint32_t count = 0;
    kk_attn_item cur{};
    bool open = false;
    std::uint64_t pos = 0;
    std::uint32_t next_cut = 1;
    // Position of the next cut, recomputed only when a cut is placed (the
    // division stays out of the per-descriptor loop).
    std::uint64_t next_target = num_parts > 1 ? target(1) : ~std::uint64_t{0};
    auto flush = [&]() {
        if (open && count - 1 < max_items) {
            items[count - 1] = cur;
        }
        open = false;
    };
    for (std::uint32_t b = 0; b < num_lanes; ++b) {
        kk_attn_lane& ln = lanes[b];
        ln.item_offset = count;
        ln.item_count = 0;
        ln.first_item_shared = 0;
        std::uint32_t const end = ln.desc_offset + ln.desc_count;
        // An item only continues into this lane when the descriptors are contiguous.
        if (open && cur.desc_end != ln.desc_offset) {
            flush();
        }
        if (ln.desc_count != 0) {
            pos += kSegmentCost;
        }
        for (std::uint32_t e = ln.desc_offset; e < end; ++e) {
            bool const halves = descs[e].kind == 1u && descs[e].valid_tokens == 64u;  // a full extent
            std::uint32_t const units = halves ? 2u : 1u;
            std::uint64_t const c = halves ? KK_ATTN_EXTENT_HALF : cost(descs[e]);
            for (std::uint32_t h = 0; h < units; ++h) {
                bool cut_before = false;
                bool cut_after = false;
                while (next_cut < num_parts && next_target < pos + c) {
                    if (2 * next_target < 2 * pos + c) {
                        cut_before = true;
                    } else {
                        cut_after = true;
                    }
                    ++next_cut;
                    next_target = next_cut < num_parts ? target(next_cut) : ~std::uint64_t{0};
                }
                if (cut_before && open) {
                    if (h == 1u) {
                        cur.reserved |= KK_ATTN_EXTENT_HALF << 16;  // ends after the first half
                    }
                    flush();
                }
                if (!open) {
                    cur = kk_attn_item{b, e, e, KK_ATTN_ITEM_MULTI_LANE | (h == 1u ? KK_ATTN_EXTENT_HALF << 8 : 0u)};
                    open = true;
                    ++count;
                }
                if (ln.item_count == 0 || ln.item_offset + ln.item_count != count) {
                    if (ln.item_count == 0) {
                        ln.item_offset = count - 1;
                        ln.first_item_shared = cur.lane != b ? 1u : 0u;
                    }
                    ++ln.item_count;
                }
                cur.desc_end = e + 1;
                pos += c;
                if (cut_after) {
                    if (h + 1u < units) {
                        cur.reserved |= KK_ATTN_EXTENT_HALF << 16;
                    }
                    flush();
                }
            }
        }
    }
    flush();
    return count;
}

uint64_t kk_attention_workspace_bytes(uint32_t num_lanes, uint32_t num_items, uint32_t q_heads,
    uint32_t head_dim)
{
    using kk::align256;
    // Two partial slots per item: an item of kk_attention_plan_balanced may
    // split both its first and its last lane.
    return align256(std::uint64_t(num_lanes) * 4u)
        + align256(2ull * num_items * q_heads * head_dim * 4u)
        + align256(2ull * num_items * q_heads * 2u * 4u);
}

int kk_attention_workspace_init(void* workspace, uint32_t num_lanes, void* stream)
{
    return static_cast<int>(cudaMemsetAsync(workspace, 0, kk::align256(std::uint64_t(num_lanes) * 4u),
        static_cast<cudaStream_t>(stream)));
}

int kk_paged_decode_attention(const kk_kv_pools* pools, uint32_t layer, uint32_t q_heads,
    const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, const uint16_t* query, uint32_t query_stride,
    uint16_t* output, uint32_t output_stride, float scale, void* workspace,
    uint64_t workspace_bytes, void* stream)
{
    return launchAttention(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items,
        nullptr, query, query_stride, output, output_stride, scale, workspace, workspace_bytes,
        kk::g_attention_variant.load(std::memory_order_relaxed), nullptr,
        static_cast<cudaStream_t>(stream));
}

int kk_paged_decode_attention_noalloc(const kk_kv_pools* pools, uint32_t layer, uint32_t q_heads,
    const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, const uint16_t* query, uint32_t query_stride,
    uint16_t* output, uint32_t output_stride, float scale, void* stream)
{
    std::uint64_t const need = kk_attention_workspace_bytes(num_lanes, num_items, q_heads, 64);
    if (need > KK_ATTN_SCRATCH_BYTES) {
        return KK_ENOSCRATCH;
    }
    // Arguments first: a rejected call writes nothing to the device.
    if (!attentionShapeValid(pools, layer, q_heads, descs, lanes, items, query, query_stride, output,
            output_stride, scale)) {
        return KK_EINVAL;
    }
    if (num_items == 0) {
        return 0;
    }
    void* scratch = nullptr;
    int const rc = kk::scratchAddress(static_cast<cudaStream_t>(stream), &scratch);
    if (rc != 0) {
        return rc;
    }
    // The completion counters must be zero when the kernel starts.
    cudaError_t const e = cudaMemsetAsync(scratch, 0, kk::align256(std::uint64_t(num_lanes) * 4u),
        static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        return static_cast<int>(e);
    }
    return launchAttention(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items,
        nullptr, query, query_stride, output, output_stride, scale, scratch, KK_ATTN_SCRATCH_BYTES,
        kk::g_attention_variant.load(std::memory_order_relaxed), nullptr,
        static_cast<cudaStream_t>(stream));
}

int kk_attention_set_variant(int variant)
{
    if (variant < KK_ATTN_AUTO || variant > KK_ATTN_TMA) {
        return KK_EINVAL;
    }
    kk::g_attention_variant.store(variant, std::memory_order_relaxed);
    return 0;
}

} // extern "C"

namespace kk {
int attentionStatus(cudaStream_t stream) { return readStatus(&g_attn_status, stream); }

int attentionDevCount(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t const* num_items, std::uint32_t max_items,
    std::uint16_t const* query, std::uint32_t query_stride, std::uint16_t* output,
    std::uint32_t output_stride, float scale, void* workspace, std::uint64_t workspace_bytes,
    unsigned int* status, cudaStream_t stream)
{
    if (num_items == nullptr || status == nullptr) {
        return KK_EINVAL;
    }
    // The runner plans with kk_attention_plan_balanced wherever the TMA kernel
    // serves the shape, so the kernel choice here does not follow the
    // process-wide variant switch.
    int const variant = attentionTmaSupported(pools, q_heads) ? KK_ATTN_TMA : KK_ATTN_DIRECT;
    return launchAttention(pools, layer, q_heads, descs, lanes, num_lanes, items, max_items,
        num_items, query, query_stride, output, output_stride, scale, workspace, workspace_bytes,
        variant, status, stream);
}

int attentionLaunchTma(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint16_t const* query,
    std::uint32_t query_stride, std::uint16_t* output, std::uint32_t output_stride, float scale,
    void* workspace, std::uint64_t workspace_bytes, unsigned int* status, cudaStream_t stream)
{
    return launchAttention(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items, nullptr,
        query, query_stride, output, output_stride, scale, workspace, workspace_bytes, KK_ATTN_TMA, status,
        stream);
}

std::uint32_t attentionPlanParts(kk_attn_lane const* lanes, std::uint32_t num_lanes, std::uint32_t sm_count)
{
    std::uint64_t cost = 0;
    for (std::uint32_t b = 0; b < num_lanes; ++b) {
        if (lanes[b].desc_count != 0) {
            cost += lanes[b].token_count + kPlanSegmentCost;
        }
    }
    std::uint64_t const parts = cost / kAttnMinPartCost;
    return parts < 1 ? 1u : parts > sm_count ? sm_count : static_cast<std::uint32_t>(parts);
}

int attentionLaunch(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint16_t const* query,
    std::uint32_t query_stride, std::uint16_t* output, std::uint32_t output_stride, float scale,
    void* workspace, std::uint64_t workspace_bytes, unsigned int* status, cudaStream_t stream)
{
    return launchAttention(pools, layer, q_heads, descs, lanes, num_lanes, items, num_items, nullptr,
        query, query_stride, output, output_stride, scale, workspace, workspace_bytes,
        g_attention_variant.load(std::memory_order_relaxed), status, stream);
}
} // namespace kk
