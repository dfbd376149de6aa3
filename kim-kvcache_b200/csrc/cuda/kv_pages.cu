// K2 — batched KV append and copy-on-write over the page pools.
//
// kk_kv_write: one launch writes the new token's K and V of a range of layers
// for every lane (the reference issues one tiny launch per lane per layer,
// src/cuda/engine/transaction.cpp:195-204). One warp moves one (lane, layer,
// K|V) row of kv_heads*head_dim FP16 values with 16-byte accesses.
// kk_kv_copy_tokens: partial-tail copy-on-write of the first `tokens` tokens
// of a page into a fresh page, for a range of layers (reference
// copyLayerTokensKernel / copyPageTokensKernel, paged_decode_kernels.cu:29-63,
// page_kernels.cu:46-75). Both are bandwidth-bound byte movers.
#include "../../../include/kk_kernels.h"
#include "kernels_internal.h"
#include "launch.cuh"

namespace kk {

__device__ unsigned int g_pages_status;

namespace {

struct PoolView {
    __half* micro;
    __half* extent;
    std::uint64_t micro_page;
    std::uint64_t extent_page;
    std::uint32_t micro_slots;
    std::uint32_t extent_slots;
    std::uint32_t row;         // kv_heads * head_dim elements per token per K|V
    std::uint32_t layers;
    std::uint32_t micro_cap;   // tokens per micro page
    unsigned int* status;      // error word of the launch (null: the module's word)
};

__device__ __forceinline__ void report(PoolView const& v, unsigned int code)
{
    atomicCAS(v.status != nullptr ? v.status : &g_pages_status, kErrNone, code);
}

PoolView view(kk_kv_pools const& p)
{
    PoolView v{};
    v.micro = static_cast<__half*>(p.micro);
    v.extent = static_cast<__half*>(p.extent);
    v.row = p.kv_heads * p.head_dim;
    v.micro_cap = microPageTokens(p);
    v.micro_page = std::uint64_t(p.layers) * 2u * v.micro_cap * v.row;
    v.extent_page = std::uint64_t(p.layers) * 2u * 64u * v.row;
    v.micro_slots = p.micro == nullptr ? 0 : p.micro_capacity;
    v.extent_slots = p.extent == nullptr ? 0 : p.extent_capacity;
    v.layers = p.layers;
    return v;
}

// Start of the (layer, component) block of a page; nullptr if out of bounds.
__device__ __forceinline__ __half* block_of(PoolView const& v, std::uint32_t kind,
    std::uint32_t slot, std::uint32_t layer, std::uint32_t component)
{
    bool const micro = kind == 0;
    if (micro ? slot >= v.micro_slots : slot >= v.extent_slots) {
        report(v, kErrBadDescriptor);
        return nullptr;
    }
    std::uint32_t const cap = micro ? v.micro_cap : 64u;
    __half* page = micro ? v.micro + std::uint64_t(slot) * v.micro_page
                         : v.extent + std::uint64_t(slot) * v.extent_page;
    return page + (std::uint64_t(layer) * 2u + component) * cap * v.row;
}

// grid: (num_lanes, layer_count, 2); one warp per row, 8 elements per thread step.
__global__ void kv_write_kernel(PoolView v, std::uint32_t layer_begin, kk_kv_slot const* slots,
    __half const* key, __half const* value, std::uint64_t lane_stride, std::uint64_t layer_stride)
{
    pdl_wait();
    std::uint32_t const lane_idx = blockIdx.x;
    std::uint32_t const layer_off = blockIdx.y;
    std::uint32_t const component = blockIdx.z;
    kk_kv_slot const s = slots[lane_idx];
    if (!s.active) {
        return;
    }
    std::uint32_t const cap = s.kind == 0 ? v.micro_cap : 64u;
    if (s.page_token >= cap) {
        report(v, kErrBadDescriptor);
        return;
    }
    __half* dst = block_of(v, s.kind, s.slot, layer_begin + layer_off, component);
    if (dst == nullptr) {
        return;
    }
    dst += std::uint64_t(s.page_token) * v.row;
    __half const* src = (component == 0 ? key : value) + lane_idx * lane_stride
        + layer_off * layer_stride;
    for (std::uint32_t i = threadIdx.x * 8u; i < v.row; i += blockDim.x * 8u) {
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<uint4 const*>(src + i);
    }
}

// grid: (num_copies, layer_count, 2): copies tokens*row contiguous elements.
__global__ void kv_copy_kernel(PoolView v, std::uint32_t layer_begin, kk_kv_copy const* copies,
    std::uint32_t const* count)
{
    pdl_wait();
    if (count != nullptr && blockIdx.x >= *count) {
        return;
    }
    kk_kv_copy const c = copies[blockIdx.x];
    std::uint32_t const layer = layer_begin + blockIdx.y;
    std::uint32_t const component = blockIdx.z;
    std::uint32_t const src_cap = c.src_kind == 0 ? v.micro_cap : 64u;
    std::uint32_t const dst_cap = c.dst_kind == 0 ? v.micro_cap : 64u;
    if (c.tokens > src_cap || c.tokens > dst_cap) {
        report(v, kErrBadDescriptor);
        return;
    }
    __half const* src = block_of(v, c.src_kind, c.src_slot, layer, component);
    __half* dst = block_of(v, c.dst_kind, c.dst_slot, layer, component);
    if (src == nullptr || dst == nullptr) {
        return;
    }
    std::uint64_t const n = std::uint64_t(c.tokens) * v.row;
    for (std::uint64_t i = threadIdx.x * 8u; i < n; i += blockDim.x * 8u) {
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<uint4 const*>(src + i);
    }
}

struct PromoteSlots {
    std::uint32_t micro[8];
};

// grid (8 source pages, layers, 2): 8 tokens x row elements per block.
__global__ void kv_promote_kernel(PoolView v, PromoteSlots src, std::uint32_t extent_slot)
{
    pdl_wait();
    std::uint32_t const k = blockIdx.x;
    std::uint32_t const layer = blockIdx.y;
    std::uint32_t const component = blockIdx.z;
    __half const* from = block_of(v, 0, src.micro[k], layer, component);
    __half* to = block_of(v, 1, extent_slot, layer, component);
    if (from == nullptr || to == nullptr) {
        return;
    }
    to += std::uint64_t(8u * k) * v.row;
    std::uint64_t const n = 8ull * v.row;
    for (std::uint64_t i = threadIdx.x * 8u; i < n; i += blockDim.x * 8u) {
        *reinterpret_cast<uint4*>(to + i) = *reinterpret_cast<uint4 const*>(from + i);
    }
}

// K6 gather / scatter between pages and a contiguous KV tensor
// [layer][K|V][token][head][dim] (the reference's gatherKernel and
// appendTokensKernel, src/cuda/kv/page_kernels.cu:77-127, :184-242, which
// search the descriptor list per element). Here one CTA moves one page's
// (layer, K|V) block: valid_tokens contiguous rows, 16-byte accesses.
// Scatter copies only the tokens of [first, first + count) into the pages.
// grid (descriptors, layers * 2).
__global__ void kv_gather_kernel(PoolView v, kk_page_desc const* descs, std::uint32_t total_tokens,
    __half* out, __half const* in, std::uint32_t first, std::uint32_t count)
{
    pdl_wait();
    kk_page_desc const d = descs[blockIdx.x];
    std::uint32_t const layer = blockIdx.y / 2u;
    std::uint32_t const component = blockIdx.y % 2u;
    bool const micro = d.kind == 0;
    std::uint32_t const cap = micro ? v.micro_cap : 64u;
    std::uint32_t const begin = d.logical_token_begin;
    std::uint32_t const end = begin + d.valid_tokens;
    __half* page = block_of(v, micro ? 0 : 1, d.slot, layer, component);
    bool const bad = page == nullptr || d.valid_tokens > cap || d.kind > 1
        || (in == nullptr ? end > total_tokens : false);
    if (bad) {
        if (threadIdx.x == 0) {
            report(v, kErrBadDescriptor);
        }
        return;
    }
    std::uint64_t const row = v.row;
    if (in == nullptr) {
        __half* dst = out + ((std::uint64_t(layer) * 2u + component) * total_tokens + begin) * row;
        std::uint64_t const n = std::uint64_t(d.valid_tokens) * row;
        for (std::uint64_t i = threadIdx.x * 8u; i < n; i += blockDim.x * 8u) {
            *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<uint4 const*>(page + i);
        }
        return;
    }
    std::uint32_t const lo = begin > first ? begin : first;
    std::uint32_t const hi = end < first + count ? end : first + count;
    if (lo >= hi) {
        return;
    }
    __half const* src = in + ((std::uint64_t(layer) * 2u + component) * count + (lo - first)) * row;
    __half* dst = page + std::uint64_t(lo - begin) * row;
    std::uint64_t const n = std::uint64_t(hi - lo) * row;
    for (std::uint64_t i = threadIdx.x * 8u; i < n; i += blockDim.x * 8u) {
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<uint4 const*>(src + i);
    }
}

// SplitMix64 finaliser: a well-mixed 64-bit hash of (seed, index).
__device__ __forceinline__ std::uint64_t mix64(std::uint64_t x)
{
    x += 0x9e3779b97f4a7c15ull;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
    return x ^ (x >> 31);
}

__global__ void fill_fp16_kernel(__half* data, std::uint64_t count, std::uint64_t seed, float scale)
{
    for (std::uint64_t i = blockIdx.x * std::uint64_t(blockDim.x) + threadIdx.x; i < count;
         i += std::uint64_t(gridDim.x) * blockDim.x) {
        std::uint64_t const h = mix64(seed * 0x100000001b3ull + i);
        float const u = static_cast<float>(h >> 40) * (1.0f / 16777216.0f);  // [0, 1)
        data[i] = __float2half_rn((2.0f * u - 1.0f) * scale);
    }
}

bool poolsOk(kk_kv_pools const* p)
{
    return p != nullptr && p->layers != 0 && p->kv_heads != 0 && p->head_dim != 0
        && (p->kv_heads * p->head_dim) % 8 == 0 && microPageTokensValid(*p);
}

} // namespace
} // namespace kk

extern "C" {

int kk_kv_write(const kk_kv_pools* pools, uint32_t layer_begin, uint32_t layer_count,
    const kk_kv_slot* slots, uint32_t num_lanes, const uint16_t* key, const uint16_t* value,
    uint64_t lane_stride, uint64_t layer_stride, void* stream)
{
    return kk::kvWrite(pools, layer_begin, layer_count, slots, num_lanes, key, value, lane_stride,
        layer_stride, nullptr, static_cast<cudaStream_t>(stream));
}

int kk_kv_copy_tokens(const kk_kv_pools* pools, uint32_t layer_begin, uint32_t layer_count,
    const kk_kv_copy* copies, uint32_t num_copies, void* stream)
{
    return kk::kvCopy(pools, layer_begin, layer_count, copies, num_copies, nullptr,
        static_cast<cudaStream_t>(stream));
}

int kk_kv_promote(const kk_kv_pools* pools, const uint32_t* micro_slots, uint32_t extent_slot,
    void* stream)
{
    using namespace kk;
    if (!poolsOk(pools) || micro_slots == nullptr || pools->extent == nullptr
        || extent_slot >= pools->extent_capacity || microPageTokens(*pools) != 8u) {
        return KK_EINVAL;
    }
    PromoteSlots src{};
    for (int k = 0; k < 8; ++k) {
        if (micro_slots[k] >= pools->micro_capacity) {
            return KK_EINVAL;
        }
        src.micro[k] = micro_slots[k];
    }
    return static_cast<int>(launch(kv_promote_kernel, dim3(8, pools->layers, 2), dim3(128), 0,
        static_cast<cudaStream_t>(stream), 1, view(*pools), src, extent_slot));
}

int kk_kv_gather(const kk_kv_pools* pools, const kk_page_desc* descs, uint32_t num_descs,
    uint32_t total_tokens, uint16_t* out, void* stream)
{
    using namespace kk;
    if (!poolsOk(pools) || (num_descs != 0 && (descs == nullptr || out == nullptr))
        || (reinterpret_cast<std::uintptr_t>(out) & 15u) != 0) {
        return KK_EINVAL;
    }
    if (num_descs == 0) {
        return 0;
    }
    return static_cast<int>(launch(kv_gather_kernel, dim3(num_descs, pools->layers * 2u), dim3(256), 0,
        static_cast<cudaStream_t>(stream), 1, view(*pools), descs, total_tokens,
        reinterpret_cast<__half*>(out), static_cast<__half const*>(nullptr), 0u, 0u));
}

int kk_kv_scatter(const kk_kv_pools* pools, const kk_page_desc* descs, uint32_t num_descs,
    uint32_t first_token, uint32_t token_count, const uint16_t* in, void* stream)
{
    using namespace kk;
    if (!poolsOk(pools) || (num_descs != 0 && (descs == nullptr || in == nullptr))
        || (reinterpret_cast<std::uintptr_t>(in) & 15u) != 0) {
        return KK_EINVAL;
    }
    if (num_descs == 0 || token_count == 0) {
        return 0;
    }
    return static_cast<int>(launch(kv_gather_kernel, dim3(num_descs, pools->layers * 2u), dim3(256), 0,
        static_cast<cudaStream_t>(stream), 1, view(*pools), descs, 0u, static_cast<__half*>(nullptr),
        reinterpret_cast<__half const*>(in), first_token, token_count));
}

int kk_fill_fp16(uint16_t* data, uint64_t count, uint64_t seed, float scale, void* stream)
{
    using namespace kk;
    if (data == nullptr) {
        return KK_EINVAL;
    }
    if (count == 0) {
        return 0;
    }
    std::uint64_t blocks = (count + 255) / 256;
    blocks = blocks > 8192 ? 8192 : blocks;
    return static_cast<int>(launch(fill_fp16_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256),
        0, static_cast<cudaStream_t>(stream), 1, reinterpret_cast<__half*>(data), count, seed, scale));
}

} // extern "C"

namespace kk {
int pagesStatus(cudaStream_t stream) { return readStatus(&g_pages_status, stream); }

int kvCopyDevCount(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_copy const* copies, std::uint32_t const* num_copies, std::uint32_t max_copies,
    unsigned int* status, cudaStream_t stream)
{
    if (!poolsOk(pools) || layer_count == 0 || layer_begin + layer_count > pools->layers
        || copies == nullptr || num_copies == nullptr || max_copies == 0 || max_copies > 65535u) {
        return KK_EINVAL;
    }
    PoolView v = view(*pools);
    v.status = status;
    return static_cast<int>(launch(kv_copy_kernel, dim3(max_copies, layer_count, 2), dim3(128), 0,
        stream, 1, v, layer_begin, copies, num_copies));
}

int kvWrite(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_slot const* slots, std::uint32_t num_lanes, std::uint16_t const* key,
    std::uint16_t const* value, std::uint64_t lane_stride, std::uint64_t layer_stride,
    unsigned int* status, cudaStream_t stream)
{
    if (!poolsOk(pools) || layer_count == 0 || layer_begin + layer_count > pools->layers
        || slots == nullptr || key == nullptr || value == nullptr || lane_stride % 8 != 0
        || layer_stride % 8 != 0 || num_lanes > 65535u) {
        return KK_EINVAL;
    }
    if (num_lanes == 0) {
        return 0;
    }
    PoolView v = view(*pools);
    v.status = status;
    return static_cast<int>(launch(kv_write_kernel, dim3(num_lanes, layer_count, 2), dim3(64), 0,
        stream, 1, v, layer_begin, slots, reinterpret_cast<__half const*>(key),
        reinterpret_cast<__half const*>(value), lane_stride, layer_stride));
}

int kvCopy(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_copy const* copies, std::uint32_t num_copies, unsigned int* status, cudaStream_t stream)
{
    if (!poolsOk(pools) || layer_count == 0 || layer_begin + layer_count > pools->layers
        || copies == nullptr || num_copies > 65535u) {
        return KK_EINVAL;
    }
    if (num_copies == 0) {
        return 0;
    }
    PoolView v = view(*pools);
    v.status = status;
    return static_cast<int>(launch(kv_copy_kernel, dim3(num_copies, layer_count, 2), dim3(128), 0,
        stream, 1, v, layer_begin, copies, static_cast<std::uint32_t const*>(nullptr)));
}
} // namespace kk
