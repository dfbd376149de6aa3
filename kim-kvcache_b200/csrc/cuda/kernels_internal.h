// Library-internal launch variants used by the model runner:
//  * counts read from device memory (so one captured CUDA graph serves every
//    step of a batch size: work lists change, kernel parameters do not);
//  * prepared GEMMs whose TMA tensor maps are encoded once at load.
#pragma once

#include "../../../include/kk_kernels.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>

namespace kk {

// Tokens per page of a pool descriptor's micro pool (0 means 8), and whether
// the descriptor names a supported size (8, or 16/32/64 for a fixed-page pool).
inline std::uint32_t microPageTokens(kk_kv_pools const& p) noexcept
{
    return p.micro_page_tokens == 0 ? 8u : p.micro_page_tokens;
}
inline bool microPageTokensValid(kk_kv_pools const& p) noexcept
{
    std::uint32_t const t = microPageTokens(p);
    return t == 8u || t == 16u || t == 32u || t == 64u;
}

// kk_paged_decode_attention with the item count in device memory; items
// beyond *num_items (<= max_items) are ignored. The grid is sized for max_items.
// Errors go to *status (a word of the caller's, zeroed by it) instead of the
// module's word that kk_device_status reads.
int attentionDevCount(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t const* num_items, std::uint32_t max_items,
    std::uint16_t const* query, std::uint32_t query_stride, std::uint16_t* output,
    std::uint32_t output_stride, float scale, void* workspace, std::uint64_t workspace_bytes,
    unsigned int* status, cudaStream_t stream);

// kk_paged_decode_attention reporting errors to *status (null: the module's
// word).
int attentionLaunch(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint16_t const* query,
    std::uint32_t query_stride, std::uint16_t* output, std::uint32_t output_stride, float scale,
    void* workspace, std::uint64_t workspace_bytes, unsigned int* status, cudaStream_t stream);

// attentionLaunch with the TMA kernel whatever the process-wide variant
// switch: the balanced work lists (kk_attention_plan_balanced) are served by
// it only. The caller checks attentionTmaSupported first.
int attentionLaunchTma(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint16_t const* query,
    std::uint32_t query_stride, std::uint16_t* output, std::uint32_t output_stride, float scale,
    void* workspace, std::uint64_t workspace_bytes, unsigned int* status, cudaStream_t stream);

// Parts for kk_attention_plan_balanced: one per SM, but none smaller than
// kAttnMinPartCost tokens of plan cost, so that a small batch is not cut
// into items shorter than what a first stage and a combine cost.
#ifdef KK_ATTN_MIN_PART_COST
constexpr std::uint32_t kAttnMinPartCost = KK_ATTN_MIN_PART_COST;
#else
constexpr std::uint32_t kAttnMinPartCost = 256;
#endif
std::uint32_t attentionPlanParts(kk_attn_lane const* lanes, std::uint32_t num_lanes, std::uint32_t sm_count);

// TMA-fed persistent attention kernel (attention_tma.cu): head_dim 64, 1/2/4/8
// KV heads, up to 16 query heads per KV head; serves both plan kinds
// (kk_attention_plan and kk_attention_plan_balanced). Arguments are validated
// by the caller; the workspace parts are as for the direct-load kernel.
bool attentionTmaSupported(kk_kv_pools const* pools, std::uint32_t q_heads);
int attentionTmaLaunch(kk_kv_pools const* pools, std::uint32_t layer, std::uint32_t q_heads,
    kk_page_desc const* descs, kk_attn_lane const* lanes, std::uint32_t num_lanes,
    kk_attn_item const* items, std::uint32_t num_items, std::uint32_t const* num_items_dev,
    std::uint16_t const* query, std::uint32_t query_stride, std::uint16_t* output,
    std::uint32_t output_stride, float scale, std::uint32_t* counters, float* part_o, float* part_ml,
    unsigned int* status, cudaStream_t stream);

// kk_kv_copy_tokens with the copy count in device memory (<= max_copies).
int kvCopyDevCount(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_copy const* copies, std::uint32_t const* num_copies, std::uint32_t max_copies,
    unsigned int* status, cudaStream_t stream);

// kk_kv_write / kk_kv_copy_tokens reporting errors to *status (null: the
// module's word).
int kvWrite(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_slot const* slots, std::uint32_t num_lanes, std::uint16_t const* key,
    std::uint16_t const* value, std::uint64_t lane_stride, std::uint64_t layer_stride,
    unsigned int* status, cudaStream_t stream);
int kvCopy(kk_kv_pools const* pools, std::uint32_t layer_begin, std::uint32_t layer_count,
    kk_kv_copy const* copies, std::uint32_t num_copies, unsigned int* status, cudaStream_t stream);

struct GemmPlan;
struct GemmPlanDeleter {
    void operator()(GemmPlan* p) const noexcept;
};
using GemmPlanPtr = std::unique_ptr<GemmPlan, GemmPlanDeleter>;

// Validates the descriptor, encodes its tensor maps and picks the split; rc
// receives 0 or the kk_gemm error code.
GemmPlanPtr gemmPlan(kk_gemm_desc const& desc, int& rc);
int gemmRun(GemmPlan const& plan, cudaStream_t stream);
// Every CTA of the plan's launches also asks L2 for its share of
// [ptr, ptr + bytes) once its own inputs are requested: bytes that a later
// kernel of the step streams (null or 0 clears it).
void gemmSetL2Prefetch(GemmPlan& plan, void const* ptr, std::uint64_t bytes);
// The plan's launches report errors to *status (null: the module's word).
void gemmSetStatus(GemmPlan& plan, unsigned int* status);

// Sums of squares for the fused RMSNorm, kept in arrays of rows of 64 floats
// (one row per 128-row tile of the producing projection, one column per
// batch row). A KK_EPI_RESIDUAL plan given an output writes, for each of its
// row tiles t and batch rows n, sq[t * 64 + n] = sum over the tile's rows of
// the new value squared; a plan with a normalised input given `tiles` such
// rows takes its RMS factors from them instead of re-reading the input rows.
bool gemmSetNormPartials(GemmPlan& plan, float const* sq_in, std::uint32_t tiles);
bool gemmSetSumSquaresOut(GemmPlan& plan, float* sq_out);

// kk_embed_rmsnorm that also writes each row's sum of squares of the
// gathered embedding to sq_out[row] (one tile's row of a sums-of-squares
// array); y may be null.
int embedSumSquares(std::uint16_t const* embed, std::uint32_t const* tokens, std::uint16_t* hidden,
    float* sq_out, std::uint32_t rows, std::uint32_t cols, cudaStream_t stream);

} // namespace kk
