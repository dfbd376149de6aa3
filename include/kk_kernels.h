/*
 * kim-kvcache B200 — C ABI of the sm_100a token-loop kernels.
 *
 * These entry points replace the reference's internal CUDA launch layer and
 * its cuBLAS calls:
 *   src/cuda/kv/kernels.cuh:31-143          cuda_detail::launch* (KV pages, attention)
 *   src/cuda/model/kernels.cuh:11-117       cuda_model_detail::launch* (norm, RoPE, ...)
 *   src/cuda/model/runner_support.cpp:196-274  cublasGemmEx wrappers (dense projections)
 *
 * Conventions: plain pointers to device memory, sizes in elements unless
 * named *_bytes, `stream` is a cudaStream_t (NULL = legacy default stream).
 * Every function returns 0 on a successful launch, KK_EINVAL for rejected
 * arguments (nothing is launched), or a CUDA runtime error code.
 * FP16 tensors are passed as uint16_t bit patterns.
 *
 * KV page layout (same as the reference, include/kim-kv/core/kv_layout.h:73-90):
 * a page holds every layer of its tokens as [layer][K/V][token][kv_head][dim];
 * micro pages hold 8 tokens, extent pages 64; pools are arrays of pages.
 */
#ifndef KK_KERNELS_H
#define KK_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KK_KAPI __attribute__((visibility("default")))
#else
#define KK_KAPI
#endif

#define KK_EINVAL 1000
/* Native error code of a transaction or step that failed because one of its
 * kernels reported an error (a descriptor outside its pool, a bounded device
 * wait that ran out) instead of the CUDA runtime. */
#define KK_EDEVICE 1002

typedef struct kk_kv_pools {
    void* micro;               /* micro_capacity pages of layers*2*T*kv_heads*head_dim fp16,
                                  T = micro_page_tokens (8 when 0) */
    void* extent;              /* extent_capacity pages of layers*2*64*kv_heads*head_dim fp16 */
    uint32_t micro_capacity;
    uint32_t extent_capacity;
    uint32_t layers;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t micro_page_tokens; /* tokens per micro page: 0 or 8 (the two-pool runtime), or
                                   16/32/64 for a fixed-page backend's pool (reference
                                   EngineBackendState(config, tokens_per_page, capacity),
                                   src/cuda/engine/backend.cpp:91-106); the extent pool is then
                                   unused (extent_capacity 0) */
} kk_kv_pools;

/* One block-table entry as the kernels read it (reference DeviceBlockDescriptor,
 * include/kim-kv/engine/engine_kv.h:100-117, without the generation). */
typedef struct kk_page_desc {
    uint32_t slot;
    uint32_t logical_token_begin;
    uint16_t valid_tokens;
    uint8_t kind;              /* 0 micro, 1 extent */
    uint8_t reserved0;
    uint32_t reserved1;
} kk_page_desc;

/* Destination of one lane's new token (reference CudaEngineTransaction::writeLayer
 * slot mapping, src/cuda/engine/transaction.cpp:158-194). */
typedef struct kk_kv_slot {
    uint32_t slot;
    uint16_t page_token;
    uint8_t kind;
    uint8_t active;            /* 0: lane skipped */
} kk_kv_slot;

/* Partial-tail copy-on-write: first `tokens` tokens of src -> dst. */
typedef struct kk_kv_copy {
    uint32_t src_slot;
    uint32_t dst_slot;
    uint16_t tokens;
    uint8_t src_kind;
    uint8_t dst_kind;
} kk_kv_copy;

/* One lane of a ragged decode-attention batch (reference DevicePagedDecodeBatchItem,
 * include/kim-kv/engine/engine_kv.h:172-181). */
typedef struct kk_attn_lane {
    uint32_t desc_offset;      /* first entry of this lane in the descriptor array */
    uint32_t desc_count;
    uint32_t token_count;      /* attended tokens, current token included */
    uint32_t item_offset;      /* filled by kk_attention_plan */
    uint32_t item_count;       /* filled by kk_attention_plan */
    uint32_t query_row;        /* row of query / output used by this lane */
    uint32_t first_item_shared; /* filled by the planners: 1 when the lane's first item
                                   begins in an earlier lane */
    uint32_t reserved;
} kk_attn_lane;

/* A split-KV work item: a run [desc_begin, desc_end) of the descriptor array.
 * Items of kk_attention_plan lie inside one lane (flags 0); items of
 * kk_attention_plan_balanced may continue from `lane` into the following
 * lanes when their descriptors are contiguous (flags KK_ATTN_ITEM_MULTI_LANE),
 * and may cut a full 64-token extent page in half: the item's first
 * descriptor then starts at token KK_ATTN_ITEM_SKIP(flags) and its last one
 * ends at token KK_ATTN_ITEM_LIMIT(flags) (0: at its valid count), so two
 * consecutive items share that descriptor. Only extent descriptors may be cut. */
#define KK_ATTN_ITEM_MULTI_LANE 1u
#define KK_ATTN_ITEM_SKIP(flags) (((flags) >> 8) & 0xffu)
#define KK_ATTN_ITEM_LIMIT(flags) (((flags) >> 16) & 0xffu)
#define KK_ATTN_EXTENT_HALF 32u
typedef struct kk_attn_item {
    uint32_t lane;             /* first lane of the item */
    uint32_t desc_begin;
    uint32_t desc_end;
    uint32_t reserved;         /* flags */
} kk_attn_item;

/* ---- K1: fused GQA paged decode attention ------------------------------------
 * Replaces launchPagedDecodeAttention / launchPagedDecodeAttentionBatch
 * (src/cuda/attention/paged_decode_kernels.cu:533-617): QK^T, online softmax and
 * PV in one pass that walks micro and extent entries directly, all lanes and
 * KV heads of a layer in one launch, split over the context with a combine.
 * head_dim must be 64; kv_heads in {1,2,4,8}; q_heads/kv_heads <= 16.
 * query/output rows: [q_heads][head_dim] fp16 at row stride *_stride elements. */
KK_KAPI uint32_t kk_attention_plan(const kk_page_desc* host_descs, kk_attn_lane* host_lanes,
    uint32_t num_lanes, uint32_t target_tokens, kk_attn_item* host_items, uint32_t max_items);
/* Token-balanced plan (no counterpart in the reference): cuts the batch's
 * token stream, lane after lane, into about num_parts runs of equal token
 * count at page granularity (use the SM count: one run per SM). Runs may span
 * lanes; a lane split across runs is combined by the split-KV combine. Fills
 * item_offset/item_count/first_item_shared of every lane; returns the item count (items beyond
 * max_items are counted, not written). Served by the TMA kernel only. */
KK_KAPI uint32_t kk_attention_plan_balanced(const kk_page_desc* host_descs,
    kk_attn_lane* host_lanes, uint32_t num_lanes, uint32_t num_parts, kk_attn_item* host_items,
    uint32_t max_items);
KK_KAPI uint64_t kk_attention_workspace_bytes(uint32_t num_lanes, uint32_t num_items,
    uint32_t q_heads, uint32_t head_dim);
/* Zero-fills the per-lane completion counters of a fresh workspace (once). */
KK_KAPI int kk_attention_workspace_init(void* workspace, uint32_t num_lanes, void* stream);
KK_KAPI int kk_paged_decode_attention(const kk_kv_pools* pools, uint32_t layer,
    uint32_t q_heads, const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, const uint16_t* query, uint32_t query_stride,
    uint16_t* output, uint32_t output_stride, float scale, void* workspace,
    uint64_t workspace_bytes, void* stream);

/* kk_paged_decode_attention without a caller workspace. No counterpart in
 * the reference, which allocates attention scratch per call.
 *
 * It is for callers that cannot allocate device memory for the workspace:
 *  - hosts that reach the library through an FFI (cgo, JNI, ctypes) with only
 *    raw stream handles and no device allocator of their own;
 *  - serving loops that must not call cudaMalloc per step, because it
 *    synchronizes the device and its latency is unbounded.
 *
 * The completion counters and partial softmax states live in one fixed
 * device array of KK_ATTN_SCRATCH_BYTES (4 MiB) per device, created with the
 * library's module. A call that needs more,
 * kk_attention_workspace_bytes(num_lanes, num_items, q_heads, 64) >
 * KK_ATTN_SCRATCH_BYTES, is rejected with KK_ENOSCRATCH and launches
 * nothing. For scale: 64 lanes x 148 items x 32 query heads need 2.5 MB.
 *
 * The per-lane completion counters at the start of the scratch must be zero
 * when a kernel starts. This entry point zeroes them on `stream` before every
 * launch. Nothing else needs initial values.
 *
 * The first call on each device (the device that owns `stream`) looks up the
 * scratch address; make it before any stream capture. Arguments are checked
 * before anything is queued: a rejected call writes nothing. Calls that can overlap on one device (different
 * streams, or several host threads) share the one scratch array and race:
 * serialize them on one stream, or use kk_paged_decode_attention with a
 * workspace per stream. Other arguments, results and errors are those of
 * kk_paged_decode_attention. */
#define KK_ATTN_SCRATCH_BYTES (4u << 20)
#define KK_ENOSCRATCH 1001
KK_KAPI int kk_paged_decode_attention_noalloc(const kk_kv_pools* pools, uint32_t layer,
    uint32_t q_heads, const kk_page_desc* descs, const kk_attn_lane* lanes, uint32_t num_lanes,
    const kk_attn_item* items, uint32_t num_items, const uint16_t* query, uint32_t query_stride,
    uint16_t* output, uint32_t output_stride, float scale, void* stream);

/* Kernel used by kk_paged_decode_attention (process-wide; default AUTO). No
 * counterpart in the reference (it has one attention implementation).
 *  KK_ATTN_AUTO   : the TMA kernel where supported (kv_heads in {1,2,4,8},
 *                   which is every shape the direct-load kernel serves);
 *  KK_ATTN_DIRECT : always the direct-load kernel (warps load K/V rows into
 *                   registers);
 *  KK_ATTN_TMA    : always the TMA kernel (persistent, warp-specialised, K/V
 *                   staged through a 3-stage shared-memory ring); calls it
 *                   cannot serve return KK_EINVAL.
 * The direct-load kernel rejects multi-lane items (device status
 * kErrBadArgument = 3, items skipped).
 * Both produce the same results within FP32 rounding of the softmax sums.
 * Returns 0 or KK_EINVAL for an unknown value. */
#define KK_ATTN_AUTO 0
#define KK_ATTN_DIRECT 1
#define KK_ATTN_TMA 2
KK_KAPI int kk_attention_set_variant(int variant);

/* ---- K2: batched KV append / copy-on-write -----------------------------------
 * kk_kv_write replaces launchWriteLayerToken (paged_decode_kernels.cu:65-99) and
 * launchAppendTokens (src/cuda/kv/page_kernels.cu:77-127) for one token per
 * lane: writes K and V of layers [layer_begin, +layer_count) for every active
 * lane. key/value element (lane, layer, head, dim) lives at
 * lane*lane_stride + layer*layer_stride + head*head_dim + dim.
 * kk_kv_copy_tokens replaces launchCopyLayerTokens / launchCopyPageTokens
 * (paged_decode_kernels.cu:29-63, page_kernels.cu:46-75). */
KK_KAPI int kk_kv_write(const kk_kv_pools* pools, uint32_t layer_begin, uint32_t layer_count,
    const kk_kv_slot* slots, uint32_t num_lanes, const uint16_t* key, const uint16_t* value,
    uint64_t lane_stride, uint64_t layer_stride, void* stream);
KK_KAPI int kk_kv_copy_tokens(const kk_kv_pools* pools, uint32_t layer_begin,
    uint32_t layer_count, const kk_kv_copy* copies, uint32_t num_copies, void* stream);

/* Promotion copy: the 8 micro pages micro_slots[0..7] (all layers) become the
 * extent page extent_slot, tokens 8k..8k+7 <- micro page k (replaces
 * launchPromotion, src/cuda/kv/page_kernels.cu:129-182). */
KK_KAPI int kk_kv_promote(const kk_kv_pools* pools, const uint32_t* micro_slots_host,
    uint32_t extent_slot, void* stream);
/* K6 data path between pages and a contiguous KV tensor
 * [layer][K|V][token][head][dim] fp16 (16-byte aligned).
 * kk_kv_gather replaces gatherAsync / launchGather (src/cuda/kv/gather.cpp:9-107,
 * page_kernels.cu:184-242): every descriptor's valid tokens are copied to
 * out at their logical positions; tokens of [0, total_tokens) not covered by
 * any descriptor are left untouched. Descriptors must not overlap.
 * kk_kv_scatter is the inverse for appended tokens (appendAsync segment
 * copies, launchAppendTokens, page_kernels.cu:77-127): `in` holds the
 * [layer][K|V][token_count][head][dim] values of logical tokens
 * [first_token, first_token + token_count), written into the pages that the
 * descriptors map there. One CTA per (descriptor, layer, K|V). A descriptor
 * outside its pool is skipped and reported by kk_device_status. */
KK_KAPI int kk_kv_gather(const kk_kv_pools* pools, const kk_page_desc* descs, uint32_t num_descs,
    uint32_t total_tokens, uint16_t* out, void* stream);
KK_KAPI int kk_kv_scatter(const kk_kv_pools* pools, const kk_page_desc* descs, uint32_t num_descs,
    uint32_t first_token, uint32_t token_count, const uint16_t* in, void* stream);
/* Deterministic pseudo-random FP16 fill (uniform in [-scale, scale)) for
 * synthetic KV pages and test tensors; same (seed, index) -> same value. */
KK_KAPI int kk_fill_fp16(uint16_t* data, uint64_t count, uint64_t seed, float scale,
    void* stream);

/* ---- K3: norms, RoPE, SiLU gate, residual -------------------------------------
 * Replace launchRmsNorm(Batch), launchRope(Batch), launchSwiGlu, launchResidualAdd,
 * launchEmbedding(Batch) (src/cuda/model/kernels.cu:16-218). */
KK_KAPI int kk_rmsnorm(const uint16_t* x, const uint16_t* weight, uint16_t* y, uint32_t rows,
    uint32_t cols, float eps, void* stream);
KK_KAPI int kk_embed_rmsnorm(const uint16_t* embed, const uint32_t* tokens,
    const uint16_t* weight, uint16_t* hidden, uint16_t* y, uint32_t rows, uint32_t cols,
    float eps, void* stream);
KK_KAPI int kk_rope(uint16_t* q, uint32_t q_stride, uint16_t* k, uint32_t k_stride,
    const uint32_t* positions, uint32_t rows, uint32_t q_heads, uint32_t kv_heads,
    uint32_t head_dim, float theta, void* stream);
KK_KAPI int kk_silu_mul(const uint16_t* gate, const uint16_t* up, uint16_t* out, uint32_t rows,
    uint32_t cols, void* stream);
KK_KAPI int kk_residual_add(uint16_t* hidden, const uint16_t* update, uint64_t count,
    void* stream);

/* ---- K4/K5: tcgen05 weight-streaming GEMM with fused epilogues ---------------
 * Y[n][m] = sum_k W[m][k] * X[n][k] for m < M, n < N (N <= 64): FP16 operands,
 * FP32 accumulation in tensor memory, split-K across a thread-block cluster with
 * a distributed-shared-memory reduction, then one of the epilogues below.
 * Replaces cublasGemmEx in gemmBatch / logitsGemmBatch
 * (src/cuda/model/runner_support.cpp:196-274) plus the elementwise kernel that
 * follows each projection. K % 8 == 0. */
enum kk_epilogue {
    KK_EPI_STORE_F16 = 0,    /* out[n*out_stride+m] = half(acc) */
    KK_EPI_STORE_F32 = 1,    /* out[n*out_stride+m] = acc */
    KK_EPI_RESIDUAL = 2,     /* out[...] = hadd(out[...], half(acc)) */
    KK_EPI_SILU_PAIRS = 3,   /* rows 2i / 2i+1 = gate_i / up_i: out[n*out_stride+i] =
                                half(silu(half(g)) * half(u)) */
    KK_EPI_QKV_ROPE = 4,     /* rows [0,q_rows): q, RoPE'd into out; next kv_rows: k,
                                RoPE'd into the KV page slot; next kv_rows: v into the page */
    KK_EPI_ARGMAX = 5,       /* fp32 logits (optional) + greedy argmax per column */
};

typedef struct kk_gemm_desc {
    const uint16_t* weight;    /* [M][K] fp16 row-major */
    uint32_t M;
    uint32_t K;
    const uint16_t* x;         /* [x_rows][x_stride] fp16 */
    uint32_t N;
    uint32_t x_stride;
    uint32_t x_rows;           /* allocated rows of x (>= N) */
    uint32_t epilogue;
    void* out;
    uint32_t out_stride;
    uint32_t split_k;          /* 0 = choose automatically */
    /* KK_EPI_QKV_ROPE */
    const uint32_t* positions; /* [N] */
    const kk_kv_slot* slots;   /* [N] */
    kk_kv_pools pools;
    uint32_t layer;
    uint32_t q_rows;
    uint32_t kv_rows;
    uint32_t head_dim;
    float rope_theta;
    /* KK_EPI_ARGMAX */
    uint32_t* tokens;          /* [N] greedy ids */
    void* argmax_workspace;    /* kk_argmax_workspace_bytes(M, N) bytes, zeroed once */
    uint32_t weight_layout;    /* KK_W_ROW_MAJOR, or KK_W_PACKED: weight holds
                                  kk_gemm_pack_weight output for (M, K) */
    /* Fused RMSNorm of the input rows (replaces a separate rmsNormBatchKernel,
     * src/cuda/model/kernels.cu:48-124, at the same FP16 rounding point): when
     * norm_input is set, every X tile is normalised in shared memory before
     * the tensor cores read it, X'[n][k] = half(x[n][k] * r[n] * g[k]) with
     * r[n] = 1 / sqrt(mean_k norm_input[n][k]^2 + norm_eps) and g =
     * norm_weight (1 when NULL); then Y = X' W^T. With x = norm_input this is
     * the reference's half(RMSNorm(x)) followed by the projection. */
    const uint16_t* norm_input; /* [N][norm_stride] fp16, 16-byte aligned, or NULL */
    uint32_t norm_stride;
    float norm_eps;
    const uint16_t* norm_weight; /* [K] fp16, 16-byte aligned, or NULL */
    /* KK_EPI_QKV_ROPE: optional table of the rotation factors, [rope_positions]
     * [head_dim / 2] pairs (cos, sin) of position * theta^(-2d / head_dim),
     * 8-byte aligned; NULL computes them in the kernel (sincosf). The runner
     * fills it once on the host, with the host math library the reference's
     * model uses, for every position up to max_position_embeddings. */
    const float* rope_cos_sin;
    uint32_t rope_positions;
} kk_gemm_desc;

#define KK_W_ROW_MAJOR 0
#define KK_W_PACKED 1
/* Weight packing (no counterpart in the reference, whose cuBLAS calls read the
 * row-major tensors): W [M][K] row-major (K % 8 == 0, 16-byte aligned) ->
 * 128x64 tiles of 16 KB, each contiguous and pre-swizzled, so that the GEMM
 * streams one tile per untiled bulk copy. Rows and columns are zero-padded to
 * multiples of 128 and 64. Done once at weight load. */
KK_KAPI uint64_t kk_gemm_packed_bytes(uint32_t M, uint32_t K);
KK_KAPI int kk_gemm_pack_weight(const uint16_t* weight, uint32_t M, uint32_t K,
    uint16_t* packed, void* stream);
/* The same with every column k scaled by col_scale[k] (fp16, 16-byte aligned)
 * before packing, W'[m][k] = half(W[m][k] * col_scale[k]): folds an RMSNorm
 * weight into the projection that consumes the normalised rows. */
KK_KAPI int kk_gemm_pack_weight_scaled(const uint16_t* weight, uint32_t M, uint32_t K,
    const uint16_t* col_scale, uint16_t* packed, void* stream);

KK_KAPI uint64_t kk_argmax_workspace_bytes(uint32_t M, uint32_t N);
KK_KAPI int kk_gemm(const kk_gemm_desc* desc, void* stream);

/* Reads and clears the device-side status words of all kernel modules
 * (synchronises the stream). 0 = no kernel recorded an error. These words
 * collect the errors of the entry points above; the runtime's own launches
 * (kk_runtime.h: the runner's fused step, the backend's per-layer
 * transactions) report into per-step and per-stream words of their own and
 * fail the affected transactions at commit. */
KK_KAPI int kk_device_status(void* stream);

/* Test hook for the bounded waits of K1 (no counterpart in the reference,
 * whose failure injection is host-side only): from the next launch on, CTA 0
 * of every TMA attention launch on the current device drops its stage number
 * `stage` (issues no copy and no arrival for it), so that the consumers'
 * bounded wait runs out after `wait_limit_ns` and the kernel reports
 * kErrWaitTimeout and returns. stage 0xFFFFFFFF and wait_limit_ns 0 restore
 * the defaults (no stage dropped, 2 s). Call it with no kernel in flight. */
KK_KAPI int kk_debug_attention_fault(uint32_t stage, uint64_t wait_limit_ns);

/* Programmatic dependent launch for subsequent launches on this thread (0/1). */
KK_KAPI void kk_set_pdl(int enabled);

#ifdef __cplusplus
}
#endif

#endif /* KK_KERNELS_H */
