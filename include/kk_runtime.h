/*
 * kim-kvcache B200 — C ABI of the host token-loop runtime.
 *
 * Plain C: fixed-width integers, opaque handles, caller-owned output buffers.
 * Return values are the reference's error enums as int (0 = success) unless a
 * function says otherwise. Nothing here throws or allocates on the caller's
 * behalf except the create functions, whose result is released by the
 * matching destroy function.
 *
 * The reference runtime is C++ only (no FFI); each entry point below wraps
 * one member of the reference's public C++ API, cited per function, so a
 * cgo / JNI / ctypes binding can drive the runtime without C++ types.
 *
 * Every kkrt_mgr_* function has a twin kref_mgr_* with identical signature in
 * the test-only oracle library (oracle/_ref/libkimkv_ref.so, built from the
 * reference's own sources) so the parity tests run identical op streams on
 * both and compare the outputs bit for bit.
 */
#ifndef KK_RUNTIME_H
#define KK_RUNTIME_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define KK_API __attribute__((visibility("default")))
#else
#define KK_API
#endif

/* One block-table entry (reference MappingEntry, include/kim-kv/core/block_table.h:13-41). */
typedef struct kk_entry {
    uint32_t logical_token_begin;
    uint16_t valid_tokens;
    uint8_t kind;        /* 0 micro (8 tokens), 1 extent (64 tokens) */
    uint8_t reserved;
    uint32_t slot;
    uint32_t generation;
} kk_entry;

/* Reference PageHandle (include/kim-kv/core/page_handle.h:10-47). */
typedef struct kk_handle {
    uint8_t kind;
    uint8_t reserved[3];
    uint32_t slot;
    uint32_t generation;
} kk_handle;

/* Reference PageMetadataSnapshot (include/kim-kv/runtime/kv_cache_manager.h:19-33). */
typedef struct kk_page_meta {
    uint8_t state;       /* 0 free, 1 mutable, 2 sealed, 3 copy_target, 4 retiring */
    uint8_t reserved;
    uint16_t valid_tokens;
    uint32_t ref_count;
    uint32_t promotion_pins;
    uint32_t inflight_readers;
    uint64_t mutable_owner;
} kk_page_meta;

/* Reference PagePoolSnapshot (include/kim-kv/core/page_pool.h:25-40). */
typedef struct kk_pool_snapshot {
    uint32_t total_slots;
    uint32_t free_slots;
    uint32_t allocated_slots;
    uint32_t reserved;
    uint64_t successful_allocations;
    uint64_t successful_releases;
    uint64_t failed_allocations;
    uint64_t rejected_releases;
} kk_pool_snapshot;

/* Reference KvCacheManagerSnapshot (include/kim-kv/runtime/kv_cache_manager.h:35-42). */
typedef struct kk_mgr_snapshot {
    uint64_t request_count;
    uint64_t promotion_count;
    uint64_t page_lease_count;
    uint64_t token_reservation_count;
    kk_pool_snapshot micro_pool;
    kk_pool_snapshot extent_pool;
} kk_mgr_snapshot;

/* A block table written into caller memory: `entries` holds `capacity`
 * slots; `count` receives the entry count (entries beyond capacity are
 * dropped, count still reports the full size). */
typedef struct kk_table_out {
    kk_entry* entries;
    uint32_t capacity;
    uint32_t count;
    uint64_t version;
} kk_table_out;

/* ---- KvCacheManager (include/kim-kv/runtime/kv_cache_manager.h:44-277) ---- */

/* KvCacheManager(micro_capacity, extent_capacity); NULL on invalid capacity. */
KK_API void* kkrt_mgr_create(uint32_t micro_capacity, uint32_t extent_capacity);
KK_API void kkrt_mgr_destroy(void* mgr);
/* createRequest (kv_cache_manager.cpp:22) */
KK_API int kkrt_mgr_create_request(void* mgr, uint64_t request_id);
/* append (kv_cache_append.cpp:12) */
KK_API int kkrt_mgr_append(void* mgr, uint64_t request_id, uint32_t token_count);
/* reserveToken (token_reservation.cpp:34): fills the reservation id and the
 * before / reserved tables. */
KK_API int kkrt_mgr_reserve_token(void* mgr, uint64_t request_id, uint32_t expected_committed,
    uint64_t* reservation_id, kk_table_out* before, kk_table_out* reserved);
/* commitTokenReservation / rollbackTokenReservation (token_reservation.cpp:190, :289) */
KK_API int kkrt_mgr_commit_reservation(void* mgr, uint64_t reservation_id);
KK_API int kkrt_mgr_rollback_reservation(void* mgr, uint64_t reservation_id);
/* sealTail / forkRequest / releaseRequest (kv_cache_lifecycle.cpp:12, :61, :145) */
KK_API int kkrt_mgr_seal_tail(void* mgr, uint64_t request_id);
KK_API int kkrt_mgr_fork(void* mgr, uint64_t source_id, uint64_t child_id);
KK_API int kkrt_mgr_release(void* mgr, uint64_t request_id);
/* preparePromotion (promotion.cpp:80): sources receives 8 handles. */
KK_API int kkrt_mgr_prepare_promotion(void* mgr, uint64_t request_id, uint32_t logical_begin,
    uint64_t* promotion_id, kk_handle* sources, kk_handle* target);
/* commitPromotion / rollbackPromotion (promotion.cpp:325, :279) */
KK_API int kkrt_mgr_commit_promotion(void* mgr, uint64_t promotion_id);
KK_API int kkrt_mgr_rollback_promotion(void* mgr, uint64_t promotion_id);
/* acquire*Lease / releasePageLease (page_lease.cpp:95-189, token_reservation.cpp:298) */
KK_API int kkrt_mgr_acquire_request_lease(void* mgr, uint64_t request_id, uint64_t* lease_id,
    uint32_t* handle_count);
KK_API int kkrt_mgr_acquire_promotion_lease(void* mgr, uint64_t promotion_id, uint64_t* lease_id,
    uint32_t* handle_count);
KK_API int kkrt_mgr_acquire_reservation_lease(void* mgr, uint64_t reservation_id,
    uint64_t* lease_id, uint32_t* handle_count);
KK_API int kkrt_mgr_release_lease(void* mgr, uint64_t lease_id);
/* blockTable (kv_cache_inspection.cpp:12): returns 1 when the request exists. */
KK_API int kkrt_mgr_block_table(void* mgr, uint64_t request_id, kk_table_out* out);
/* pageMetadata (kv_cache_inspection.cpp:27): returns 1 when the handle is current. */
KK_API int kkrt_mgr_page_metadata(void* mgr, kk_handle handle, kk_page_meta* out);
/* snapshot / checkInvariants (kv_cache_inspection.cpp:50, kv_cache_invariants.cpp:88) */
KK_API void kkrt_mgr_snapshot(void* mgr, kk_mgr_snapshot* out);
KK_API int kkrt_mgr_check_invariants(void* mgr);

/* ---- FixedPageManager (include/kim-kv/fixed/fixed_page_manager.h:30-166) ----
 * The single-kind page runtime (Fixed-8/16/32/64): same create / append /
 * reserve / seal / fork / partial-tail COW / release semantics with every page
 * holding tokens_per_page tokens; no promotion, no leases. Return values are
 * KvCacheError values. Every kkrt_fixed_* has a kref_fixed_* twin in the
 * parity oracle. */
typedef struct kk_fixed_snapshot {
    uint64_t request_count;
    uint64_t successful_allocations;
    uint64_t peak_allocated_pages;
    uint64_t token_reservation_count;
    kk_pool_snapshot pool;
} kk_fixed_snapshot;

/* Constructor (fixed_page_manager.cpp:28): NULL when tokens_per_page or
 * page_capacity is 0. */
KK_API void* kkrt_fixed_create(uint16_t tokens_per_page, uint32_t page_capacity);
KK_API void kkrt_fixed_destroy(void* mgr);
KK_API uint32_t kkrt_fixed_tokens_per_page(void* mgr);
KK_API int kkrt_fixed_create_request(void* mgr, uint64_t request_id);
/* append (fixed_page_manager.cpp:218): multi-token append with partial-tail COW. */
KK_API int kkrt_fixed_append(void* mgr, uint64_t request_id, uint32_t token_count);
/* reserveToken / commit / rollback (fixed_token_reservation.cpp:32, :172, :250). */
KK_API int kkrt_fixed_reserve_token(void* mgr, uint64_t request_id, uint32_t expected_committed,
    uint64_t* reservation_id, kk_table_out* before, kk_table_out* reserved);
KK_API int kkrt_fixed_commit_reservation(void* mgr, uint64_t reservation_id);
KK_API int kkrt_fixed_rollback_reservation(void* mgr, uint64_t reservation_id);
KK_API int kkrt_fixed_seal_tail(void* mgr, uint64_t request_id);
KK_API int kkrt_fixed_fork(void* mgr, uint64_t source_id, uint64_t child_id);
KK_API int kkrt_fixed_release(void* mgr, uint64_t request_id);
/* blockTable: returns 1 when the request exists. */
KK_API int kkrt_fixed_block_table(void* mgr, uint64_t request_id, kk_table_out* out);
KK_API void kkrt_fixed_snapshot(void* mgr, kk_fixed_snapshot* out);
KK_API int kkrt_fixed_check_invariants(void* mgr);

/* ---- weight manifest (include/kim-kv/model/weight_manifest.h:111-134) ---- */
/* loadWeightManifest, then validateWeightDataFile when data_path is not NULL;
 * returns the WeightManifestError of the first failing step (0 = valid). */
KK_API int kkrt_manifest_check(const char* manifest_path, const char* data_path);
/* computeWeightDataSha256: lower-case hex digest into out (65 bytes). */
KK_API int kkrt_sha256_range(const char* data_path, uint64_t offset, uint64_t byte_size, char* out);

/* ---- FP16 codec (include/kim-kv/reference/kv_reference.h:10-13) ---- */
KK_API uint16_t kkrt_float_to_half(float value);
KK_API float kkrt_half_to_float(uint16_t value);


/* ---- CUDA KV backend (include/kim-kv/cuda/cuda_engine_kv_backend.h:11-29) ---- */

typedef struct kk_backend_snapshot {  /* reference EngineKvBackendSnapshot (engine_kv.h:372-391) */
    uint64_t request_count;
    uint64_t active_transaction_count;
    uint64_t committed_token_count;
    uint64_t batched_attention_submissions;
    uint64_t batched_attention_lanes;
    uint32_t allocated_micro_pages;
    uint32_t allocated_extent_pages;
    uint64_t storage_reserved_bytes;
} kk_backend_snapshot;

/* createHeterogeneousCudaEngineKvBackend (backend.cpp:557): NULL on failure. */
KK_API void* kkrt_backend_create(uint32_t layers, uint32_t kv_heads, uint32_t head_dim,
    uint32_t q_heads, uint64_t attention_workspace_bytes, uint32_t micro_capacity,
    uint32_t extent_capacity);
/* createFixedCudaEngineKvBackend (include/kim-kv/cuda/cuda_engine_kv_backend.h:19-22,
 * src/cuda/engine/backend.cpp:579-598): FixedPageManager metadata and one device pool of
 * page_capacity pages of tokens_per_page (8, 16, 32 or 64) tokens; NULL on failure.
 * Every kkrt_backend_* call, the runner and the scheduler accept it; promotion does not
 * apply (kkrt_backend_promote returns EngineKvError::InvalidArgument). */
KK_API void* kkrt_fixed_backend_create(uint32_t layers, uint32_t kv_heads, uint32_t head_dim,
    uint32_t q_heads, uint64_t attention_workspace_bytes, uint32_t tokens_per_page,
    uint32_t page_capacity);
/* EngineKvBackend::kind(): 0 heterogeneous (two pools), 1 fixed-page. */
KK_API int kkrt_backend_kind(void* backend);
KK_API void kkrt_backend_destroy(void* backend);
/* createRequest / forkRequest / releaseRequest (backend.cpp:341-384): EngineKvError. */
KK_API int kkrt_backend_create_request(void* backend, uint64_t request_id);
KK_API int kkrt_backend_fork(void* backend, uint64_t source_id, uint64_t child_id);
KK_API int kkrt_backend_release(void* backend, uint64_t request_id);
KK_API int kkrt_backend_check_invariants(void* backend);
KK_API void kkrt_backend_snapshot(void* backend, kk_backend_snapshot* out);
/* injectCudaEngineFailureOnce (backend.cpp:600): point 0 submission, 1 completion. */
KK_API int kkrt_backend_inject_failure(void* backend, int point);
/* Device page pools of the backend (this library's kernel ABI view). */
KK_API int kkrt_backend_pools(void* backend, void* pools_out /* kk_kv_pools* */);
/* Committed block table of a request (1 = found). */
KK_API int kkrt_backend_block_table(void* backend, uint64_t request_id, kk_table_out* out);
/* Library extensions for building long prefixes without running the model:
 * metadata append of n tokens (KvCacheManager::append, kv_cache_append.cpp:12),
 * sealTail (kv_cache_lifecycle.cpp:12), and one promotion of the 8 micro pages
 * at logical_begin into an extent page, data copy included
 * (CudaKvCache::promote, src/cuda/kv/cache.cpp:172-229). EngineKvError. */
KK_API int kkrt_backend_append(void* backend, uint64_t request_id, uint32_t token_count);
KK_API int kkrt_backend_seal(void* backend, uint64_t request_id);
KK_API int kkrt_backend_promote(void* backend, uint64_t request_id, uint32_t logical_begin,
    void* stream);
/* K6 gather (CudaKvCache::gather, src/cuda/kv/gather.cpp:9-107): the
 * request's committed KV as one contiguous [layer][K|V][token][head][dim] fp16
 * tensor at device_output (16-byte aligned, committed-token-count tokens),
 * under a read lease; waits for the copy. Returns EngineKvError. */
KK_API int kkrt_backend_gather(void* backend, uint64_t request_id, void* device_output, void* stream);

/* ---- per-layer token transactions (engine_kv.h:255-351) ---- */
/* reserveToken: returns a transaction handle or NULL; *status = EngineKvError. */
KK_API void* kkrt_txn_reserve(void* backend, uint64_t request_id, uint32_t expected_committed,
    void* stream, int* status);
KK_API int kkrt_txn_write_layer(void* txn, uint32_t layer, const void* device_key,
    const void* device_value);
KK_API int kkrt_txn_attend_layer(void* txn, uint32_t layer, const void* device_query,
    void* device_output, void* device_workspace, uint64_t workspace_bytes, float scale);
/* attendLayerBatch over n transactions; queries/outputs are rows of one buffer each
 * (row stride row_bytes); statuses receives one EngineKvError per lane. */
KK_API void kkrt_txn_attend_batch(void* const* txns, uint32_t n, uint32_t layer,
    const void* device_query, void* device_output, uint64_t row_bytes, void* device_workspace,
    uint64_t workspace_bytes, float scale, int* statuses);
KK_API int kkrt_txn_commit(void* txn);
KK_API int kkrt_txn_rollback(void* txn);
/* Reserved block table of a transaction from this library's CUDA backend
 * (committed prefix + the current token; TokenReservationResult::reserved). */
KK_API int kkrt_txn_reserved_table(void* txn, kk_table_out* out);
/* TokenTransactionPhase (engine_kv.h:210-218). */
KK_API int kkrt_txn_phase(void* txn);
KK_API void kkrt_txn_destroy(void* txn);   /* rolls back if still active */

/* ---- CUDA TinyLlama runner (include/kim-kv/cuda/cuda_model_runner.h:178-184) ---- */
KK_API void* kkrt_runner_create(const char* manifest_path, const char* data_path, void* backend,
    void* stream, uint32_t max_batch_size, int use_cuda_graphs, int verify_checksums,
    int* status, char* detail, uint32_t detail_capacity);
/* Auto-promotion in the generation path (no counterpart in the reference,
 * which never promotes while generating): after a step commits a lane's
 * 64th token of a 64-aligned run, its 8 sealed micro pages become one extent
 * page (reference promotion semantics, src/runtime/promotion.cpp:80-457).
 * Returns 1 for a CUDA runner, 0 otherwise. Off by default. */
KK_API int kkrt_runner_set_auto_promote(void* runner, int enabled);
KK_API void kkrt_runner_destroy(void* runner);
/* generationForwardBatch (runner.cpp:410): per lane ok flag + greedy token.
 * Returns 1 when the batch result is well formed. */
KK_API int kkrt_runner_forward_batch(void* runner, uint32_t n, const uint64_t* request_ids,
    const uint32_t* token_ids, const uint32_t* positions, uint32_t* out_tokens, uint8_t* out_ok);
/* kkrt_runner_forward_batch that also fills logits [n][vocab] f32 (rows of
 * failed lanes zero). No counterpart in the reference (its batched path
 * returns tokens only): the same fused step run outside the captured graph,
 * for checking every lane against the reference arithmetic. */
KK_API int kkrt_runner_forward_batch_logits(void* runner, uint32_t n, const uint64_t* request_ids,
    const uint32_t* token_ids, const uint32_t* positions, uint32_t* out_tokens, uint8_t* out_ok,
    float* logits);
/* Fused multi-token prefill (no counterpart in the reference, which feeds a
 * prompt one position per scheduler wave): appends n prompt tokens of one
 * request at positions first_position.. (KvCacheManager::append semantics,
 * partial-tail copy-on-write included) and runs them through the decode step
 * in chunks of up to max_batch_size consecutive positions, each position
 * attending causally to the request's tokens [0, p]. The committed length
 * must equal first_position. *out_token receives the greedy token after the
 * last prompt position. Returns 1 on success, 0 on failure (detail via
 * kkrt_runner_last_error); a device failure releases the request. */
KK_API int kkrt_runner_prefill(void* runner, uint64_t request_id, const uint32_t* token_ids, uint32_t n,
    uint32_t first_position, uint32_t* out_token);
/* forwardToken (runner.cpp:53) with optional captures (each may be NULL):
 * logits [vocab] f32, embedding / final_hidden [hidden] f16, layer_hidden
 * [n_layers][hidden] f16 for the listed layers. Returns CudaModelRunnerError. */
KK_API int kkrt_runner_forward_token(void* runner, uint64_t request_id, uint32_t token_id,
    uint32_t position, uint32_t* out_token, float* logits, uint16_t* embedding,
    uint16_t* final_hidden, const uint32_t* layers, uint32_t n_layers, uint16_t* layer_hidden);
KK_API float kkrt_runner_last_step_ms(void* runner);
KK_API uint32_t kkrt_runner_last_launches(void* runner);
/* Host<->device bytes of the last fused step: the step-record upload and the
 * token (and logits) readback. Returns 0 for a non-CUDA runner. No counterpart
 * in the reference (its per-lane uploads are not aggregated). */
KK_API int kkrt_runner_last_transfer_bytes(void* runner, uint64_t* h2d, uint64_t* d2h);
/* Host wall time of the last fused step in microseconds, by phase, into
 * out[5]: lane reservations, step record (descriptors + work list), upload +
 * graph launch, wait for the device, commits + auto-promotion. Returns 5, or
 * 0 for a non-CUDA runner. No counterpart in the reference. */
KK_API int kkrt_runner_last_host_us(void* runner, float* out);
/* Detail text of the last failed fused step into out (NUL-terminated); returns its length. */
KK_API uint32_t kkrt_runner_last_error(void* runner, char* out, uint32_t capacity);

/* ---- generation loops (generation.h:178-202, iteration_scheduler.h:139-181) ---- */
typedef struct kk_terminal {
    uint64_t request_id;
    uint8_t reason;            /* GenerationTerminalReason */
    uint8_t error;             /* GenerationError */
    uint16_t reserved;
    uint32_t token_count;
    uint32_t prompt_tokens;
    uint32_t completion_tokens;
    uint64_t ttft_ns;
    uint64_t tpot_ns;
    uint64_t e2e_ns;
} kk_terminal;

typedef struct kk_iteration {
    uint64_t iteration;
    uint32_t model_forward_tokens;
    uint32_t model_forward_batches;
    uint32_t prefill_tokens;
    uint32_t decode_tokens;
    uint32_t terminals_produced;
    uint32_t reserved;
} kk_iteration;

/* model_runner: a runner handle from kkrt_runner_create or kkrt_fake_runner_create. */
KK_API void* kkrt_sched_create(void* backend, void* model_runner, uint32_t max_active,
    uint32_t max_batched_tokens, uint64_t max_kv_tokens, uint32_t prefill_chunk);
KK_API void kkrt_sched_destroy(void* sched);
/* submit: returns SchedulerAdmissionError (0 accepted). eos < 0: model default. */
KK_API int kkrt_sched_submit(void* sched, uint64_t request_id, const uint32_t* prompt,
    uint32_t prompt_len, uint32_t max_new_tokens, int64_t eos);
/* Extensions (no counterpart in the reference):
 * kkrt_sched_create_ex: flags bit 0 (KKRT_SCHED_FUSED_PREFILL) hands each
 * request's prompt quota of an iteration to the runner's fused prefill as one
 * multi-position call (IterationSchedulerConfig::fused_prefill).
 * kkrt_sched_submit_prefixed: the first kv_prefix_tokens prompt positions
 * are already committed under request_id in the KV backend (e.g. a prefix
 * shared by forking another request); the scheduler neither creates the KV
 * request nor feeds those positions (GenerationRequest::kv_prefix_tokens). */
#define KKRT_SCHED_FUSED_PREFILL 1u
KK_API void* kkrt_sched_create_ex(void* backend, void* model_runner, uint32_t max_active,
    uint32_t max_batched_tokens, uint64_t max_kv_tokens, uint32_t prefill_chunk, uint32_t flags);
KK_API int kkrt_sched_submit_prefixed(void* sched, uint64_t request_id, const uint32_t* prompt,
    uint32_t prompt_len, uint32_t max_new_tokens, int64_t eos, uint32_t kv_prefix_tokens);
KK_API int kkrt_sched_cancel(void* sched, uint64_t request_id);
KK_API void kkrt_sched_run_iteration(void* sched, kk_iteration* out);
KK_API void kkrt_sched_stop(void* sched);
KK_API int kkrt_sched_idle(void* sched);
/* drain / takeTerminals: fills up to cap terminals and their output tokens
 * (concatenated, token_capacity total); returns the number of terminals. */
KK_API uint32_t kkrt_sched_drain(void* sched, kk_terminal* out, uint32_t cap, uint32_t* tokens,
    uint32_t token_capacity);
KK_API uint32_t kkrt_sched_take_terminals(void* sched, kk_terminal* out, uint32_t cap,
    uint32_t* tokens, uint32_t token_capacity);
/* SingleRequestGenerationRuntime::generate; returns 1 and fills out/tokens. */
KK_API int kkrt_generate(void* backend, void* model_runner, uint64_t request_id,
    const uint32_t* prompt, uint32_t prompt_len, uint32_t max_new_tokens, int64_t eos,
    kk_terminal* out, uint32_t* tokens, uint32_t token_capacity);

/* ---- SPI test doubles (no device): the reference contract tests' fakes ---- */
/* A KV backend that only tracks request lifecycles. */
KK_API void* kkrt_fake_backend_create(void);
KK_API void kkrt_fake_backend_destroy(void* backend);
/* A model runner whose greedy token is a fixed hash of (request, token,
 * position) mod vocab; it logs every batch it receives. fail_request: a
 * request id whose steps fail (0 = none). */
KK_API void* kkrt_fake_runner_create(uint32_t vocab, uint32_t max_batch, uint32_t eos,
    uint32_t max_positions, uint64_t fail_request);
KK_API void kkrt_fake_runner_destroy(void* runner);
/* Batch log: sizes of the batches so far and their items (request, token, position). */
KK_API uint32_t kkrt_fake_runner_log(void* runner, uint32_t* batch_sizes, uint32_t cap_batches,
    uint64_t* items, uint32_t cap_items);

#ifdef __cplusplus
}
#endif

#endif /* KK_RUNTIME_H */
