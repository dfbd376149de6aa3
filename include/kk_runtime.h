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

/* ---- FP16 codec (include/kim-kv/reference/kv_reference.h:10-13) ---- */
KK_API uint16_t kkrt_float_to_half(float value);
KK_API float kkrt_half_to_float(uint16_t value);

#ifdef __cplusplus
}
#endif

#endif /* KK_RUNTIME_H */
