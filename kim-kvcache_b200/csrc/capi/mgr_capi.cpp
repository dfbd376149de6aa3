// C ABI over KvCacheManager (declarations and reference citations in
// include/kk_runtime.h).
#include "../../../include/kk_runtime.h"
#include "../host/fixed_page_manager.h"
#include "../host/fp16_codec.h"
#include "../host/kv_cache_manager.h"
#include "../host/weight_manifest.h"

#include <cstring>

#include <new>

using namespace kimkvcache;

namespace {

KvCacheManager* M(void* mgr) { return static_cast<KvCacheManager*>(mgr); }
FixedPageManager* F(void* mgr) { return static_cast<FixedPageManager*>(mgr); }

void writeTable(BlockTable const& table, kk_table_out* out)
{
    if (out == nullptr) {
        return;
    }
    auto const& entries = table.entries();
    out->count = static_cast<uint32_t>(entries.size());
    out->version = table.version();
    for (std::size_t i = 0; i < entries.size() && i < out->capacity; ++i) {
        kk_entry& e = out->entries[i];
        e.logical_token_begin = entries[i].logical_token_begin;
        e.valid_tokens = entries[i].valid_tokens;
        e.kind = static_cast<uint8_t>(entries[i].kind);
        e.reserved = 0;
        e.slot = entries[i].handle.slot;
        e.generation = entries[i].handle.generation;
    }
}

kk_handle toC(PageHandle h)
{
    kk_handle out{};
    out.kind = static_cast<uint8_t>(h.kind);
    out.slot = h.slot;
    out.generation = h.generation;
    return out;
}

int leaseOut(PageLeaseAcquireResult const& r, uint64_t* lease_id, uint32_t* handle_count)
{
    if (lease_id != nullptr) {
        *lease_id = r.lease_id;
    }
    if (handle_count != nullptr) {
        *handle_count = static_cast<uint32_t>(r.handles.size());
    }
    return static_cast<int>(r.error);
}

} // namespace

extern "C" {

void* kkrt_mgr_create(uint32_t micro_capacity, uint32_t extent_capacity)
{
    try {
        return new KvCacheManager(micro_capacity, extent_capacity);
    } catch (...) {
        return nullptr;
    }
}

void kkrt_mgr_destroy(void* mgr) { delete M(mgr); }

int kkrt_mgr_create_request(void* mgr, uint64_t id) { return int(M(mgr)->createRequest(id)); }
int kkrt_mgr_append(void* mgr, uint64_t id, uint32_t n) { return int(M(mgr)->append(id, n)); }

int kkrt_mgr_reserve_token(void* mgr, uint64_t request_id, uint32_t expected,
    uint64_t* reservation_id, kk_table_out* before, kk_table_out* reserved)
{
    TokenReservationResult const r = M(mgr)->reserveToken(request_id, expected);
    if (reservation_id != nullptr) {
        *reservation_id = r.reservation_id;
    }
    writeTable(r.before, before);
    writeTable(r.reserved, reserved);
    return static_cast<int>(r.error);
}

int kkrt_mgr_commit_reservation(void* mgr, uint64_t id)
{
    return int(M(mgr)->commitTokenReservation(id));
}
int kkrt_mgr_rollback_reservation(void* mgr, uint64_t id)
{
    return int(M(mgr)->rollbackTokenReservation(id));
}
int kkrt_mgr_seal_tail(void* mgr, uint64_t id) { return int(M(mgr)->sealTail(id)); }
int kkrt_mgr_fork(void* mgr, uint64_t s, uint64_t c) { return int(M(mgr)->forkRequest(s, c)); }
int kkrt_mgr_release(void* mgr, uint64_t id) { return int(M(mgr)->releaseRequest(id)); }

int kkrt_mgr_prepare_promotion(void* mgr, uint64_t request_id, uint32_t begin,
    uint64_t* promotion_id, kk_handle* sources, kk_handle* target)
{
    PromotionPrepareResult const r = M(mgr)->preparePromotion(request_id, begin);
    if (promotion_id != nullptr) {
        *promotion_id = r.promotion_id;
    }
    for (std::size_t k = 0; sources != nullptr && k < kPromotionSourcePageCount; ++k) {
        sources[k] = toC(r.source_handles[k]);
    }
    if (target != nullptr) {
        *target = toC(r.target_handle);
    }
    return static_cast<int>(r.error);
}

int kkrt_mgr_commit_promotion(void* mgr, uint64_t id) { return int(M(mgr)->commitPromotion(id)); }
int kkrt_mgr_rollback_promotion(void* mgr, uint64_t id)
{
    return int(M(mgr)->rollbackPromotion(id));
}

int kkrt_mgr_acquire_request_lease(void* mgr, uint64_t id, uint64_t* lease, uint32_t* n)
{
    return leaseOut(M(mgr)->acquireRequestReadLease(id), lease, n);
}
int kkrt_mgr_acquire_promotion_lease(void* mgr, uint64_t id, uint64_t* lease, uint32_t* n)
{
    return leaseOut(M(mgr)->acquirePromotionIoLease(id), lease, n);
}
int kkrt_mgr_acquire_reservation_lease(void* mgr, uint64_t id, uint64_t* lease, uint32_t* n)
{
    return leaseOut(M(mgr)->acquireTokenReservationLease(id), lease, n);
}
int kkrt_mgr_release_lease(void* mgr, uint64_t id) { return int(M(mgr)->releasePageLease(id)); }

int kkrt_mgr_block_table(void* mgr, uint64_t request_id, kk_table_out* out)
{
    std::optional<BlockTable> const table = M(mgr)->blockTable(request_id);
    if (!table) {
        return 0;
    }
    writeTable(*table, out);
    return 1;
}

int kkrt_mgr_page_metadata(void* mgr, kk_handle handle, kk_page_meta* out)
{
    PageHandle const h{static_cast<PageKind>(handle.kind), handle.slot, handle.generation};
    std::optional<PageMetadataSnapshot> const meta = M(mgr)->pageMetadata(h);
    if (!meta) {
        return 0;
    }
    out->state = static_cast<uint8_t>(meta->state);
    out->reserved = 0;
    out->valid_tokens = meta->valid_tokens;
    out->ref_count = meta->ref_count;
    out->promotion_pins = meta->promotion_pins;
    out->inflight_readers = meta->inflight_readers;
    out->mutable_owner = meta->mutable_owner;
    return 1;
}

static void poolOut(PagePoolSnapshot const& s, kk_pool_snapshot* out)
{
    out->total_slots = s.total_slots;
    out->free_slots = s.free_slots;
    out->allocated_slots = s.allocated_slots;
    out->reserved = 0;
    out->successful_allocations = s.successful_allocations;
    out->successful_releases = s.successful_releases;
    out->failed_allocations = s.failed_allocations;
    out->rejected_releases = s.rejected_releases;
}

void kkrt_mgr_snapshot(void* mgr, kk_mgr_snapshot* out)
{
    KvCacheManagerSnapshot const s = M(mgr)->snapshot();
    out->request_count = s.request_count;
    out->promotion_count = s.promotion_count;
    out->page_lease_count = s.page_lease_count;
    out->token_reservation_count = s.token_reservation_count;
    poolOut(s.micro_pool, &out->micro_pool);
    poolOut(s.extent_pool, &out->extent_pool);
}

int kkrt_mgr_check_invariants(void* mgr) { return M(mgr)->checkInvariants() ? 1 : 0; }

void* kkrt_fixed_create(uint16_t tokens_per_page, uint32_t page_capacity)
{
    try {
        return new FixedPageManager(tokens_per_page, page_capacity);
    } catch (...) {
        return nullptr;
    }
}

void kkrt_fixed_destroy(void* mgr) { delete F(mgr); }
uint32_t kkrt_fixed_tokens_per_page(void* mgr) { return F(mgr)->tokensPerPage(); }
int kkrt_fixed_create_request(void* mgr, uint64_t id) { return int(F(mgr)->createRequest(id)); }
int kkrt_fixed_append(void* mgr, uint64_t id, uint32_t n) { return int(F(mgr)->append(id, n)); }

int kkrt_fixed_reserve_token(void* mgr, uint64_t request_id, uint32_t expected,
    uint64_t* reservation_id, kk_table_out* before, kk_table_out* reserved)
{
    TokenReservationResult const r = F(mgr)->reserveToken(request_id, expected);
    if (reservation_id != nullptr) {
        *reservation_id = r.reservation_id;
    }
    writeTable(r.before, before);
    writeTable(r.reserved, reserved);
    return static_cast<int>(r.error);
}

int kkrt_fixed_commit_reservation(void* mgr, uint64_t id) { return int(F(mgr)->commitTokenReservation(id)); }
int kkrt_fixed_rollback_reservation(void* mgr, uint64_t id)
{
    return int(F(mgr)->rollbackTokenReservation(id));
}
int kkrt_fixed_seal_tail(void* mgr, uint64_t id) { return int(F(mgr)->sealTail(id)); }
int kkrt_fixed_fork(void* mgr, uint64_t s, uint64_t c) { return int(F(mgr)->forkRequest(s, c)); }
int kkrt_fixed_release(void* mgr, uint64_t id) { return int(F(mgr)->releaseRequest(id)); }

int kkrt_fixed_block_table(void* mgr, uint64_t id, kk_table_out* out)
{
    std::optional<BlockTable> const t = F(mgr)->blockTable(id);
    if (!t) {
        return 0;
    }
    writeTable(*t, out);
    return 1;
}

void kkrt_fixed_snapshot(void* mgr, kk_fixed_snapshot* out)
{
    FixedPageManagerSnapshot const s = F(mgr)->snapshot();
    out->request_count = s.request_count;
    out->successful_allocations = s.successful_allocations;
    out->peak_allocated_pages = s.peak_allocated_pages;
    out->token_reservation_count = s.token_reservation_count;
    poolOut(s.pool, &out->pool);
}

int kkrt_fixed_check_invariants(void* mgr) { return F(mgr)->checkInvariants() ? 1 : 0; }

int kkrt_manifest_check(const char* manifest_path, const char* data_path)
{
    WeightManifestLoadResult const loaded = loadWeightManifest(manifest_path);
    if (!loaded.ok()) {
        return static_cast<int>(loaded.status.error);
    }
    if (data_path == nullptr) {
        return 0;
    }
    return static_cast<int>(validateWeightDataFile(loaded.manifest, data_path).error);
}

int kkrt_sha256_range(const char* data_path, uint64_t offset, uint64_t bytes, char* out)
{
    std::string digest;
    WeightManifestStatus const s = computeWeightDataSha256(data_path, offset, bytes, digest);
    if (!s.ok()) {
        return static_cast<int>(s.error);
    }
    std::memcpy(out, digest.c_str(), digest.size() + 1);
    return 0;
}

uint16_t kkrt_float_to_half(float value) { return floatToKvScalar(value); }
float kkrt_half_to_float(uint16_t value) { return kvScalarToFloat(value); }

} // extern "C"
