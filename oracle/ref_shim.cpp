// TEST INFRASTRUCTURE ONLY — never linked into, loaded by, or called from the
// product library.
//
// C shim over the reference implementation itself: compiled together with
// the reference's own CPU sources (read in place from the reference tree by
// oracle/Makefile) into oracle/_ref/libkimkv_ref.so. Exposes kref_* twins of
// the kkrt_* entry points in include/kk_runtime.h so the parity tests can run
// identical operation streams on the reference and on the product runtime.
#include "../include/kk_runtime.h"

#include "kim-kv/fixed/fixed_page_manager.h"
#include "kim-kv/model/weight_manifest.h"
#include "kim-kv/reference/kv_reference.h"
#include "kim-kv/runtime/kv_cache_manager.h"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <thread>
#include <vector>

using namespace kimkvcache;

namespace {

KvCacheManager* M(void* p) { return static_cast<KvCacheManager*>(p); }
FixedPageManager* F(void* p) { return static_cast<FixedPageManager*>(p); }

void tableOut(BlockTable const& t, kk_table_out* out)
{
    if (out == nullptr) {
        return;
    }
    out->count = static_cast<uint32_t>(t.entries().size());
    out->version = t.version();
    for (std::size_t i = 0; i < t.entries().size() && i < out->capacity; ++i) {
        MappingEntry const& m = t.entries()[i];
        out->entries[i] = kk_entry{m.logical_token_begin, m.valid_tokens,
            static_cast<uint8_t>(m.kind), 0, m.handle.slot, m.handle.generation};
    }
}

kk_handle handleOut(PageHandle h)
{
    kk_handle out{};
    out.kind = static_cast<uint8_t>(h.kind);
    out.slot = h.slot;
    out.generation = h.generation;
    return out;
}

int leaseOut(PageLeaseAcquireResult const& r, uint64_t* lease, uint32_t* n)
{
    if (lease != nullptr) *lease = r.lease_id;
    if (n != nullptr) *n = static_cast<uint32_t>(r.handles.size());
    return static_cast<int>(r.error);
}

void poolOut(PagePoolSnapshot const& s, kk_pool_snapshot* o)
{
    o->total_slots = s.total_slots;
    o->free_slots = s.free_slots;
    o->allocated_slots = s.allocated_slots;
    o->reserved = 0;
    o->successful_allocations = s.successful_allocations;
    o->successful_releases = s.successful_releases;
    o->failed_allocations = s.failed_allocations;
    o->rejected_releases = s.rejected_releases;
}

} // namespace

extern "C" {

KK_API void* kref_mgr_create(uint32_t micro, uint32_t extent)
{
    try {
        return new KvCacheManager(micro, extent);
    } catch (...) {
        return nullptr;
    }
}
KK_API void kref_mgr_destroy(void* p) { delete M(p); }
KK_API int kref_mgr_create_request(void* p, uint64_t id) { return int(M(p)->createRequest(id)); }
KK_API int kref_mgr_append(void* p, uint64_t id, uint32_t n) { return int(M(p)->append(id, n)); }
KK_API int kref_mgr_reserve_token(void* p, uint64_t id, uint32_t expected, uint64_t* rid,
    kk_table_out* before, kk_table_out* reserved)
{
    TokenReservationResult const r = M(p)->reserveToken(id, expected);
    if (rid != nullptr) *rid = r.reservation_id;
    tableOut(r.before, before);
    tableOut(r.reserved, reserved);
    return static_cast<int>(r.error);
}
KK_API int kref_mgr_commit_reservation(void* p, uint64_t id)
{
    return int(M(p)->commitTokenReservation(id));
}
KK_API int kref_mgr_rollback_reservation(void* p, uint64_t id)
{
    return int(M(p)->rollbackTokenReservation(id));
}
KK_API int kref_mgr_seal_tail(void* p, uint64_t id) { return int(M(p)->sealTail(id)); }
KK_API int kref_mgr_fork(void* p, uint64_t s, uint64_t c) { return int(M(p)->forkRequest(s, c)); }
KK_API int kref_mgr_release(void* p, uint64_t id) { return int(M(p)->releaseRequest(id)); }
KK_API int kref_mgr_prepare_promotion(void* p, uint64_t id, uint32_t begin, uint64_t* pid,
    kk_handle* sources, kk_handle* target)
{
    PromotionPrepareResult const r = M(p)->preparePromotion(id, begin);
    if (pid != nullptr) *pid = r.promotion_id;
    for (std::size_t k = 0; sources != nullptr && k < kPromotionSourcePageCount; ++k) {
        sources[k] = handleOut(r.source_handles[k]);
    }
    if (target != nullptr) *target = handleOut(r.target_handle);
    return static_cast<int>(r.error);
}
KK_API int kref_mgr_commit_promotion(void* p, uint64_t id) { return int(M(p)->commitPromotion(id)); }
KK_API int kref_mgr_rollback_promotion(void* p, uint64_t id)
{
    return int(M(p)->rollbackPromotion(id));
}
KK_API int kref_mgr_acquire_request_lease(void* p, uint64_t id, uint64_t* l, uint32_t* n)
{
    return leaseOut(M(p)->acquireRequestReadLease(id), l, n);
}
KK_API int kref_mgr_acquire_promotion_lease(void* p, uint64_t id, uint64_t* l, uint32_t* n)
{
    return leaseOut(M(p)->acquirePromotionIoLease(id), l, n);
}
KK_API int kref_mgr_acquire_reservation_lease(void* p, uint64_t id, uint64_t* l, uint32_t* n)
{
    return leaseOut(M(p)->acquireTokenReservationLease(id), l, n);
}
KK_API int kref_mgr_release_lease(void* p, uint64_t id) { return int(M(p)->releasePageLease(id)); }
KK_API int kref_mgr_block_table(void* p, uint64_t id, kk_table_out* out)
{
    std::optional<BlockTable> const t = M(p)->blockTable(id);
    if (!t) return 0;
    tableOut(*t, out);
    return 1;
}
KK_API int kref_mgr_page_metadata(void* p, kk_handle h, kk_page_meta* out)
{
    std::optional<PageMetadataSnapshot> const m =
        M(p)->pageMetadata(PageHandle{static_cast<PageKind>(h.kind), h.slot, h.generation});
    if (!m) return 0;
    out->state = static_cast<uint8_t>(m->state);
    out->reserved = 0;
    out->valid_tokens = m->valid_tokens;
    out->ref_count = m->ref_count;
    out->promotion_pins = m->promotion_pins;
    out->inflight_readers = m->inflight_readers;
    out->mutable_owner = m->mutable_owner;
    return 1;
}
KK_API void kref_mgr_snapshot(void* p, kk_mgr_snapshot* out)
{
    KvCacheManagerSnapshot const s = M(p)->snapshot();
    out->request_count = s.request_count;
    out->promotion_count = s.promotion_count;
    out->page_lease_count = s.page_lease_count;
    out->token_reservation_count = s.token_reservation_count;
    poolOut(s.micro_pool, &out->micro_pool);
    poolOut(s.extent_pool, &out->extent_pool);
}
KK_API int kref_mgr_check_invariants(void* p) { return M(p)->checkInvariants() ? 1 : 0; }

KK_API uint16_t kref_float_to_half(float v) { return floatToKvScalar(v); }
KK_API float kref_half_to_float(uint16_t v) { return kvScalarToFloat(v); }

// referenceAttention (src/reference/kv_reference.cpp:136-234) on a contiguous
// [layer][K/V][token][head][dim] FP16 buffer with an FP32 query [layer][head][dim].
// Returns 1 on success.
KK_API int kref_reference_attention(uint32_t layers, uint32_t heads, uint32_t dim,
    uint16_t const* kv, uint32_t token_count, float const* query, float* output)
{
    KvLayout const layout{layers, heads, dim};
    std::size_t elements = 0;
    if (!layout.elementsForTokens(token_count, elements)) return 0;
    std::vector<KvScalar> contiguous(kv, kv + elements);
    std::size_t const q_elems = static_cast<std::size_t>(layers) * heads * dim;
    std::vector<float> q(query, query + q_elems);
    std::vector<float> out;
    if (!referenceAttention(layout, contiguous, token_count, q, out)) return 0;
    std::memcpy(output, out.data(), out.size() * sizeof(float));
    return 1;
}

// One step of the config-1 workload on the host, with the reference's own
// parts: per lane KvCacheManager::reserveToken(expected) for the next token,
// the new token's K / V (FP16, [lanes][kv_heads][dim]) stored into the host
// pools at the reserved page, the lane's reserved table gathered per KV head
// into a contiguous [K|V][token][dim] buffer (the CPU form of gatherKernel,
// src/cuda/kv/page_kernels.cu:184-242), referenceAttention per query head on
// its KV head (KvLayout{1, 1, dim}) rounded to FP16 as the paged kernel
// stores it, then commit (commit != 0) or rollback of every reservation.
// Pools: micro [slot][layers][K|V][8][kv_heads][dim], extent the same with
// 64 tokens. (lane, KV head) pairs run on `threads` std::threads.
// Returns 1 on success, 0 when a reservation or an attention call fails.
KK_API int kref_c1_step(void* mgr, uint32_t lanes, uint64_t const* ids, uint32_t const* expected,
    uint16_t* micro, uint16_t* extent, uint32_t layers, uint32_t layer, uint32_t kv_heads, uint32_t dim,
    uint32_t q_heads, uint16_t const* k_new, uint16_t const* v_new, uint16_t const* q, uint16_t* out,
    int commit, uint32_t threads)
{
    if (kv_heads == 0 || q_heads % kv_heads != 0 || layer >= layers) return 0;
    std::vector<TokenReservationResult> res;
    res.reserve(lanes);
    bool ok = true;
    for (uint32_t i = 0; i < lanes && ok; ++i) {
        res.push_back(M(mgr)->reserveToken(ids[i], expected[i]));
        ok = res.back().ok();
    }
    auto element = [&](MappingEntry const& m, uint32_t within, uint32_t kv, uint32_t h) -> uint16_t* {
        std::size_t const page_tokens = m.kind == PageKind::Micro ? 8 : 64;
        uint16_t* pool = m.kind == PageKind::Micro ? micro : extent;
        std::size_t const off = ((((std::size_t(m.handle.slot) * layers + layer) * 2 + kv) * page_tokens
                                     + within) * kv_heads + h) * dim;
        return pool + off;
    };
    auto locate = [](BlockTable const& t, uint32_t token, uint32_t& within) -> MappingEntry const* {
        for (MappingEntry const& m : t.entries()) {
            if (token >= m.logical_token_begin && token < m.logical_token_begin + m.valid_tokens) {
                within = token - m.logical_token_begin;
                return &m;
            }
        }
        return nullptr;
    };
    for (uint32_t i = 0; i < lanes && ok; ++i) {
        // Partial-tail copy-on-write, as the reference backend performs it
        // (src/cuda/kv/append.cpp:45-98): an entry of `before` whose handle
        // changed in `reserved` is the shared partial tail, and its valid
        // tokens are copied into the new page (every layer, K and V).
        for (MappingEntry const& old_entry : res[i].before.entries()) {
            for (MappingEntry const& now : res[i].reserved.entries()) {
                if (now.logical_token_begin != old_entry.logical_token_begin || now.handle == old_entry.handle) {
                    continue;
                }
                for (uint32_t l = 0; l < layers; ++l) {
                    for (uint32_t kv = 0; kv < 2; ++kv) {
                        for (uint32_t t = 0; t < old_entry.valid_tokens; ++t) {
                            std::size_t const row = std::size_t(kv_heads) * dim;
                            std::size_t const src = (((std::size_t(old_entry.handle.slot) * layers + l) * 2 + kv) * 8 + t) * row;
                            std::size_t const dst = (((std::size_t(now.handle.slot) * layers + l) * 2 + kv) * 8 + t) * row;
                            std::memcpy(micro + dst, micro + src, row * 2);
                        }
                    }
                }
            }
        }
        uint32_t within = 0;
        MappingEntry const* m = locate(res[i].reserved, expected[i], within);
        if (m == nullptr) {
            ok = false;
            break;
        }
        for (uint32_t h = 0; h < kv_heads; ++h) {
            std::memcpy(element(*m, within, 0, h), k_new + (std::size_t(i) * kv_heads + h) * dim, dim * 2);
            std::memcpy(element(*m, within, 1, h), v_new + (std::size_t(i) * kv_heads + h) * dim, dim * 2);
        }
    }
    std::atomic<uint32_t> next{0};
    std::atomic<bool> failed{false};
    uint32_t const group = q_heads / kv_heads;
    auto work = [&]() {
        std::vector<KvScalar> kv;
        std::vector<float> query(dim), o;
        for (uint32_t w = next.fetch_add(1); w < lanes * kv_heads; w = next.fetch_add(1)) {
            uint32_t const i = w / kv_heads;
            uint32_t const h = w % kv_heads;
            uint32_t const tokens = expected[i] + 1;
            kv.assign(std::size_t(2) * tokens * dim, 0);
            for (MappingEntry const& m : res[i].reserved.entries()) {
                for (uint32_t t = 0; t < m.valid_tokens; ++t) {
                    uint32_t const token = m.logical_token_begin + t;
                    if (token >= tokens) continue;
                    std::memcpy(&kv[std::size_t(token) * dim], element(m, t, 0, h), dim * 2);
                    std::memcpy(&kv[(std::size_t(tokens) + token) * dim], element(m, t, 1, h), dim * 2);
                }
            }
            for (uint32_t g = 0; g < group; ++g) {
                uint32_t const qh = h * group + g;
                uint16_t const* qs = q + (std::size_t(i) * q_heads + qh) * dim;
                for (uint32_t d = 0; d < dim; ++d) {
                    query[d] = kvScalarToFloat(qs[d]);
                }
                if (!referenceAttention(KvLayout{1, 1, dim}, kv, tokens, query, o)) {
                    failed = true;
                    return;
                }
                uint16_t* os = out + (std::size_t(i) * q_heads + qh) * dim;
                for (uint32_t d = 0; d < dim; ++d) {
                    os[d] = floatToKvScalar(o[d]);
                }
            }
        }
    };
    if (ok) {
        std::vector<std::thread> pool;
        for (uint32_t t = 1; t < std::max<uint32_t>(1u, std::min(threads, lanes * kv_heads)); ++t) {
            pool.emplace_back(work);
        }
        work();
        for (std::thread& t : pool) {
            t.join();
        }
    }
    for (TokenReservationResult const& r : res) {
        if (r.ok()) {
            KvCacheError const e = commit != 0 && ok && !failed
                ? M(mgr)->commitTokenReservation(r.reservation_id)
                : M(mgr)->rollbackTokenReservation(r.reservation_id);
            ok = ok && e == KvCacheError::None;
        }
    }
    return ok && !failed ? 1 : 0;
}

// loadWeightManifest + validateWeightDataFile (src/model/weight_manifest.cpp:461-684).
// Returns the WeightManifestError of the first failing step (0 = both ok).
KK_API int kref_manifest_check(char const* manifest_path, char const* data_path)
{
    WeightManifestLoadResult const loaded = loadWeightManifest(manifest_path);
    if (!loaded.ok()) return static_cast<int>(loaded.status.error);
    if (data_path == nullptr) return 0;
    return static_cast<int>(validateWeightDataFile(loaded.manifest, data_path).error);
}

// computeWeightDataSha256 (src/model/weight_manifest.cpp:648-684); hex digest
// into out (65 bytes).
KK_API int kref_sha256_range(char const* data_path, uint64_t offset, uint64_t bytes, char* out)
{
    std::string digest;
    WeightManifestStatus const s = computeWeightDataSha256(data_path, offset, bytes, digest);
    if (!s.ok()) return static_cast<int>(s.error);
    std::memcpy(out, digest.c_str(), digest.size() + 1);
    return 0;
}

KK_API void* kref_fixed_create(uint16_t tokens, uint32_t capacity)
{
    try {
        return new FixedPageManager(tokens, capacity);
    } catch (...) {
        return nullptr;
    }
}
KK_API void kref_fixed_destroy(void* p) { delete F(p); }
KK_API uint32_t kref_fixed_tokens_per_page(void* p) { return F(p)->tokensPerPage(); }
KK_API int kref_fixed_create_request(void* p, uint64_t id) { return int(F(p)->createRequest(id)); }
KK_API int kref_fixed_append(void* p, uint64_t id, uint32_t n) { return int(F(p)->append(id, n)); }
KK_API int kref_fixed_reserve_token(void* p, uint64_t id, uint32_t expected, uint64_t* rid,
    kk_table_out* before, kk_table_out* reserved)
{
    TokenReservationResult const r = F(p)->reserveToken(id, expected);
    if (rid != nullptr) *rid = r.reservation_id;
    tableOut(r.before, before);
    tableOut(r.reserved, reserved);
    return int(r.error);
}
KK_API int kref_fixed_commit_reservation(void* p, uint64_t id) { return int(F(p)->commitTokenReservation(id)); }
KK_API int kref_fixed_rollback_reservation(void* p, uint64_t id)
{
    return int(F(p)->rollbackTokenReservation(id));
}
KK_API int kref_fixed_seal_tail(void* p, uint64_t id) { return int(F(p)->sealTail(id)); }
KK_API int kref_fixed_fork(void* p, uint64_t s, uint64_t c) { return int(F(p)->forkRequest(s, c)); }
KK_API int kref_fixed_release(void* p, uint64_t id) { return int(F(p)->releaseRequest(id)); }
KK_API int kref_fixed_block_table(void* p, uint64_t id, kk_table_out* out)
{
    std::optional<BlockTable> const t = F(p)->blockTable(id);
    if (!t) return 0;
    tableOut(*t, out);
    return 1;
}
KK_API void kref_fixed_snapshot(void* p, kk_fixed_snapshot* out)
{
    FixedPageManagerSnapshot const s = F(p)->snapshot();
    out->request_count = s.request_count;
    out->successful_allocations = s.successful_allocations;
    out->peak_allocated_pages = s.peak_allocated_pages;
    out->token_reservation_count = s.token_reservation_count;
    poolOut(s.pool, &out->pool);
}
KK_API int kref_fixed_check_invariants(void* p) { return F(p)->checkInvariants() ? 1 : 0; }

} // extern "C"
