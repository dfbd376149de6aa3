// Heterogeneous (8-token micro + 64-token extent) KV page metadata runtime.
//
// Public surface and semantics follow the reference KvCacheManager
// (include/kim-kv/runtime/kv_cache_manager.h:44-277 and the sources under
// src/runtime/): multi-token append, single-token reservations with
// commit/rollback, sealing, prefix fork with partial-tail copy-on-write,
// 8-micro -> 1-extent promotion, page leases and a full invariant checker.
// Every observable value (page tables, versions, slot numbers, generations,
// page states and counters) is bit-identical to the reference for the same
// sequence of calls; the parity tests drive both with identical op streams.
#pragma once

#include "kv_types.h"
#include "paged_tables.h"

#include <array>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <optional>
#include <unordered_map>
#include <vector>

namespace kimkvcache {

constexpr std::size_t kPromotionSourcePageCount = 8;

struct PromotionPrepareResult final {
    KvCacheError error{KvCacheError::None};
    PromotionId promotion_id{kInvalidPromotionId};
    RequestId request_id{kInvalidRequestId};
    std::uint32_t logical_token_begin{0};
    std::array<PageHandle, kPromotionSourcePageCount> source_handles{};
    PageHandle target_handle{PageHandle::invalid()};

    [[nodiscard]] constexpr bool ok() const noexcept { return error == KvCacheError::None; }
    [[nodiscard]] explicit constexpr operator bool() const noexcept { return ok(); }
};

struct PromotionTransactionSnapshot final {
    PromotionId promotion_id{kInvalidPromotionId};
    RequestId request_id{kInvalidRequestId};
    std::uint64_t prepared_table_version{0};
    std::uint32_t logical_token_begin{0};
    std::array<PageHandle, kPromotionSourcePageCount> source_handles{};
    PageHandle target_handle{PageHandle::invalid()};
};

// A lease pins pages against reuse while device work may still touch them:
// a page that loses its last table reference while leased goes to Retiring
// and returns to its pool only when the lease is released.
struct PageLeaseAcquireResult final {
    KvCacheError error{KvCacheError::None};
    PageLeaseId lease_id{kInvalidPageLeaseId};
    BlockTable table{};
    std::vector<PageHandle> handles{};

    [[nodiscard]] bool ok() const noexcept { return error == KvCacheError::None; }
    [[nodiscard]] explicit operator bool() const noexcept { return ok(); }
};

struct PageMetadataSnapshot final {
    PageHandle handle{PageHandle::invalid()};
    PageState state{PageState::Free};
    std::uint16_t valid_tokens{0};
    std::uint32_t ref_count{0};
    std::uint32_t promotion_pins{0};
    std::uint32_t inflight_readers{0};
    RequestId mutable_owner{kInvalidRequestId};

    [[nodiscard]] constexpr bool shared() const noexcept
    {
        return state == PageState::Sealed && ref_count > 1;
    }
};

struct KvCacheManagerSnapshot final {
    std::uint64_t request_count{0};
    std::uint64_t promotion_count{0};
    std::uint64_t page_lease_count{0};
    std::uint64_t token_reservation_count{0};
    PagePoolSnapshot micro_pool{};
    PagePoolSnapshot extent_pool{};
};

class KvCacheManager final {
public:
    KvCacheManager(std::uint32_t micro_capacity, std::uint32_t extent_capacity);

    KvCacheManager(KvCacheManager const&) = delete;
    KvCacheManager& operator=(KvCacheManager const&) = delete;

    [[nodiscard]] KvCacheError createRequest(RequestId request_id);
    [[nodiscard]] KvCacheError append(RequestId request_id, std::uint32_t token_count);

    [[nodiscard]] TokenReservationResult reserveToken(
        RequestId request_id, std::uint32_t expected_committed_tokens);
    [[nodiscard]] KvCacheError commitTokenReservation(KvTokenReservationId id);
    [[nodiscard]] KvCacheError rollbackTokenReservation(KvTokenReservationId id);

    [[nodiscard]] KvCacheError sealTail(RequestId request_id);
    [[nodiscard]] KvCacheError forkRequest(RequestId source, RequestId child);
    [[nodiscard]] KvCacheError releaseRequest(RequestId request_id);

    [[nodiscard]] PromotionPrepareResult preparePromotion(
        RequestId request_id, std::uint32_t logical_token_begin);
    [[nodiscard]] KvCacheError commitPromotion(PromotionId id);
    [[nodiscard]] KvCacheError rollbackPromotion(PromotionId id);

    [[nodiscard]] PageLeaseAcquireResult acquireRequestReadLease(RequestId request_id);
    [[nodiscard]] PageLeaseAcquireResult acquirePromotionIoLease(PromotionId id);
    [[nodiscard]] PageLeaseAcquireResult acquireTokenReservationLease(KvTokenReservationId id);
    // The same lease, returning only its id (table and handles left empty):
    // for a caller that already holds the reserved table, as the device
    // backend does on every token reservation.
    [[nodiscard]] PageLeaseAcquireResult acquireTokenReservationPin(KvTokenReservationId id);
    [[nodiscard]] KvCacheError releasePageLease(PageLeaseId lease_id);

    [[nodiscard]] std::optional<BlockTable> blockTable(RequestId request_id) const;
    [[nodiscard]] std::optional<PageMetadataSnapshot> pageMetadata(PageHandle handle) const;
    [[nodiscard]] std::optional<PromotionTransactionSnapshot> promotionTransaction(
        PromotionId id) const;
    [[nodiscard]] KvCacheManagerSnapshot snapshot() const;
    [[nodiscard]] bool checkInvariants() const;

private:
    // A prepared promotion: the 8 source pages stay pinned and the target
    // extent staged until commit or rollback.
    struct Promotion final {
        RequestId request_id{kInvalidRequestId};
        std::uint64_t prepared_version{0};
        std::uint32_t logical_token_begin{0};
        std::size_t first_entry{0};
        std::array<PageHandle, kPromotionSourcePageCount> sources{};
        PageHandle target{};
    };

    [[nodiscard]] bool promoting(RequestId request_id) const;
    [[nodiscard]] bool runEligible(BlockTable const& table, std::size_t first, std::uint32_t begin,
        std::array<PageHandle, kPromotionSourcePageCount> const* expect, std::uint32_t pins) const;
    [[nodiscard]] KvCacheError undoPromotion(PromotionId id);
    [[nodiscard]] PageLeaseAcquireResult lease(std::vector<PageHandle> handles, BlockTable const* table);
    [[nodiscard]] PageLeaseAcquireResult leaseReservation(KvTokenReservationId id, bool describe);

    TableEngine core_;
    // Iteration order of this map decides which pending promotions a request
    // release rolls back first, which is observable through the free-list
    // order; a libstdc++ unordered_map fed the same insert/erase sequence as
    // the reference reproduces it exactly.
    std::unordered_map<PromotionId, Promotion> promotions_;
    std::unordered_map<PageLeaseId, std::vector<PageHandle>> leases_;
    IdSequence promotion_ids_;
    IdSequence lease_ids_;
    mutable std::mutex mutex_;
};

} // namespace kimkvcache
