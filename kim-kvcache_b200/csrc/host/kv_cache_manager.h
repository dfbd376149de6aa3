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
#include "page_pool.h"

#include <array>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <optional>
#include <unordered_map>
#include <vector>

namespace kimkvcache {

using RequestId = std::uint64_t;
using PromotionId = std::uint64_t;
using KvTokenReservationId = std::uint64_t;
using PageLeaseId = std::uint64_t;

constexpr RequestId kInvalidRequestId = 0;
constexpr PromotionId kInvalidPromotionId = 0;
constexpr KvTokenReservationId kInvalidKvTokenReservationId = 0;
constexpr PageLeaseId kInvalidPageLeaseId = 0;
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

// `before` stays globally visible until commit; `reserved` includes the
// uncommitted current token and is visible only to the owning transaction.
struct TokenReservationResult final {
    KvCacheError error{KvCacheError::None};
    KvTokenReservationId reservation_id{kInvalidKvTokenReservationId};
    RequestId request_id{kInvalidRequestId};
    std::uint32_t logical_token_position{0};
    BlockTable before{};
    BlockTable reserved{};

    [[nodiscard]] constexpr bool ok() const noexcept
    {
        return error == KvCacheError::None && reservation_id != kInvalidKvTokenReservationId;
    }
    [[nodiscard]] explicit constexpr operator bool() const noexcept { return ok(); }
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
    struct Page final {  // per-slot runtime state
        PageState state{PageState::Free};
        std::uint32_t generation{0};
        std::uint16_t valid_tokens{0};
        std::uint32_t ref_count{0};
        std::uint32_t promotion_pins{0};
        std::uint32_t inflight_readers{0};
        RequestId mutable_owner{kInvalidRequestId};
    };
    struct Staged final {
        PageHandle handle{};
        std::size_t entry_index{0};
    };
    struct Promotion final {
        PromotionId id{kInvalidPromotionId};
        RequestId request_id{kInvalidRequestId};
        std::uint64_t prepared_version{0};
        std::uint32_t logical_token_begin{0};
        std::size_t source_entry_index{0};
        std::array<PageHandle, kPromotionSourcePageCount> sources{};
        PageHandle target{};
    };
    struct Reservation final {
        KvTokenReservationId id{kInvalidKvTokenReservationId};
        RequestId request_id{kInvalidRequestId};
        std::uint64_t prepared_version{0};
        BlockTable candidate{};
        PageHandle staged_target{};
        PageHandle existing_mutable{};
        PageHandle replaced_sealed_tail{};
    };
    struct Lease final {
        PageLeaseId id{kInvalidPageLeaseId};
        std::vector<PageHandle> handles;
    };
    struct Audit;

    Page* page(PageHandle handle) noexcept;
    Page const* page(PageHandle handle) const noexcept;
    PagePool& poolFor(PageKind kind) noexcept { return kind == PageKind::Micro ? micro_pool_ : extent_pool_; }

    KvCacheError stageMicro(std::uint16_t initial_valid_tokens, PageHandle& out);
    KvCacheError stageExtent(PageHandle& out);
    void unstage(std::vector<Staged> const& staged) noexcept;
    KvCacheError dropReference(PageHandle handle);
    KvCacheError retireOrFree(PageHandle handle);
    static void clearFreed(Page& page) noexcept;
    bool hasReservation(RequestId request_id) const noexcept;

    // Next unused id from a wrapping counter that skips 0; among
    // live.size()+1 consecutive candidates at least one is unused.
    template <typename Map>
    static std::uint64_t nextFreeId(std::uint64_t& counter, Map const& live)
    {
        for (std::size_t attempt = 0; attempt <= live.size(); ++attempt) {
            std::uint64_t const candidate = counter++;
            if (counter == 0) {
                counter = 1;
            }
            if (candidate != 0 && live.find(candidate) == live.end()) {
                return candidate;
            }
        }
        return 0;
    }

    PageLeaseAcquireResult pinPages(std::vector<PageHandle> handles, BlockTable const* table);
    PageLeaseAcquireResult pinTokenReservation(KvTokenReservationId id, bool describe);
    KvCacheError rollbackReservationLocked(KvTokenReservationId id);
    KvCacheError rollbackPromotionLocked(PromotionId id);
    KvCacheError rollbackRequestPromotionsLocked(RequestId request_id);

    bool auditLocked() const;
    bool auditRequests(Audit& audit) const;
    bool auditPromotions(Audit& audit) const;
    bool auditReservations(Audit& audit) const;
    bool auditLeases(Audit& audit) const;
    bool auditPool(PageKind kind, Audit const& audit) const;

    PagePool micro_pool_;
    PagePool extent_pool_;
    std::vector<Page> micro_pages_;
    std::vector<Page> extent_pages_;

    std::unordered_map<RequestId, BlockTable> requests_;
    // Iteration order of this map decides which pending promotions a request
    // release rolls back first, which is observable through the free-list
    // order; a libstdc++ unordered_map fed the same insert/erase sequence as
    // the reference reproduces it exactly.
    std::unordered_map<PromotionId, Promotion> promotions_;
    std::unordered_map<KvTokenReservationId, Reservation> reservations_;
    std::unordered_map<RequestId, KvTokenReservationId> request_reservation_;
    std::unordered_map<PageLeaseId, Lease> leases_;

    std::uint64_t next_promotion_id_{1};
    std::uint64_t next_reservation_id_{1};
    std::uint64_t next_lease_id_{1};

    mutable std::mutex mutex_;
};
// Page records by handle (inline: every lease pins and releases each page of
// a table, so this runs tens of times per token reservation).
inline KvCacheManager::Page const* KvCacheManager::page(PageHandle handle) const noexcept
{
    if (!handle.isStructurallyValid()) {
        return nullptr;
    }
    std::vector<Page> const& pages =
        handle.kind == PageKind::Micro ? micro_pages_ : extent_pages_;
    if (handle.slot >= pages.size() || pages[handle.slot].generation != handle.generation) {
        return nullptr;
    }
    return &pages[handle.slot];
}

inline KvCacheManager::Page* KvCacheManager::page(PageHandle handle) noexcept
{
    return const_cast<Page*>(static_cast<KvCacheManager const*>(this)->page(handle));
}


} // namespace kimkvcache
