// Fixed-page KV metadata runtime: one page kind, a configurable token
// capacity per page (Fixed-8/16/32/64), the strategy baseline the reference
// compares its two-pool runtime against
// (include/kim-kv/fixed/fixed_page_manager.h:30-166,
// src/fixed/fixed_page_manager.cpp, src/fixed/fixed_token_reservation.cpp).
//
// Create / append / reserve-commit-rollback / seal / fork / partial-tail COW /
// release follow the two-pool manager's semantics with every page of size
// tokens_per_page; there is no promotion and there are no leases. Pages carry
// PageKind::Micro in block tables (the kind only names the pool), and table
// invariants are checked against tokens_per_page.
#pragma once

#include "kv_cache_manager.h"
#include "page_pool.h"

#include <cstdint>
#include <mutex>
#include <optional>
#include <unordered_map>
#include <vector>

namespace kimkvcache {

struct FixedPageManagerSnapshot final {
    std::uint64_t request_count{0};
    std::uint64_t successful_allocations{0};
    std::uint64_t peak_allocated_pages{0};
    std::uint64_t token_reservation_count{0};
    PagePoolSnapshot pool{};
};

class FixedPageManager final {
public:
    // Throws std::invalid_argument when tokens_per_page or page_capacity is 0.
    FixedPageManager(std::uint16_t tokens_per_page, std::uint32_t page_capacity);

    FixedPageManager(FixedPageManager const&) = delete;
    FixedPageManager& operator=(FixedPageManager const&) = delete;

    [[nodiscard]] std::uint16_t tokensPerPage() const noexcept { return page_tokens_; }

    [[nodiscard]] KvCacheError createRequest(RequestId request_id);
    [[nodiscard]] KvCacheError append(RequestId request_id, std::uint32_t token_count);
    [[nodiscard]] TokenReservationResult reserveToken(RequestId request_id,
        std::uint32_t expected_committed_tokens);
    [[nodiscard]] KvCacheError commitTokenReservation(KvTokenReservationId reservation_id);
    [[nodiscard]] KvCacheError rollbackTokenReservation(KvTokenReservationId reservation_id);
    [[nodiscard]] KvCacheError sealTail(RequestId request_id);
    [[nodiscard]] KvCacheError forkRequest(RequestId source_request_id, RequestId child_request_id);
    [[nodiscard]] KvCacheError releaseRequest(RequestId request_id);
    [[nodiscard]] std::optional<BlockTable> blockTable(RequestId request_id) const;
    [[nodiscard]] FixedPageManagerSnapshot snapshot() const;
    [[nodiscard]] bool checkInvariants() const;

private:
    // Per physical page: lifecycle state and sharing. The handle generation
    // is kept when a page is freed, so stale handles stay detectable.
    struct Page {
        PageState state{PageState::Free};
        std::uint32_t generation{0};
        std::uint16_t valid_tokens{0};
        std::uint32_t ref_count{0};
        RequestId owner{kInvalidRequestId};  // the one request that may write a Mutable page
    };

    // A reserved next token: exactly one of `target` (a new page, or the copy
    // of a sealed partial tail) and `in_place` (the request's own Mutable
    // tail) is set.
    struct Reservation {
        RequestId request{kInvalidRequestId};
        std::uint64_t table_version{0};
        BlockTable candidate{};
        PageHandle target{PageHandle::invalid()};
        PageHandle in_place{PageHandle::invalid()};
        PageHandle replaced_tail{PageHandle::invalid()};
    };

    [[nodiscard]] Page* page(PageHandle h) noexcept;
    [[nodiscard]] Page const* page(PageHandle h) const noexcept;
    [[nodiscard]] KvCacheError stage(std::uint16_t initial_valid, PageHandle& out);
    void unstage(std::vector<PageHandle> const& staged) noexcept;
    void markFree(Page& p) noexcept;
    [[nodiscard]] KvCacheError freePage(PageHandle h);
    [[nodiscard]] KvCacheError dropReference(PageHandle h);
    // A page that now backs `entry` of `owner`'s committed table.
    void publish(Page& p, std::uint16_t valid_tokens, RequestId owner) noexcept;
    [[nodiscard]] bool reserved(RequestId r) const noexcept { return by_request_.count(r) != 0; }
    [[nodiscard]] KvTokenReservationId nextReservationId();
    [[nodiscard]] bool consistent() const;

    std::uint16_t page_tokens_;
    PagePool pool_;
    std::vector<Page> pages_;
    std::unordered_map<RequestId, BlockTable> requests_;
    std::unordered_map<KvTokenReservationId, Reservation> reservations_;
    std::unordered_map<RequestId, KvTokenReservationId> by_request_;
    KvTokenReservationId next_reservation_{1};
    std::uint64_t peak_allocated_{0};
    mutable std::mutex mutex_;
};

} // namespace kimkvcache
