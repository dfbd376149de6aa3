// Fixed-page KV metadata runtime: one page kind, a configurable token
// capacity per page (Fixed-8/16/32/64), the strategy baseline the reference
// compares its two-pool runtime against
// (include/kim-kv/fixed/fixed_page_manager.h:30-166,
// src/fixed/fixed_page_manager.cpp, src/fixed/fixed_token_reservation.cpp).
//
// It is the single-pool configuration of the page-table engine that also
// runs KvCacheManager (paged_tables.h): create / append / reserve-commit-
// rollback / seal / fork / partial-tail COW / release with every page of
// size tokens_per_page; there is no promotion and there are no leases. Pages
// carry PageKind::Micro in block tables (the kind only names the pool), and
// table invariants are checked against tokens_per_page.
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
    std::uint16_t page_tokens_;
    TableEngine core_;
    mutable std::mutex mutex_;
};

} // namespace kimkvcache
