// FixedPageManager: the single-pool configuration of the page-table engine
// (paged_tables.h). Reference semantics: src/fixed/fixed_page_manager.cpp,
// src/fixed/fixed_token_reservation.cpp.
#include "fixed_page_manager.h"

#include <stdexcept>

namespace kimkvcache {

FixedPageManager::FixedPageManager(std::uint16_t tokens_per_page, std::uint32_t page_capacity)
    : page_tokens_(tokens_per_page != 0
              ? tokens_per_page
              : throw std::invalid_argument("fixed page token capacity must be greater than zero"))
    , core_(tokens_per_page, page_capacity, 0)
{
}

KvCacheError FixedPageManager::createRequest(RequestId request_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.create(request_id);
}

KvCacheError FixedPageManager::append(RequestId request_id, std::uint32_t token_count)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.append(request_id, token_count);
}

TokenReservationResult FixedPageManager::reserveToken(RequestId request_id,
    std::uint32_t expected_committed_tokens)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.reserve(request_id, expected_committed_tokens, false);
}

KvCacheError FixedPageManager::commitTokenReservation(KvTokenReservationId reservation_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.commit(reservation_id);
}

KvCacheError FixedPageManager::rollbackTokenReservation(KvTokenReservationId reservation_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.rollback(reservation_id);
}

KvCacheError FixedPageManager::sealTail(RequestId request_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.seal(request_id);
}

KvCacheError FixedPageManager::forkRequest(RequestId source_request_id, RequestId child_request_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.fork(source_request_id, child_request_id);
}

KvCacheError FixedPageManager::releaseRequest(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    if (core_.table(request_id) == nullptr) {
        return KvCacheError::RequestNotFound;
    }
    if (core_.pending(request_id)) {
        return KvCacheError::RequestConflict;
    }
    return core_.release(request_id);
}

std::optional<BlockTable> FixedPageManager::blockTable(RequestId request_id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    BlockTable const* t = core_.table(request_id);
    return t == nullptr ? std::nullopt : std::optional<BlockTable>(*t);
}

FixedPageManagerSnapshot FixedPageManager::snapshot() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    FixedPageManagerSnapshot s;
    s.request_count = core_.requestCount();
    s.pool = core_.slots(PageKind::Micro).pool.snapshot();
    s.successful_allocations = s.pool.successful_allocations;
    s.peak_allocated_pages = core_.peakAllocated();
    s.token_reservation_count = core_.reservationCount();
    return s;
}

bool FixedPageManager::checkInvariants() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    PageSlots const& pages = core_.slots(PageKind::Micro);
    ExpectedCounts expect(pages.size());
    return core_.auditTables(expect, nullptr) && core_.auditSlots(pages, expect);
}

} // namespace kimkvcache
