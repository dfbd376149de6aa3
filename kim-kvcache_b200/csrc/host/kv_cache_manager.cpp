// KvCacheManager: the two-pool configuration of the page-table engine
// (paged_tables.h) plus what only this runtime has: promotion of 8 sealed
// micro pages into one extent page, and page leases.
//
// Reference semantics: src/runtime/kv_cache_manager.cpp, kv_cache_append.cpp,
// token_reservation.cpp, kv_cache_lifecycle.cpp, promotion.cpp:80-457,
// page_lease.cpp:31-189, kv_cache_invariants.cpp.
#include "kv_cache_manager.h"

#include <algorithm>
#include <limits>
#include <utility>

namespace kimkvcache {

KvCacheManager::KvCacheManager(std::uint32_t micro_capacity, std::uint32_t extent_capacity)
    : core_(kMicroPageTokenCapacity, micro_capacity, extent_capacity)
{
}

bool KvCacheManager::promoting(RequestId request_id) const
{
    return std::any_of(promotions_.begin(), promotions_.end(),
        [request_id](auto const& p) { return p.second.request_id == request_id; });
}

// ---- delegated table operations ----------------------------------------------------------

KvCacheError KvCacheManager::createRequest(RequestId request_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.create(request_id);
}

KvCacheError KvCacheManager::append(RequestId request_id, std::uint32_t token_count)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.append(request_id, token_count);
}

TokenReservationResult KvCacheManager::reserveToken(RequestId request_id, std::uint32_t expected)
{
    std::lock_guard<std::mutex> lock(mutex_);
    // A prepared promotion holds the request's table version: no token may
    // be reserved until it is committed or rolled back.
    bool const busy = request_id != kInvalidRequestId && core_.table(request_id) != nullptr
        && promoting(request_id);
    return core_.reserve(request_id, expected, busy);
}

KvCacheError KvCacheManager::commitTokenReservation(KvTokenReservationId id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.commit(id);
}

KvCacheError KvCacheManager::rollbackTokenReservation(KvTokenReservationId id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.rollback(id);
}

KvCacheError KvCacheManager::sealTail(RequestId request_id)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.seal(request_id);
}

KvCacheError KvCacheManager::forkRequest(RequestId source, RequestId child)
{
    std::lock_guard<std::mutex> lock(mutex_);
    return core_.fork(source, child);
}

KvCacheError KvCacheManager::releaseRequest(RequestId request_id)
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
    // Pending promotions of the request are undone first, in the map's order.
    for (;;) {
        auto const p = std::find_if(promotions_.begin(), promotions_.end(),
            [request_id](auto const& e) { return e.second.request_id == request_id; });
        if (p == promotions_.end()) {
            break;
        }
        KvCacheError const err = undoPromotion(p->first);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    return core_.release(request_id);
}

std::optional<BlockTable> KvCacheManager::blockTable(RequestId request_id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    BlockTable const* t = core_.table(request_id);
    return t == nullptr ? std::nullopt : std::optional<BlockTable>(*t);
}

std::optional<PageMetadataSnapshot> KvCacheManager::pageMetadata(PageHandle handle) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    auto const [s, i] = core_.find(handle);
    if (s == nullptr) {
        return std::nullopt;
    }
    return PageMetadataSnapshot{handle, s->state[i], s->valid[i], s->refs[i], s->pins[i], s->readers[i],
        s->owner[i]};
}

KvCacheManagerSnapshot KvCacheManager::snapshot() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return KvCacheManagerSnapshot{core_.requestCount(), promotions_.size(), leases_.size(),
        core_.reservationCount(), core_.slots(PageKind::Micro).pool.snapshot(),
        core_.slots(PageKind::Extent).pool.snapshot()};
}

// ---- promotion -------------------------------------------------------------------------------

// Entries [first, first + 8) of `table` form a promotable run starting at
// logical token `begin`: full, sealed, unshared micro pages in order, each
// pinned exactly `pins` times (0 before prepare, 1 by the prepared
// promotion) and, when `expect` is given, exactly the prepared pages.
bool KvCacheManager::runEligible(BlockTable const& table, std::size_t first, std::uint32_t begin,
    std::array<PageHandle, kPromotionSourcePageCount> const* expect, std::uint32_t pins) const
{
    if (first > table.entries_.size() || table.entries_.size() - first < kPromotionSourcePageCount) {
        return false;
    }
    PageSlots const& micro = core_.slots(PageKind::Micro);
    for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
        MappingEntry const& m = table.entries_[first + k];
        std::uint64_t const at = std::uint64_t(begin) + k * kMicroPageTokenCapacity;
        if (at > std::numeric_limits<std::uint32_t>::max() || m.logical_token_begin != at
            || m.kind != PageKind::Micro || m.valid_tokens != kMicroPageTokenCapacity
            || (expect != nullptr && m.handle != (*expect)[k])) {
            return false;
        }
        std::int64_t const i = micro.slotOf(m.handle);
        if (i < 0 || micro.state[i] != PageState::Sealed || micro.valid[i] != kMicroPageTokenCapacity
            || micro.refs[i] != 1 || micro.pins[i] != pins || micro.owner[i] != kInvalidRequestId
            || micro.pool.validate(m.handle) != PagePoolError::None) {
            return false;
        }
    }
    return true;
}

PromotionPrepareResult KvCacheManager::preparePromotion(RequestId request_id, std::uint32_t begin)
{
    PromotionPrepareResult r;
    r.request_id = request_id;
    r.logical_token_begin = begin;
    if (request_id == kInvalidRequestId) {
        r.error = KvCacheError::InvalidArgument;
        return r;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    BlockTable const* t = core_.table(request_id);
    if (t == nullptr) {
        r.error = KvCacheError::RequestNotFound;
        return r;
    }
    if (core_.pending(request_id)) {
        r.error = KvCacheError::RequestConflict;
        return r;
    }
    if (t->version_ == std::numeric_limits<std::uint64_t>::max()) {
        r.error = KvCacheError::PromotionConflict;
        return r;
    }
    auto const at = std::find_if(t->entries_.begin(), t->entries_.end(),
        [begin](MappingEntry const& m) { return m.logical_token_begin == begin; });
    std::size_t const first = static_cast<std::size_t>(at - t->entries_.begin());
    if (at == t->entries_.end() || !runEligible(*t, first, begin, nullptr, 0)) {
        r.error = KvCacheError::PromotionNotEligible;
        return r;
    }
    Promotion p{request_id, t->version_, begin, first, {}, PageHandle::invalid()};
    for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
        p.sources[k] = t->entries_[first + k].handle;
    }
    if ((r.error = core_.stage(PageKind::Extent, kExtentPageTokenCapacity, p.target)) != KvCacheError::None) {
        return r;
    }
    PromotionId const id = promotion_ids_.next(promotions_);
    if (id == kInvalidPromotionId) {
        static_cast<void>(core_.retire(p.target));
        r.error = KvCacheError::InternalInvariantViolation;
        return r;
    }
    PageSlots& micro = core_.slots(PageKind::Micro);
    for (PageHandle const h : p.sources) {
        ++micro.pins[h.slot];
    }
    r.promotion_id = id;
    r.source_handles = p.sources;
    r.target_handle = p.target;
    promotions_.emplace(id, p);
    return r;
}

// Returns the staged target and unpins the sources; a source whose last
// table reference went while it was pinned leaves now.
KvCacheError KvCacheManager::undoPromotion(PromotionId id)
{
    auto const f = promotions_.find(id);
    if (f == promotions_.end()) {
        return KvCacheError::PromotionNotFound;
    }
    Promotion const& p = f->second;
    PageSlots& micro = core_.slots(PageKind::Micro);
    PageSlots const& extent = core_.slots(PageKind::Extent);
    std::int64_t const ti = extent.slotOf(p.target);
    bool intact = ti >= 0 && extent.state[ti] == PageState::CopyTarget
        && extent.valid[ti] == kExtentPageTokenCapacity && extent.refs[ti] == 0 && extent.pins[ti] == 0
        && extent.owner[ti] == kInvalidRequestId && extent.pool.validate(p.target) == PagePoolError::None;
    for (PageHandle const h : p.sources) {
        std::int64_t const i = micro.slotOf(h);
        intact = intact && i >= 0
            && (micro.state[i] == PageState::Sealed || micro.state[i] == PageState::Retiring)
            && micro.valid[i] == kMicroPageTokenCapacity && micro.pins[i] == 1
            && micro.owner[i] == kInvalidRequestId && micro.pool.validate(h) == PagePoolError::None;
    }
    if (!intact) {
        return KvCacheError::InternalInvariantViolation;
    }
    KvCacheError err = core_.retire(p.target);
    for (std::size_t k = 0; err == KvCacheError::None && k < kPromotionSourcePageCount; ++k) {
        std::uint32_t const i = p.sources[k].slot;
        --micro.pins[i];
        if (micro.refs[i] == 0) {
            err = core_.retire(p.sources[k]);
        }
    }
    if (err == KvCacheError::None) {
        promotions_.erase(f);
    }
    return err;
}

KvCacheError KvCacheManager::rollbackPromotion(PromotionId id)
{
    if (id == kInvalidPromotionId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    return undoPromotion(id);
}

KvCacheError KvCacheManager::commitPromotion(PromotionId id)
{
    if (id == kInvalidPromotionId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto const f = promotions_.find(id);
    if (f == promotions_.end()) {
        return KvCacheError::PromotionNotFound;
    }
    Promotion const p = f->second;
    BlockTable* t = core_.table(p.request_id);
    PageSlots& extent = core_.slots(PageKind::Extent);
    std::int64_t const ti = extent.slotOf(p.target);
    // The table must still be the prepared version, with the run in place,
    // and the target untouched; otherwise the promotion is abandoned (its
    // own undo error wins over the conflict).
    bool ok = t != nullptr && t->version_ == p.prepared_version
        && t->version_ != std::numeric_limits<std::uint64_t>::max() && ti >= 0
        && extent.state[ti] == PageState::CopyTarget && extent.valid[ti] == kExtentPageTokenCapacity
        && extent.refs[ti] == 0 && extent.pins[ti] == 0 && extent.readers[ti] == 0
        && extent.owner[ti] == kInvalidRequestId && extent.pool.validate(p.target) == PagePoolError::None
        && runEligible(*t, p.first_entry, p.logical_token_begin, &p.sources, 1);
    BlockTable next;
    if (ok) {
        next = *t;
        auto const run = next.entries_.begin() + static_cast<std::ptrdiff_t>(p.first_entry);
        *run = MappingEntry{p.logical_token_begin, kExtentPageTokenCapacity, PageKind::Extent, p.target};
        next.entries_.erase(run + 1, run + static_cast<std::ptrdiff_t>(kPromotionSourcePageCount));
        next.version_ = t->version_ + 1;
        if (!next.checkInvariants()) {
            KvCacheError const undone = undoPromotion(id);
            return undone == KvCacheError::None ? KvCacheError::InternalInvariantViolation : undone;
        }
    } else {
        KvCacheError const undone = undoPromotion(id);
        return undone == KvCacheError::None ? KvCacheError::PromotionConflict : undone;
    }
    // No-fail from here: the extent replaces the run, the sources drop out.
    *t = std::move(next);
    extent.state[ti] = PageState::Sealed;
    extent.refs[ti] = 1;
    PageSlots& micro = core_.slots(PageKind::Micro);
    for (PageHandle const h : p.sources) {
        --micro.refs[h.slot];
        --micro.pins[h.slot];
        KvCacheError const err = core_.retire(h);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    promotions_.erase(id);
    return KvCacheError::None;
}

std::optional<PromotionTransactionSnapshot> KvCacheManager::promotionTransaction(PromotionId id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    auto const f = promotions_.find(id);
    if (f == promotions_.end()) {
        return std::nullopt;
    }
    Promotion const& p = f->second;
    return PromotionTransactionSnapshot{id, p.request_id, p.prepared_version, p.logical_token_begin,
        p.sources, p.target};
}

// ---- leases ------------------------------------------------------------------------------------

// Pins every page of `handles` as read by device work in flight. `table`
// (when given) and the handles are echoed in the result.
PageLeaseAcquireResult KvCacheManager::lease(std::vector<PageHandle> handles, BlockTable const* table)
{
    PageLeaseAcquireResult r;
    for (PageHandle const h : handles) {
        auto const [s, i] = core_.find(h);
        if (s == nullptr || s->state[i] == PageState::Free || s->state[i] == PageState::Retiring
            || s->readers[i] == std::numeric_limits<std::uint32_t>::max()) {
            r.error = KvCacheError::InvalidState;
            return r;
        }
    }
    PageLeaseId const id = lease_ids_.next(leases_);
    if (id == kInvalidPageLeaseId) {
        r.error = KvCacheError::InternalInvariantViolation;
        return r;
    }
    for (PageHandle const h : handles) {
        auto const [s, i] = core_.find(h);
        ++s->readers[i];
    }
    if (table != nullptr) {
        r.table = *table;
        r.handles = handles;
    }
    leases_.emplace(id, std::move(handles));
    r.lease_id = id;
    return r;
}

PageLeaseAcquireResult KvCacheManager::acquireRequestReadLease(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return PageLeaseAcquireResult{KvCacheError::InvalidArgument, kInvalidPageLeaseId, {}, {}};
    }
    std::lock_guard<std::mutex> lock(mutex_);
    BlockTable const* t = core_.table(request_id);
    if (t == nullptr) {
        return PageLeaseAcquireResult{KvCacheError::RequestNotFound, kInvalidPageLeaseId, {}, {}};
    }
    std::vector<PageHandle> pages;
    pages.reserve(t->entries_.size());
    for (MappingEntry const& m : t->entries_) {
        pages.push_back(m.handle);
    }
    return lease(std::move(pages), t);
}

PageLeaseAcquireResult KvCacheManager::acquirePromotionIoLease(PromotionId id)
{
    if (id == kInvalidPromotionId) {
        return PageLeaseAcquireResult{KvCacheError::InvalidArgument, kInvalidPageLeaseId, {}, {}};
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto const f = promotions_.find(id);
    if (f == promotions_.end()) {
        return PageLeaseAcquireResult{KvCacheError::PromotionNotFound, kInvalidPageLeaseId, {}, {}};
    }
    std::vector<PageHandle> pages(f->second.sources.begin(), f->second.sources.end());
    pages.push_back(f->second.target);
    BlockTable const no_table;
    return lease(std::move(pages), &no_table);
}

PageLeaseAcquireResult KvCacheManager::acquireTokenReservationLease(KvTokenReservationId id)
{
    return leaseReservation(id, true);
}

PageLeaseAcquireResult KvCacheManager::acquireTokenReservationPin(KvTokenReservationId id)
{
    return leaseReservation(id, false);
}

// The reserved table's pages, plus the sealed tail a copy-on-write reads from.
PageLeaseAcquireResult KvCacheManager::leaseReservation(KvTokenReservationId id, bool describe)
{
    if (id == kInvalidKvTokenReservationId) {
        return PageLeaseAcquireResult{KvCacheError::InvalidArgument, kInvalidPageLeaseId, {}, {}};
    }
    std::lock_guard<std::mutex> lock(mutex_);
    PendingToken const* p = core_.reservation(id);
    if (p == nullptr) {
        return PageLeaseAcquireResult{KvCacheError::TokenReservationNotFound, kInvalidPageLeaseId, {}, {}};
    }
    std::vector<PageHandle> pages;
    pages.reserve(p->edit.table.entries_.size() + 1);
    for (MappingEntry const& m : p->edit.table.entries_) {
        pages.push_back(m.handle);
    }
    if (p->edit.replaced.isStructurallyValid()) {
        pages.push_back(p->edit.replaced);
    }
    return lease(std::move(pages), describe ? &p->edit.table : nullptr);
}

KvCacheError KvCacheManager::releasePageLease(PageLeaseId lease_id)
{
    if (lease_id == kInvalidPageLeaseId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto const f = leases_.find(lease_id);
    if (f == leases_.end()) {
        return KvCacheError::InvalidState;
    }
    for (PageHandle const h : f->second) {
        auto const [s, i] = core_.find(h);
        if (s == nullptr || s->state[i] == PageState::Free || s->readers[i] == 0) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    std::vector<PageHandle> const pages = std::move(f->second);
    leases_.erase(f);
    for (PageHandle const h : pages) {
        auto const [s, i] = core_.find(h);
        --s->readers[i];
        // A page that only the lease kept alive leaves with it.
        if (s->state[i] == PageState::Retiring && s->refs[i] == 0 && s->pins[i] == 0 && s->readers[i] == 0) {
            KvCacheError const err = core_.retire(h);
            if (err != KvCacheError::None) {
                return err;
            }
        }
    }
    return KvCacheError::None;
}

// ---- invariants --------------------------------------------------------------------------------

bool KvCacheManager::checkInvariants() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    PageSlots const& micro = core_.slots(PageKind::Micro);
    PageSlots const& extent = core_.slots(PageKind::Extent);
    ExpectedCounts xm(micro.size());
    ExpectedCounts xe(extent.size());
    if (!core_.auditTables(xm, &xe)) {
        return false;
    }
    // Promotions: a staged extent target each, and one pin on each source of
    // a run that is still in place in the request's table.
    for (auto const& [id, p] : promotions_) {
        BlockTable const* t = core_.table(p.request_id);
        std::int64_t const ti = extent.slotOf(p.target);
        if (id == kInvalidPromotionId || t == nullptr || p.prepared_version > t->version_ || ti < 0
            || xe.staged[ti] != 0 || extent.state[ti] != PageState::CopyTarget) {
            return false;
        }
        xe.staged[ti] = 1;
        auto const at = std::find_if(t->entries_.begin(), t->entries_.end(),
            [&p](MappingEntry const& m) { return m.handle == p.sources[0]; });
        std::size_t const first = static_cast<std::size_t>(at - t->entries_.begin());
        if (at == t->entries_.end() || first + kPromotionSourcePageCount > t->entries_.size()) {
            return false;
        }
        for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
            MappingEntry const& m = t->entries_[first + k];
            std::int64_t const i = micro.slotOf(p.sources[k]);
            if (i < 0 || m.handle != p.sources[k] || m.kind != PageKind::Micro
                || m.valid_tokens != kMicroPageTokenCapacity
                || m.logical_token_begin != std::uint64_t(p.logical_token_begin) + k * kMicroPageTokenCapacity
                || micro.state[i] != PageState::Sealed || xm.pins[i] != 0) {
                return false;
            }
            xm.pins[i] = 1;
        }
    }
    for (auto const& [id, pages] : leases_) {
        if (id == kInvalidPageLeaseId) {
            return false;
        }
        for (PageHandle const h : pages) {
            auto const [s, i] = core_.find(h);
            ExpectedCounts& x = h.kind == PageKind::Extent ? xe : xm;
            if (s == nullptr || s->state[i] == PageState::Free
                || x.readers[i] == std::numeric_limits<std::uint32_t>::max()) {
                return false;
            }
            ++x.readers[i];
        }
    }
    return core_.auditSlots(micro, xm) && core_.auditSlots(extent, xe);
}

} // namespace kimkvcache
