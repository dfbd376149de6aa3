// KvCacheManager: promotion (8 sealed micro pages -> 1 extent page), page
// leases and the invariant auditor.
// Reference semantics: src/runtime/promotion.cpp:12-480,
// src/runtime/page_lease.cpp:8-189, src/runtime/kv_cache_invariants.cpp:10-495.
#include "kv_cache_manager.h"

#include <algorithm>
#include <limits>
#include <utility>

namespace kimkvcache {

KvCacheError KvCacheManager::stageExtent(PageHandle& out)
{
    PageAllocationResult const got = extent_pool_.allocate();
    if (!got.ok()) {
        return got.error == PagePoolError::Exhausted ? KvCacheError::ResourceExhausted
                                                     : KvCacheError::InternalInvariantViolation;
    }
    out = got.handle;
    if (out.slot >= extent_pages_.size()) {
        static_cast<void>(extent_pool_.release(out));
        out = PageHandle::invalid();
        return KvCacheError::InternalInvariantViolation;
    }
    Page& p = extent_pages_[out.slot];
    if (p.state != PageState::Free || p.ref_count != 0 || p.promotion_pins != 0
        || p.inflight_readers != 0) {
        static_cast<void>(extent_pool_.release(out));
        out = PageHandle::invalid();
        return KvCacheError::InternalInvariantViolation;
    }
    p = Page{PageState::CopyTarget, out.generation, kExtentPageTokenCapacity, 0, 0, 0,
        kInvalidRequestId};
    return KvCacheError::None;
}

PromotionPrepareResult KvCacheManager::preparePromotion(
    RequestId request_id, std::uint32_t logical_token_begin)
{
    PromotionPrepareResult result;
    result.request_id = request_id;
    result.logical_token_begin = logical_token_begin;
    if (request_id == kInvalidRequestId) {
        result.error = KvCacheError::InvalidArgument;
        return result;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        result.error = KvCacheError::RequestNotFound;
        return result;
    }
    if (hasReservation(request_id)) {
        result.error = KvCacheError::RequestConflict;
        return result;
    }
    BlockTable const& table = found->second;
    if (table.version_ == std::numeric_limits<std::uint64_t>::max()) {
        result.error = KvCacheError::PromotionConflict;
        return result;
    }
    auto const first = std::find_if(table.entries_.begin(), table.entries_.end(),
        [logical_token_begin](MappingEntry const& e) {
            return e.logical_token_begin == logical_token_begin;
        });
    std::size_t const index = static_cast<std::size_t>(first - table.entries_.begin());
    if (first == table.entries_.end()
        || table.entries_.size() - index < kPromotionSourcePageCount) {
        result.error = KvCacheError::PromotionNotEligible;
        return result;
    }
    // Eligible run: 8 consecutive full, sealed, unshared, unpinned micro pages.
    std::array<PageHandle, kPromotionSourcePageCount> sources{};
    for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
        MappingEntry const& entry = table.entries_[index + k];
        std::uint64_t const expected_begin =
            static_cast<std::uint64_t>(logical_token_begin) + k * kMicroPageTokenCapacity;
        Page const* p = page(entry.handle);
        if (expected_begin > std::numeric_limits<std::uint32_t>::max()
            || entry.logical_token_begin != expected_begin || entry.kind != PageKind::Micro
            || entry.handle.kind != PageKind::Micro
            || entry.valid_tokens != kMicroPageTokenCapacity || p == nullptr
            || p->state != PageState::Sealed || p->valid_tokens != kMicroPageTokenCapacity
            || p->ref_count != 1 || p->promotion_pins != 0
            || p->mutable_owner != kInvalidRequestId
            || micro_pool_.validate(entry.handle) != PagePoolError::None) {
            result.error = KvCacheError::PromotionNotEligible;
            return result;
        }
        sources[k] = entry.handle;
    }
    PageHandle target = PageHandle::invalid();
    KvCacheError const staged = stageExtent(target);
    if (staged != KvCacheError::None) {
        result.error = staged;
        return result;
    }
    PromotionId const id = nextFreeId(next_promotion_id_, promotions_);
    if (id == kInvalidPromotionId
        || !promotions_.emplace(id, Promotion{id, request_id, table.version_,
               logical_token_begin, index, sources, target}).second) {
        static_cast<void>(retireOrFree(target));
        result.error = KvCacheError::InternalInvariantViolation;
        return result;
    }
    for (PageHandle const source : sources) {
        ++page(source)->promotion_pins;
    }
    result.error = KvCacheError::None;
    result.promotion_id = id;
    result.source_handles = sources;
    result.target_handle = target;
    return result;
}

KvCacheError KvCacheManager::rollbackPromotionLocked(PromotionId id)
{
    auto found = promotions_.find(id);
    if (found == promotions_.end()) {
        return KvCacheError::PromotionNotFound;
    }
    Promotion const& promotion = found->second;
    Page const* target = page(promotion.target);
    if (target == nullptr || target->state != PageState::CopyTarget
        || target->valid_tokens != kExtentPageTokenCapacity || target->ref_count != 0
        || target->promotion_pins != 0 || target->mutable_owner != kInvalidRequestId
        || extent_pool_.validate(promotion.target) != PagePoolError::None) {
        return KvCacheError::InternalInvariantViolation;
    }
    for (PageHandle const source : promotion.sources) {
        Page const* p = page(source);
        if (p == nullptr
            || (p->state != PageState::Sealed && p->state != PageState::Retiring)
            || p->valid_tokens != kMicroPageTokenCapacity || p->promotion_pins != 1
            || p->mutable_owner != kInvalidRequestId
            || micro_pool_.validate(source) != PagePoolError::None) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    KvCacheError const dropped = retireOrFree(promotion.target);
    if (dropped != KvCacheError::None) {
        return dropped;
    }
    for (PageHandle const source : promotion.sources) {
        Page* p = page(source);
        --p->promotion_pins;
        if (p->ref_count == 0) {
            KvCacheError const error = retireOrFree(source);
            if (error != KvCacheError::None) {
                return error;
            }
        }
    }
    promotions_.erase(found);
    return KvCacheError::None;
}

KvCacheError KvCacheManager::rollbackPromotion(PromotionId id)
{
    if (id == kInvalidPromotionId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    return rollbackPromotionLocked(id);
}

KvCacheError KvCacheManager::rollbackRequestPromotionsLocked(RequestId request_id)
{
    for (;;) {
        auto const found = std::find_if(promotions_.begin(), promotions_.end(),
            [request_id](auto const& p) { return p.second.request_id == request_id; });
        if (found == promotions_.end()) {
            return KvCacheError::None;
        }
        KvCacheError const error = rollbackPromotionLocked(found->first);
        if (error != KvCacheError::None) {
            return error;
        }
    }
}

KvCacheError KvCacheManager::commitPromotion(PromotionId id)
{
    if (id == kInvalidPromotionId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = promotions_.find(id);
    if (found == promotions_.end()) {
        return KvCacheError::PromotionNotFound;
    }
    Promotion const promotion = found->second;
    // Any failed check abandons the promotion; its own rollback error wins.
    auto abandon = [this, id](KvCacheError error) {
        KvCacheError const rolled = rollbackPromotionLocked(id);
        return rolled == KvCacheError::None ? error : rolled;
    };
    auto request = requests_.find(promotion.request_id);
    if (request == requests_.end()) {
        return abandon(KvCacheError::PromotionConflict);
    }
    BlockTable& table = request->second;
    if (table.version_ != promotion.prepared_version
        || promotion.source_entry_index > table.entries_.size()
        || table.entries_.size() - promotion.source_entry_index < kPromotionSourcePageCount
        || table.version_ == std::numeric_limits<std::uint64_t>::max()) {
        return abandon(KvCacheError::PromotionConflict);
    }
    Page* target = page(promotion.target);
    if (target == nullptr || target->state != PageState::CopyTarget
        || target->valid_tokens != kExtentPageTokenCapacity || target->ref_count != 0
        || target->promotion_pins != 0 || target->inflight_readers != 0
        || target->mutable_owner != kInvalidRequestId
        || extent_pool_.validate(promotion.target) != PagePoolError::None) {
        return abandon(KvCacheError::PromotionConflict);
    }
    for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
        MappingEntry const& entry = table.entries_[promotion.source_entry_index + k];
        PageHandle const source = promotion.sources[k];
        Page const* p = page(source);
        std::uint64_t const expected_begin =
            static_cast<std::uint64_t>(promotion.logical_token_begin)
            + k * kMicroPageTokenCapacity;
        if (expected_begin > std::numeric_limits<std::uint32_t>::max()
            || entry.logical_token_begin != expected_begin || entry.kind != PageKind::Micro
            || entry.valid_tokens != kMicroPageTokenCapacity || entry.handle != source
            || p == nullptr || p->state != PageState::Sealed
            || p->valid_tokens != kMicroPageTokenCapacity || p->ref_count != 1
            || p->promotion_pins != 1 || p->mutable_owner != kInvalidRequestId
            || micro_pool_.validate(source) != PagePoolError::None) {
            return abandon(KvCacheError::PromotionConflict);
        }
    }
    BlockTable candidate = table;
    auto const first = candidate.entries_.begin()
        + static_cast<std::ptrdiff_t>(promotion.source_entry_index);
    *first = MappingEntry{promotion.logical_token_begin, kExtentPageTokenCapacity,
        PageKind::Extent, promotion.target};
    candidate.entries_.erase(first + 1,
        first + static_cast<std::ptrdiff_t>(kPromotionSourcePageCount));
    candidate.version_ = table.version_ + 1;
    if (!candidate.checkInvariants()) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    // No-fail section: publish the new mapping, then retire the sources.
    table = std::move(candidate);
    target->state = PageState::Sealed;
    target->ref_count = 1;
    for (PageHandle const source : promotion.sources) {
        Page* p = page(source);
        --p->ref_count;
        --p->promotion_pins;
        KvCacheError const error = retireOrFree(source);
        if (error != KvCacheError::None) {
            return error;
        }
    }
    promotions_.erase(id);
    return KvCacheError::None;
}

std::optional<PromotionTransactionSnapshot> KvCacheManager::promotionTransaction(
    PromotionId id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = promotions_.find(id);
    if (found == promotions_.end()) {
        return std::nullopt;
    }
    Promotion const& p = found->second;
    return PromotionTransactionSnapshot{p.id, p.request_id, p.prepared_version,
        p.logical_token_begin, p.sources, p.target};
}

PageLeaseAcquireResult KvCacheManager::pinPages(std::vector<PageHandle> handles, BlockTable const* table)
{
    PageLeaseAcquireResult result;
    for (PageHandle const handle : handles) {
        Page const* p = page(handle);
        if (p == nullptr || p->state == PageState::Free || p->state == PageState::Retiring
            || p->inflight_readers == std::numeric_limits<std::uint32_t>::max()) {
            result.error = KvCacheError::InvalidState;
            return result;
        }
    }
    PageLeaseId const id = nextFreeId(next_lease_id_, leases_);
    if (id == kInvalidPageLeaseId) {
        result.error = KvCacheError::InternalInvariantViolation;
        return result;
    }
    if (table != nullptr) {  // callers that keep only the id skip both copies
        result.table = *table;
        result.handles = handles;
    }
    auto const inserted = leases_.emplace(id, Lease{id, std::move(handles)});
    if (!inserted.second) {
        result.error = KvCacheError::InternalInvariantViolation;
        return result;
    }
    for (PageHandle const handle : inserted.first->second.handles) {
        ++page(handle)->inflight_readers;
    }
    result.error = KvCacheError::None;
    result.lease_id = id;
    return result;
}

PageLeaseAcquireResult KvCacheManager::acquireRequestReadLease(RequestId request_id)
{
    PageLeaseAcquireResult result;
    if (request_id == kInvalidRequestId) {
        result.error = KvCacheError::InvalidArgument;
        return result;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        result.error = KvCacheError::RequestNotFound;
        return result;
    }
    std::vector<PageHandle> handles;
    handles.reserve(found->second.entries_.size());
    for (MappingEntry const& entry : found->second.entries_) {
        handles.push_back(entry.handle);
    }
    return pinPages(std::move(handles), &found->second);
}

PageLeaseAcquireResult KvCacheManager::acquirePromotionIoLease(PromotionId id)
{
    PageLeaseAcquireResult result;
    if (id == kInvalidPromotionId) {
        result.error = KvCacheError::InvalidArgument;
        return result;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = promotions_.find(id);
    if (found == promotions_.end()) {
        result.error = KvCacheError::PromotionNotFound;
        return result;
    }
    std::vector<PageHandle> handles(found->second.sources.begin(), found->second.sources.end());
    handles.push_back(found->second.target);
    BlockTable const none;
    return pinPages(std::move(handles), &none);
}

PageLeaseAcquireResult KvCacheManager::acquireTokenReservationLease(KvTokenReservationId id)
{
    return pinTokenReservation(id, true);
}

PageLeaseAcquireResult KvCacheManager::acquireTokenReservationPin(KvTokenReservationId id)
{
    return pinTokenReservation(id, false);
}

PageLeaseAcquireResult KvCacheManager::pinTokenReservation(KvTokenReservationId id, bool describe)
{
    PageLeaseAcquireResult result;
    if (id == kInvalidKvTokenReservationId) {
        result.error = KvCacheError::InvalidArgument;
        return result;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = reservations_.find(id);
    if (found == reservations_.end()) {
        result.error = KvCacheError::TokenReservationNotFound;
        return result;
    }
    Reservation const& r = found->second;
    std::vector<PageHandle> handles;
    handles.reserve(r.candidate.entries_.size() + 1);
    for (MappingEntry const& entry : r.candidate.entries_) {
        handles.push_back(entry.handle);
    }
    if (r.replaced_sealed_tail.isStructurallyValid()) {
        handles.push_back(r.replaced_sealed_tail);  // COW source stays readable
    }
    return pinPages(std::move(handles), describe ? &r.candidate : nullptr);
}

KvCacheError KvCacheManager::releasePageLease(PageLeaseId lease_id)
{
    if (lease_id == kInvalidPageLeaseId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = leases_.find(lease_id);
    if (found == leases_.end()) {
        return KvCacheError::InvalidState;
    }
    for (PageHandle const handle : found->second.handles) {
        Page const* p = page(handle);
        if (p == nullptr || p->state == PageState::Free || p->inflight_readers == 0) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    std::vector<PageHandle> const handles = std::move(found->second.handles);
    leases_.erase(found);
    for (PageHandle const handle : handles) {
        Page* p = page(handle);
        --p->inflight_readers;
        if (p->state == PageState::Retiring && p->ref_count == 0 && p->promotion_pins == 0
            && p->inflight_readers == 0) {
            KvCacheError const error = retireOrFree(handle);
            if (error != KvCacheError::None) {
                return error;
            }
        }
    }
    return KvCacheError::None;
}

// ---------------------------------------------------------------------------
// Invariant audit: recount references, pins, readers and staged targets from
// the tables/transactions/leases and compare with every slot's runtime state.

struct KvCacheManager::Audit final {
    struct PerKind {
        std::vector<std::uint32_t> refs, pins, readers;
        std::vector<std::uint8_t> targets;
        explicit PerKind(std::size_t n) : refs(n, 0), pins(n, 0), readers(n, 0), targets(n, 0) {}
    };
    PerKind micro;
    PerKind extent;
    Audit(std::size_t m, std::size_t e) : micro(m), extent(e) {}
    PerKind& of(PageKind kind) { return kind == PageKind::Micro ? micro : extent; }
    PerKind const& of(PageKind kind) const { return kind == PageKind::Micro ? micro : extent; }
};

bool KvCacheManager::checkInvariants() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return auditLocked();
}

bool KvCacheManager::auditLocked() const
{
    if (!micro_pool_.checkInvariants() || !extent_pool_.checkInvariants()) {
        return false;
    }
    Audit audit(micro_pages_.size(), extent_pages_.size());
    return auditRequests(audit) && auditPromotions(audit) && auditReservations(audit)
        && auditLeases(audit) && auditPool(PageKind::Micro, audit)
        && auditPool(PageKind::Extent, audit);
}

bool KvCacheManager::auditRequests(Audit& audit) const
{
    constexpr std::uint32_t kMax = std::numeric_limits<std::uint32_t>::max();
    for (auto const& [request_id, table] : requests_) {
        if (request_id == kInvalidRequestId || !table.checkInvariants()) {
            return false;
        }
        for (std::size_t i = 0; i < table.entries_.size(); ++i) {
            MappingEntry const& entry = table.entries_[i];
            Page const* p = page(entry.handle);
            if (p == nullptr || p->state == PageState::Free || p->state == PageState::CopyTarget
                || p->state == PageState::Retiring || p->valid_tokens != entry.valid_tokens
                || p->ref_count == 0) {
                return false;
            }
            if (p->state == PageState::Mutable) {
                if (i + 1 != table.entries_.size() || entry.kind != PageKind::Micro
                    || p->ref_count != 1 || p->mutable_owner != request_id
                    || p->valid_tokens == 0 || p->valid_tokens >= kMicroPageTokenCapacity) {
                    return false;
                }
            } else if (p->state != PageState::Sealed || p->mutable_owner != kInvalidRequestId) {
                return false;
            }
            auto& refs = audit.of(entry.kind).refs;
            if (entry.handle.slot >= refs.size() || refs[entry.handle.slot] == kMax) {
                return false;
            }
            ++refs[entry.handle.slot];
        }
    }
    return true;
}

bool KvCacheManager::auditPromotions(Audit& audit) const
{
    for (auto const& [id, promotion] : promotions_) {
        if (id == kInvalidPromotionId || promotion.id != id
            || promotion.request_id == kInvalidRequestId
            || promotion.target.kind != PageKind::Extent) {
            return false;
        }
        auto request = requests_.find(promotion.request_id);
        if (request == requests_.end()) {
            return false;
        }
        BlockTable const& table = request->second;
        if (promotion.prepared_version > table.version_) {
            return false;
        }
        Page const* target = page(promotion.target);
        auto& targets = audit.extent.targets;
        if (target == nullptr || target->state != PageState::CopyTarget
            || target->valid_tokens != kExtentPageTokenCapacity || target->ref_count != 0
            || target->promotion_pins != 0 || target->mutable_owner != kInvalidRequestId
            || promotion.target.slot >= targets.size() || targets[promotion.target.slot] != 0) {
            return false;
        }
        targets[promotion.target.slot] = 1;
        auto const first = std::find_if(table.entries_.begin(), table.entries_.end(),
            [&promotion](MappingEntry const& e) { return e.handle == promotion.sources[0]; });
        if (first == table.entries_.end()) {
            return false;
        }
        std::size_t const index = static_cast<std::size_t>(first - table.entries_.begin());
        if (table.entries_.size() - index < kPromotionSourcePageCount) {
            return false;
        }
        auto& pins = audit.micro.pins;
        for (std::size_t k = 0; k < kPromotionSourcePageCount; ++k) {
            PageHandle const source = promotion.sources[k];
            MappingEntry const& entry = table.entries_[index + k];
            Page const* p = page(source);
            std::uint64_t const expected_begin =
                static_cast<std::uint64_t>(promotion.logical_token_begin)
                + k * kMicroPageTokenCapacity;
            if (expected_begin > std::numeric_limits<std::uint32_t>::max()
                || source.kind != PageKind::Micro || entry.handle != source
                || entry.kind != PageKind::Micro || entry.logical_token_begin != expected_begin
                || entry.valid_tokens != kMicroPageTokenCapacity || p == nullptr
                || p->state != PageState::Sealed || p->valid_tokens != kMicroPageTokenCapacity
                || p->ref_count == 0 || p->promotion_pins == 0
                || p->mutable_owner != kInvalidRequestId || source.slot >= pins.size()
                || pins[source.slot] != 0) {
                return false;
            }
            pins[source.slot] = 1;
        }
    }
    return true;
}

bool KvCacheManager::auditReservations(Audit& audit) const
{
    if (request_reservation_.size() != reservations_.size()) {
        return false;
    }
    for (auto const& [id, r] : reservations_) {
        if (id == kInvalidKvTokenReservationId || r.id != id
            || r.request_id == kInvalidRequestId || !r.candidate.checkInvariants()) {
            return false;
        }
        auto request = requests_.find(r.request_id);
        auto owned = request_reservation_.find(r.request_id);
        if (request == requests_.end() || owned == request_reservation_.end()
            || owned->second != id) {
            return false;
        }
        BlockTable const& before = request->second;
        if (before.version() != r.prepared_version
            || r.candidate.version() != before.version() + 1
            || r.candidate.tokenCount() != before.tokenCount() + 1) {
            return false;
        }
        // Exactly one of: a staged target page, or growth of the mutable tail.
        if (r.staged_target.isStructurallyValid() == r.existing_mutable.isStructurallyValid()) {
            return false;
        }
        if (r.staged_target.isStructurallyValid()) {
            Page const* target = page(r.staged_target);
            auto& targets = audit.micro.targets;
            if (target == nullptr || target->state != PageState::CopyTarget
                || target->ref_count != 0 || target->promotion_pins != 0
                || target->mutable_owner != kInvalidRequestId
                || r.staged_target.slot >= targets.size() || targets[r.staged_target.slot] != 0) {
                return false;
            }
            std::uint16_t const expected_tokens = r.replaced_sealed_tail.isStructurallyValid()
                ? static_cast<std::uint16_t>(r.candidate.entries().back().valid_tokens - 1) : 0;
            if (target->valid_tokens != expected_tokens) {
                return false;
            }
            targets[r.staged_target.slot] = 1;
        }
        if (r.existing_mutable.isStructurallyValid()) {
            Page const* p = page(r.existing_mutable);
            if (p == nullptr || p->state != PageState::Mutable || p->ref_count != 1
                || p->mutable_owner != r.request_id || before.entries().empty()
                || before.entries().back().handle != r.existing_mutable) {
                return false;
            }
        }
        if (r.replaced_sealed_tail.isStructurallyValid()) {
            Page const* p = page(r.replaced_sealed_tail);
            if (p == nullptr || p->state != PageState::Sealed || p->ref_count == 0
                || before.entries().empty()
                || before.entries().back().handle != r.replaced_sealed_tail) {
                return false;
            }
        }
    }
    return true;
}

bool KvCacheManager::auditLeases(Audit& audit) const
{
    for (auto const& [id, lease] : leases_) {
        if (id == kInvalidPageLeaseId || lease.id != id) {
            return false;
        }
        for (PageHandle const handle : lease.handles) {
            Page const* p = page(handle);
            auto& readers = audit.of(handle.kind).readers;
            if (p == nullptr || p->state == PageState::Free || p->inflight_readers == 0
                || handle.slot >= readers.size()
                || readers[handle.slot] == std::numeric_limits<std::uint32_t>::max()) {
                return false;
            }
            ++readers[handle.slot];
        }
    }
    return true;
}

bool KvCacheManager::auditPool(PageKind kind, Audit const& audit) const
{
    Audit::PerKind const& expect = audit.of(kind);
    std::vector<Page> const& pages = kind == PageKind::Micro ? micro_pages_ : extent_pages_;
    PagePool const& pool = kind == PageKind::Micro ? micro_pool_ : extent_pool_;
    std::uint16_t const capacity = pageTokenCapacity(kind);
    std::uint32_t allocated = 0;
    for (std::size_t i = 0; i < pages.size(); ++i) {
        Page const& p = pages[i];
        if (p.state == PageState::Free) {
            if (p.valid_tokens != 0 || p.ref_count != 0 || p.promotion_pins != 0
                || p.inflight_readers != 0 || p.mutable_owner != kInvalidRequestId
                || expect.refs[i] != 0 || expect.pins[i] != 0 || expect.readers[i] != 0
                || expect.targets[i] != 0) {
                return false;
            }
            continue;
        }
        ++allocated;
        if (p.generation == PageHandle::kInvalidGeneration) {
            return false;
        }
        PageHandle const handle{kind, static_cast<std::uint32_t>(i), p.generation};
        if (pool.validate(handle) != PagePoolError::None || p.ref_count != expect.refs[i]
            || p.promotion_pins != expect.pins[i] || p.inflight_readers != expect.readers[i]) {
            return false;
        }
        bool const is_target = expect.targets[i] != 0;
        switch (p.state) {
        case PageState::Mutable:
            if (kind != PageKind::Micro || p.ref_count != 1 || p.valid_tokens == 0
                || p.valid_tokens >= capacity || p.mutable_owner == kInvalidRequestId
                || p.promotion_pins != 0 || is_target) {
                return false;
            }
            break;
        case PageState::Sealed:
            if (p.ref_count == 0 || p.valid_tokens == 0 || p.valid_tokens > capacity
                || p.mutable_owner != kInvalidRequestId || is_target) {
                return false;
            }
            break;
        case PageState::CopyTarget:
            if (!is_target || p.ref_count != 0 || p.promotion_pins != 0
                || p.mutable_owner != kInvalidRequestId
                || (kind == PageKind::Extent && p.valid_tokens != capacity)
                || (kind == PageKind::Micro && p.valid_tokens >= capacity)) {
                return false;
            }
            break;
        case PageState::Retiring:
            if (p.ref_count != 0 || p.mutable_owner != kInvalidRequestId || is_target
                || (p.promotion_pins == 0 && p.inflight_readers == 0)) {
                return false;
            }
            break;
        default:
            return false;
        }
    }
    PagePoolSnapshot const snap = pool.snapshot();
    return snap.allocated_slots == allocated && snap.capacityBalanced();
}

} // namespace kimkvcache
