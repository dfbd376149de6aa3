// KvCacheManager: request lifecycle, append, token reservations.
// Reference semantics: src/runtime/kv_cache_manager.cpp:12-249,
// kv_cache_append.cpp:12-258, token_reservation.cpp:10-326,
// kv_cache_lifecycle.cpp:12-195, kv_cache_inspection.cpp:12-78.
#include "kv_cache_manager.h"

#include <algorithm>
#include <limits>
#include <utility>

namespace kimkvcache {

KvCacheManager::KvCacheManager(std::uint32_t micro_capacity, std::uint32_t extent_capacity)
    : micro_pool_(PageKind::Micro, micro_capacity)
    , extent_pool_(PageKind::Extent, extent_capacity)
    , micro_pages_(micro_capacity)
    , extent_pages_(extent_capacity)
{
}

// Takes a fresh micro page for a staged copy-on-write or growth target. The
// page stays CopyTarget (unreferenced) until the owning operation commits.
KvCacheError KvCacheManager::stageMicro(std::uint16_t initial_valid_tokens, PageHandle& out)
{
    if (initial_valid_tokens >= kMicroPageTokenCapacity) {
        return KvCacheError::InvalidArgument;
    }
    PageAllocationResult const got = micro_pool_.allocate();
    if (!got.ok()) {
        return got.error == PagePoolError::Exhausted ? KvCacheError::ResourceExhausted
                                                     : KvCacheError::InternalInvariantViolation;
    }
    out = got.handle;
    if (out.slot >= micro_pages_.size()) {
        static_cast<void>(micro_pool_.release(out));
        out = PageHandle::invalid();
        return KvCacheError::InternalInvariantViolation;
    }
    Page& p = micro_pages_[out.slot];
    if (p.state != PageState::Free || p.ref_count != 0 || p.promotion_pins != 0
        || p.inflight_readers != 0) {
        static_cast<void>(micro_pool_.release(out));
        out = PageHandle::invalid();
        return KvCacheError::InternalInvariantViolation;
    }
    p = Page{PageState::CopyTarget, out.generation, initial_valid_tokens, 0, 0, 0,
        kInvalidRequestId};
    return KvCacheError::None;
}

void KvCacheManager::clearFreed(Page& p) noexcept
{
    // The generation is kept: it identifies the last handle issued for the slot.
    p.state = PageState::Free;
    p.valid_tokens = 0;
    p.ref_count = 0;
    p.promotion_pins = 0;
    p.inflight_readers = 0;
    p.mutable_owner = kInvalidRequestId;
}

void KvCacheManager::unstage(std::vector<Staged> const& staged) noexcept
{
    for (auto it = staged.rbegin(); it != staged.rend(); ++it) {
        Page* p = page(it->handle);
        if (p == nullptr || p->state != PageState::CopyTarget || p->ref_count != 0) {
            continue;
        }
        if (micro_pool_.release(it->handle) == PagePoolError::None) {
            clearFreed(*p);
        }
    }
}

// Drops an unreferenced page: back to its pool, or Retiring while a lease or
// a promotion still pins it.
KvCacheError KvCacheManager::retireOrFree(PageHandle handle)
{
    Page* p = page(handle);
    if (p == nullptr || p->state == PageState::Free) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (p->ref_count != 0) {
        return KvCacheError::InvalidState;
    }
    p->mutable_owner = kInvalidRequestId;
    if (p->promotion_pins != 0 || p->inflight_readers != 0) {
        p->state = PageState::Retiring;
        return KvCacheError::None;
    }
    PagePool& pool = poolFor(handle.kind);
    if (pool.validate(handle) != PagePoolError::None
        || pool.release(handle) != PagePoolError::None) {
        return KvCacheError::InternalInvariantViolation;
    }
    clearFreed(*p);
    return KvCacheError::None;
}

KvCacheError KvCacheManager::dropReference(PageHandle handle)
{
    Page* p = page(handle);
    if (p == nullptr || p->state == PageState::Free || p->state == PageState::CopyTarget
        || p->ref_count == 0) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (--p->ref_count != 0) {
        return KvCacheError::None;
    }
    return retireOrFree(handle);
}

bool KvCacheManager::hasReservation(RequestId request_id) const noexcept
{
    return request_reservation_.find(request_id) != request_reservation_.end();
}

KvCacheError KvCacheManager::createRequest(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    return requests_.emplace(request_id, BlockTable{}).second
        ? KvCacheError::None : KvCacheError::RequestAlreadyExists;
}

KvCacheError KvCacheManager::append(RequestId request_id, std::uint32_t token_count)
{
    if (request_id == kInvalidRequestId || token_count == 0) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (hasReservation(request_id)) {
        return KvCacheError::RequestConflict;
    }
    BlockTable& table = found->second;
    std::uint32_t const old_tokens = table.tokenCount();
    if (token_count > std::numeric_limits<std::uint32_t>::max() - old_tokens) {
        return KvCacheError::InvalidArgument;
    }

    constexpr std::size_t kNone = std::numeric_limits<std::size_t>::max();
    std::size_t const max_new_pages =
        (static_cast<std::size_t>(token_count) + kMicroPageTokenCapacity - 1)
            / kMicroPageTokenCapacity + 1;
    BlockTable candidate = table;
    candidate.entries_.reserve(candidate.entries_.size() + max_new_pages);
    std::vector<Staged> staged;
    staged.reserve(max_new_pages);
    std::size_t active = kNone;
    PageHandle existing_mutable = PageHandle::invalid();
    PageHandle replaced_sealed_tail = PageHandle::invalid();

    if (!candidate.entries_.empty()) {
        std::size_t const tail_index = candidate.entries_.size() - 1;
        MappingEntry& tail = candidate.entries_[tail_index];
        Page* tail_page = page(tail.handle);
        if (tail_page == nullptr || tail_page->valid_tokens != tail.valid_tokens) {
            return KvCacheError::InternalInvariantViolation;
        }
        if (tail.kind == PageKind::Micro && tail.valid_tokens < kMicroPageTokenCapacity) {
            if (tail_page->state == PageState::Mutable) {
                if (tail_page->ref_count != 1 || tail_page->mutable_owner != request_id) {
                    return KvCacheError::InternalInvariantViolation;
                }
                existing_mutable = tail.handle;
                active = tail_index;
            } else if (tail_page->state == PageState::Sealed) {
                // Shared or sealed partial tail: copy-on-write into a new page.
                PageHandle copy = PageHandle::invalid();
                KvCacheError const error = stageMicro(tail.valid_tokens, copy);
                if (error != KvCacheError::None) {
                    return error;
                }
                staged.push_back(Staged{copy, tail_index});
                replaced_sealed_tail = tail.handle;
                tail.kind = PageKind::Micro;
                tail.handle = copy;
                active = tail_index;
            } else {
                return KvCacheError::InvalidState;
            }
        } else if (tail_page->state != PageState::Sealed) {
            return KvCacheError::InternalInvariantViolation;
        }
    }

    std::uint32_t remaining = token_count;
    std::uint32_t logical_end = old_tokens;
    while (remaining != 0) {
        if (active == kNone) {
            PageHandle fresh = PageHandle::invalid();
            KvCacheError const error = stageMicro(0, fresh);
            if (error != KvCacheError::None) {
                unstage(staged);
                return error;
            }
            active = candidate.entries_.size();
            candidate.entries_.push_back(MappingEntry{logical_end, 0, PageKind::Micro, fresh});
            staged.push_back(Staged{fresh, active});
        }
        MappingEntry& entry = candidate.entries_[active];
        std::uint32_t const take = std::min<std::uint32_t>(
            remaining, kMicroPageTokenCapacity - entry.valid_tokens);
        entry.valid_tokens = static_cast<std::uint16_t>(entry.valid_tokens + take);
        logical_end += take;
        remaining -= take;
        if (entry.valid_tokens == kMicroPageTokenCapacity) {
            active = kNone;
        }
    }
    candidate.version_ = table.version_ + 1;

    // Re-validate everything before entering the no-fail commit section.
    bool consistent = candidate.checkInvariants();
    if (consistent && existing_mutable.isStructurallyValid()) {
        Page const* p = page(existing_mutable);
        consistent = p != nullptr && p->state == PageState::Mutable && p->ref_count == 1
            && p->mutable_owner == request_id;
    }
    if (consistent && replaced_sealed_tail.isStructurallyValid()) {
        Page const* p = page(replaced_sealed_tail);
        consistent = p != nullptr && p->state == PageState::Sealed && p->ref_count != 0;
    }
    for (std::size_t i = 0; consistent && i < staged.size(); ++i) {
        Page const* p = page(staged[i].handle);
        consistent = p != nullptr && p->state == PageState::CopyTarget && p->ref_count == 0
            && staged[i].entry_index < candidate.entries_.size()
            && candidate.entries_[staged[i].entry_index].handle == staged[i].handle;
    }
    if (!consistent) {
        unstage(staged);
        return KvCacheError::InternalInvariantViolation;
    }

    if (replaced_sealed_tail.isStructurallyValid()) {
        KvCacheError const error = dropReference(replaced_sealed_tail);
        if (error != KvCacheError::None) {
            unstage(staged);
            return error;
        }
    }
    if (existing_mutable.isStructurallyValid()) {
        Page* p = page(existing_mutable);
        for (MappingEntry const& entry : candidate.entries_) {
            if (entry.handle == existing_mutable) {
                p->valid_tokens = entry.valid_tokens;
                if (entry.valid_tokens == kMicroPageTokenCapacity) {
                    p->state = PageState::Sealed;
                    p->mutable_owner = kInvalidRequestId;
                }
                break;
            }
        }
    }
    for (Staged const& s : staged) {
        Page* p = page(s.handle);
        MappingEntry const& entry = candidate.entries_[s.entry_index];
        p->valid_tokens = entry.valid_tokens;
        p->ref_count = 1;
        bool const full = entry.valid_tokens == kMicroPageTokenCapacity;
        p->state = full ? PageState::Sealed : PageState::Mutable;
        p->mutable_owner = full ? kInvalidRequestId : request_id;
    }
    table = std::move(candidate);
    return KvCacheError::None;
}

TokenReservationResult KvCacheManager::reserveToken(
    RequestId request_id, std::uint32_t expected_committed_tokens)
{
    TokenReservationResult result;
    result.request_id = request_id;
    result.logical_token_position = expected_committed_tokens;
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
    bool const promoting = std::any_of(promotions_.begin(), promotions_.end(),
        [request_id](auto const& p) { return p.second.request_id == request_id; });
    if (hasReservation(request_id) || promoting) {
        result.error = KvCacheError::RequestConflict;
        return result;
    }
    BlockTable const& before = found->second;
    if (before.tokenCount() != expected_committed_tokens
        || before.version_ == std::numeric_limits<std::uint64_t>::max()
        || expected_committed_tokens == std::numeric_limits<std::uint32_t>::max()) {
        result.error = KvCacheError::InvalidState;
        return result;
    }

    BlockTable candidate = before;
    candidate.entries_.reserve(candidate.entries_.size() + 1);
    PageHandle staged = PageHandle::invalid();
    PageHandle existing_mutable = PageHandle::invalid();
    PageHandle replaced_sealed_tail = PageHandle::invalid();

    bool const needs_new_page = candidate.entries_.empty()
        || candidate.entries_.back().kind == PageKind::Extent
        || candidate.entries_.back().valid_tokens == kMicroPageTokenCapacity;
    if (needs_new_page) {
        KvCacheError const error = stageMicro(0, staged);
        if (error != KvCacheError::None) {
            result.error = error;
            return result;
        }
        candidate.entries_.push_back(
            MappingEntry{expected_committed_tokens, 1, PageKind::Micro, staged});
    } else {
        MappingEntry& tail = candidate.entries_.back();
        Page const* tail_page = page(tail.handle);
        if (tail_page == nullptr || tail.kind != PageKind::Micro
            || tail_page->valid_tokens != tail.valid_tokens) {
            result.error = KvCacheError::InternalInvariantViolation;
            return result;
        }
        if (tail_page->state == PageState::Mutable) {
            if (tail_page->ref_count != 1 || tail_page->mutable_owner != request_id) {
                result.error = KvCacheError::InternalInvariantViolation;
                return result;
            }
            existing_mutable = tail.handle;
        } else if (tail_page->state == PageState::Sealed) {
            KvCacheError const error = stageMicro(tail.valid_tokens, staged);
            if (error != KvCacheError::None) {
                result.error = error;
                return result;
            }
            replaced_sealed_tail = tail.handle;
            tail.handle = staged;
        } else {
            result.error = KvCacheError::InvalidState;
            return result;
        }
        ++tail.valid_tokens;
    }
    candidate.version_ = before.version_ + 1;

    auto abandon = [&](KvCacheError error) {
        if (staged.isStructurallyValid()) {
            static_cast<void>(retireOrFree(staged));
        }
        result.error = error;
        return result;
    };
    if (!candidate.checkInvariants()) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    KvTokenReservationId const id = nextFreeId(next_reservation_id_, reservations_);
    if (id == kInvalidKvTokenReservationId) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    auto const inserted = reservations_.emplace(id, Reservation{id, request_id,
        before.version_, candidate, staged, existing_mutable, replaced_sealed_tail});
    if (!inserted.second) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    if (!request_reservation_.emplace(request_id, id).second) {
        reservations_.erase(inserted.first);
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    result.error = KvCacheError::None;
    result.reservation_id = id;
    result.before = before;
    result.reserved = std::move(candidate);
    return result;
}

KvCacheError KvCacheManager::commitTokenReservation(KvTokenReservationId id)
{
    if (id == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = reservations_.find(id);
    if (found == reservations_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    Reservation& r = found->second;
    auto request = requests_.find(r.request_id);
    if (request == requests_.end() || request->second.version_ != r.prepared_version) {
        return KvCacheError::RequestConflict;
    }
    MappingEntry const tail = r.candidate.entries_.back();
    Page* staged = r.staged_target.isStructurallyValid() ? page(r.staged_target) : nullptr;
    Page* existing = r.existing_mutable.isStructurallyValid() ? page(r.existing_mutable) : nullptr;
    Page* replaced = r.replaced_sealed_tail.isStructurallyValid()
        ? page(r.replaced_sealed_tail) : nullptr;
    if ((staged != nullptr && (staged->state != PageState::CopyTarget || staged->ref_count != 0))
        || (existing != nullptr
            && (existing->state != PageState::Mutable || existing->ref_count != 1
                || existing->mutable_owner != r.request_id))
        || (replaced != nullptr
            && (replaced->state != PageState::Sealed || replaced->ref_count == 0))) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (r.replaced_sealed_tail.isStructurallyValid()) {
        KvCacheError const error = dropReference(r.replaced_sealed_tail);
        if (error != KvCacheError::None) {
            return error;
        }
    }
    bool const full = tail.valid_tokens == kMicroPageTokenCapacity;
    if (existing != nullptr) {
        existing->valid_tokens = tail.valid_tokens;
        if (full) {
            existing->state = PageState::Sealed;
            existing->mutable_owner = kInvalidRequestId;
        }
    }
    if (staged != nullptr) {
        staged->valid_tokens = tail.valid_tokens;
        staged->ref_count = 1;
        staged->state = full ? PageState::Sealed : PageState::Mutable;
        staged->mutable_owner = full ? kInvalidRequestId : r.request_id;
    }
    request->second = std::move(r.candidate);
    request_reservation_.erase(r.request_id);
    reservations_.erase(found);
    return KvCacheError::None;
}

KvCacheError KvCacheManager::rollbackReservationLocked(KvTokenReservationId id)
{
    auto found = reservations_.find(id);
    if (found == reservations_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    if (found->second.staged_target.isStructurallyValid()) {
        KvCacheError const error = retireOrFree(found->second.staged_target);
        if (error != KvCacheError::None) {
            return error;
        }
    }
    request_reservation_.erase(found->second.request_id);
    reservations_.erase(found);
    return KvCacheError::None;
}

KvCacheError KvCacheManager::rollbackTokenReservation(KvTokenReservationId id)
{
    if (id == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    return rollbackReservationLocked(id);
}

KvCacheError KvCacheManager::sealTail(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (hasReservation(request_id)) {
        return KvCacheError::RequestConflict;
    }
    BlockTable const& table = found->second;
    if (table.entries_.empty()) {
        return KvCacheError::InvalidState;
    }
    MappingEntry const& tail = table.entries_.back();
    Page* p = page(tail.handle);
    if (p == nullptr || p->valid_tokens != tail.valid_tokens) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (p->state == PageState::Sealed) {
        return KvCacheError::None;
    }
    if (p->state != PageState::Mutable || p->ref_count != 1 || p->mutable_owner != request_id) {
        return KvCacheError::InvalidState;
    }
    p->state = PageState::Sealed;  // mapping unchanged: the version stays
    p->mutable_owner = kInvalidRequestId;
    return KvCacheError::None;
}

KvCacheError KvCacheManager::forkRequest(RequestId source, RequestId child)
{
    if (source == kInvalidRequestId || child == kInvalidRequestId || source == child) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(source);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (hasReservation(source)) {
        return KvCacheError::RequestConflict;
    }
    if (requests_.find(child) != requests_.end()) {
        return KvCacheError::RequestAlreadyExists;
    }
    BlockTable const& table = found->second;
    for (std::size_t i = 0; i < table.entries_.size(); ++i) {
        MappingEntry const& entry = table.entries_[i];
        Page const* p = page(entry.handle);
        if (p == nullptr || p->valid_tokens != entry.valid_tokens || p->ref_count == 0
            || p->ref_count == std::numeric_limits<std::uint32_t>::max()) {
            return KvCacheError::InternalInvariantViolation;
        }
        if (p->state == PageState::Mutable) {
            if (i + 1 != table.entries_.size() || p->ref_count != 1
                || p->mutable_owner != source) {
                return KvCacheError::InternalInvariantViolation;
            }
        } else if (p->state != PageState::Sealed) {
            return KvCacheError::InvalidState;
        }
    }
    BlockTable child_table = table;
    child_table.version_ = child_table.entries_.empty() ? 0 : 1;
    if (!requests_.emplace(child, std::move(child_table)).second) {
        return KvCacheError::RequestAlreadyExists;
    }
    // Both requests now share every page; the source's mutable tail becomes
    // sealed so that the next write by either side copies it.
    for (MappingEntry const& entry : table.entries_) {
        Page* p = page(entry.handle);
        if (p->state == PageState::Mutable) {
            p->state = PageState::Sealed;
            p->mutable_owner = kInvalidRequestId;
        }
        ++p->ref_count;
    }
    return KvCacheError::None;
}

KvCacheError KvCacheManager::releaseRequest(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (hasReservation(request_id)) {
        return KvCacheError::RequestConflict;
    }
    KvCacheError const rolled = rollbackRequestPromotionsLocked(request_id);
    if (rolled != KvCacheError::None) {
        return rolled;
    }
    BlockTable const& table = found->second;
    for (MappingEntry const& entry : table.entries_) {
        Page const* p = page(entry.handle);
        if (p == nullptr || p->state == PageState::Free || p->state == PageState::CopyTarget
            || p->ref_count == 0) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    for (MappingEntry const& entry : table.entries_) {
        KvCacheError const error = dropReference(entry.handle);
        if (error != KvCacheError::None) {
            return error;
        }
    }
    requests_.erase(found);
    return KvCacheError::None;
}

std::optional<BlockTable> KvCacheManager::blockTable(RequestId request_id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return std::nullopt;
    }
    return found->second;
}

std::optional<PageMetadataSnapshot> KvCacheManager::pageMetadata(PageHandle handle) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    Page const* p = page(handle);
    if (p == nullptr) {
        return std::nullopt;
    }
    return PageMetadataSnapshot{handle, p->state, p->valid_tokens, p->ref_count,
        p->promotion_pins, p->inflight_readers, p->mutable_owner};
}

KvCacheManagerSnapshot KvCacheManager::snapshot() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return KvCacheManagerSnapshot{requests_.size(), promotions_.size(), leases_.size(),
        reservations_.size(), micro_pool_.snapshot(), extent_pool_.snapshot()};
}

} // namespace kimkvcache
