// Fixed-page KV metadata runtime (reference semantics:
// src/fixed/fixed_page_manager.cpp:28-850, src/fixed/fixed_token_reservation.cpp:8-271).
//
// Observable behaviour that the parity tests pin: error precedence of every
// call, the order in which pages are taken from and returned to the LIFO
// pool (it fixes slot numbers and generations), table versions (+1 per
// committed mapping change; a fork child starts at 1, or 0 when empty), and
// the snapshot counters.
#include "fixed_page_manager.h"

#include <algorithm>
#include <limits>
#include <stdexcept>

namespace kimkvcache {
namespace {

constexpr std::size_t kNoEntry = std::numeric_limits<std::size_t>::max();

std::uint16_t checkedPageTokens(std::uint16_t tokens_per_page)
{
    if (tokens_per_page == 0) {
        throw std::invalid_argument("fixed page token capacity must be greater than zero");
    }
    return tokens_per_page;
}

} // namespace

FixedPageManager::FixedPageManager(std::uint16_t tokens_per_page, std::uint32_t page_capacity)
    : page_tokens_(checkedPageTokens(tokens_per_page))
    , pool_(PageKind::Micro, page_capacity)
    , pages_(page_capacity)
{
}

FixedPageManager::Page* FixedPageManager::page(PageHandle h) noexcept
{
    if (!h.isStructurallyValid() || h.kind != PageKind::Micro || h.slot >= pages_.size()
        || pages_[h.slot].generation != h.generation) {
        return nullptr;
    }
    return &pages_[h.slot];
}

FixedPageManager::Page const* FixedPageManager::page(PageHandle h) const noexcept
{
    return const_cast<FixedPageManager*>(this)->page(h);
}

// Takes a page from the pool as a CopyTarget holding `initial_valid` tokens
// (0 for a fresh page, the old tail's count for a copy-on-write target).
KvCacheError FixedPageManager::stage(std::uint16_t initial_valid, PageHandle& out)
{
    if (initial_valid >= page_tokens_) {
        return KvCacheError::InvalidArgument;
    }
    PageAllocationResult const got = pool_.allocate();
    if (!got.ok()) {
        return got.error == PagePoolError::Exhausted ? KvCacheError::ResourceExhausted
                                                     : KvCacheError::InternalInvariantViolation;
    }
    out = got.handle;
    peak_allocated_ = std::max<std::uint64_t>(peak_allocated_, pool_.snapshot().allocated_slots);
    if (out.slot >= pages_.size() || pages_[out.slot].state != PageState::Free
        || pages_[out.slot].ref_count != 0) {
        static_cast<void>(pool_.release(out));
        out = PageHandle::invalid();
        return KvCacheError::InternalInvariantViolation;
    }
    Page& p = pages_[out.slot];
    p.state = PageState::CopyTarget;
    p.generation = out.generation;
    p.valid_tokens = initial_valid;
    p.ref_count = 0;
    p.owner = kInvalidRequestId;
    return KvCacheError::None;
}

// Returns staged pages newest first, so the pool's free stack ends up as it
// was before the failed operation.
void FixedPageManager::unstage(std::vector<PageHandle> const& staged) noexcept
{
    for (auto it = staged.rbegin(); it != staged.rend(); ++it) {
        Page* p = page(*it);
        if (p != nullptr && p->state == PageState::CopyTarget && p->ref_count == 0
            && pool_.release(*it) == PagePoolError::None) {
            markFree(*p);
        }
    }
}

void FixedPageManager::markFree(Page& p) noexcept
{
    p.state = PageState::Free;
    p.valid_tokens = 0;
    p.ref_count = 0;
    p.owner = kInvalidRequestId;
}

KvCacheError FixedPageManager::freePage(PageHandle h)
{
    Page* p = page(h);
    if (p == nullptr || p->state == PageState::Free) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (p->ref_count != 0) {
        return KvCacheError::InvalidState;
    }
    p->owner = kInvalidRequestId;
    if (pool_.validate(h) != PagePoolError::None || pool_.release(h) != PagePoolError::None) {
        return KvCacheError::InternalInvariantViolation;
    }
    markFree(*p);
    return KvCacheError::None;
}

KvCacheError FixedPageManager::dropReference(PageHandle h)
{
    Page* p = page(h);
    if (p == nullptr || p->state == PageState::Free || p->state == PageState::CopyTarget
        || p->ref_count == 0) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (--p->ref_count != 0) {
        return KvCacheError::None;
    }
    return freePage(h);
}

void FixedPageManager::publish(Page& p, std::uint16_t valid_tokens, RequestId owner) noexcept
{
    p.valid_tokens = valid_tokens;
    p.ref_count = 1;
    bool const full = valid_tokens == page_tokens_;
    p.state = full ? PageState::Sealed : PageState::Mutable;
    p.owner = full ? kInvalidRequestId : owner;
}

KvCacheError FixedPageManager::createRequest(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    return requests_.emplace(request_id, BlockTable{}).second ? KvCacheError::None
                                                              : KvCacheError::RequestAlreadyExists;
}

KvCacheError FixedPageManager::append(RequestId request_id, std::uint32_t token_count)
{
    if (request_id == kInvalidRequestId || token_count == 0) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (reserved(request_id)) {
        return KvCacheError::RequestConflict;
    }
    BlockTable& table = found->second;
    std::uint32_t const old_tokens = table.tokenCount();
    if (token_count > std::numeric_limits<std::uint32_t>::max() - old_tokens) {
        return KvCacheError::InvalidArgument;
    }

    BlockTable candidate = table;
    std::size_t const max_new = (std::size_t(token_count) + page_tokens_ - 1) / page_tokens_ + 1;
    candidate.entries_.reserve(candidate.entries_.size() + max_new);
    std::vector<PageHandle> staged;
    std::vector<std::size_t> staged_entry;
    staged.reserve(max_new);
    staged_entry.reserve(max_new);
    std::size_t open = kNoEntry;  // entry still taking tokens
    PageHandle in_place = PageHandle::invalid();
    PageHandle replaced_tail = PageHandle::invalid();

    if (!candidate.entries_.empty()) {
        std::size_t const tail_index = candidate.entries_.size() - 1;
        MappingEntry& tail = candidate.entries_[tail_index];
        Page const* tp = page(tail.handle);
        if (tp == nullptr || tp->valid_tokens != tail.valid_tokens) {
            return KvCacheError::InternalInvariantViolation;
        }
        if (tail.valid_tokens < page_tokens_) {
            if (tp->state == PageState::Mutable) {
                if (tp->ref_count != 1 || tp->owner != request_id) {
                    return KvCacheError::InternalInvariantViolation;
                }
                in_place = tail.handle;
                open = tail_index;
            } else if (tp->state == PageState::Sealed) {
                // A sealed (possibly shared) partial tail is never written:
                // its tokens go to a copy that replaces it in this table.
                PageHandle copy = PageHandle::invalid();
                KvCacheError const e = stage(tail.valid_tokens, copy);
                if (e != KvCacheError::None) {
                    return e;
                }
                staged.push_back(copy);
                staged_entry.push_back(tail_index);
                replaced_tail = tail.handle;
                tail.handle = copy;
                open = tail_index;
            } else {
                return KvCacheError::InvalidState;
            }
        } else if (tp->state != PageState::Sealed) {
            return KvCacheError::InternalInvariantViolation;
        }
    }

    std::uint32_t remaining = token_count;
    std::uint32_t logical_end = old_tokens;
    while (remaining != 0) {
        if (open == kNoEntry) {
            PageHandle fresh = PageHandle::invalid();
            KvCacheError const e = stage(0, fresh);
            if (e != KvCacheError::None) {
                unstage(staged);
                return e;
            }
            open = candidate.entries_.size();
            candidate.entries_.push_back(MappingEntry{logical_end, 0, PageKind::Micro, fresh});
            staged.push_back(fresh);
            staged_entry.push_back(open);
        }
        MappingEntry& entry = candidate.entries_[open];
        std::uint32_t const take = std::min<std::uint32_t>(remaining, page_tokens_ - entry.valid_tokens);
        entry.valid_tokens = static_cast<std::uint16_t>(entry.valid_tokens + take);
        logical_end += take;
        remaining -= take;
        if (entry.valid_tokens == page_tokens_) {
            open = kNoEntry;
        }
    }
    candidate.version_ = table.version_ + 1;
    if (!candidate.checkInvariants(page_tokens_)) {
        unstage(staged);
        return KvCacheError::InternalInvariantViolation;
    }

    // Commit: nothing below can fail on a consistent state.
    if (replaced_tail.isStructurallyValid()) {
        KvCacheError const e = dropReference(replaced_tail);
        if (e != KvCacheError::None) {
            unstage(staged);
            return e;
        }
    }
    if (in_place.isStructurallyValid()) {
        Page* p = page(in_place);
        auto const e = std::find_if(candidate.entries_.begin(), candidate.entries_.end(),
            [in_place](MappingEntry const& m) { return m.handle == in_place; });
        p->valid_tokens = e->valid_tokens;
        if (e->valid_tokens == page_tokens_) {
            p->state = PageState::Sealed;
            p->owner = kInvalidRequestId;
        }
    }
    for (std::size_t k = 0; k < staged.size(); ++k) {
        publish(*page(staged[k]), candidate.entries_[staged_entry[k]].valid_tokens, request_id);
    }
    table = std::move(candidate);
    return KvCacheError::None;
}

KvTokenReservationId FixedPageManager::nextReservationId()
{
    for (std::size_t attempt = 0; attempt <= reservations_.size(); ++attempt) {
        KvTokenReservationId const id = next_reservation_++;
        if (next_reservation_ == kInvalidKvTokenReservationId) {
            next_reservation_ = 1;
        }
        if (id != kInvalidKvTokenReservationId && reservations_.count(id) == 0) {
            return id;
        }
    }
    return kInvalidKvTokenReservationId;
}

TokenReservationResult FixedPageManager::reserveToken(RequestId request_id,
    std::uint32_t expected_committed_tokens)
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
    if (reserved(request_id)) {
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

    Reservation r;
    r.request = request_id;
    r.table_version = before.version_;
    r.candidate = before;
    BlockTable& c = r.candidate;
    c.entries_.reserve(c.entries_.size() + 1);
    if (c.entries_.empty() || c.entries_.back().valid_tokens == page_tokens_) {
        KvCacheError const e = stage(0, r.target);
        if (e != KvCacheError::None) {
            result.error = e;
            return result;
        }
        c.entries_.push_back(MappingEntry{expected_committed_tokens, 1, PageKind::Micro, r.target});
    } else {
        MappingEntry& tail = c.entries_.back();
        Page const* tp = page(tail.handle);
        if (tp == nullptr || tp->valid_tokens != tail.valid_tokens) {
            result.error = KvCacheError::InternalInvariantViolation;
            return result;
        }
        if (tp->state == PageState::Mutable) {
            if (tp->ref_count != 1 || tp->owner != request_id) {
                result.error = KvCacheError::InternalInvariantViolation;
                return result;
            }
            r.in_place = tail.handle;
        } else if (tp->state == PageState::Sealed) {
            KvCacheError const e = stage(tail.valid_tokens, r.target);
            if (e != KvCacheError::None) {
                result.error = e;
                return result;
            }
            r.replaced_tail = tail.handle;
            tail.handle = r.target;
        } else {
            result.error = KvCacheError::InvalidState;
            return result;
        }
        ++tail.valid_tokens;
    }
    c.version_ = before.version_ + 1;

    auto abandon = [&](KvCacheError e) {
        if (r.target.isStructurallyValid()) {
            static_cast<void>(freePage(r.target));
        }
        result.error = e;
        result.before = BlockTable{};
        result.reserved = BlockTable{};
        return result;
    };
    if (!c.checkInvariants(page_tokens_)) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    KvTokenReservationId const id = nextReservationId();
    if (id == kInvalidKvTokenReservationId) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    result.before = before;
    result.reserved = c;
    if (!reservations_.emplace(id, std::move(r)).second) {
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    if (!by_request_.emplace(request_id, id).second) {
        reservations_.erase(id);
        return abandon(KvCacheError::InternalInvariantViolation);
    }
    result.error = KvCacheError::None;
    result.reservation_id = id;
    return result;
}

KvCacheError FixedPageManager::commitTokenReservation(KvTokenReservationId reservation_id)
{
    if (reservation_id == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = reservations_.find(reservation_id);
    if (found == reservations_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    Reservation& r = found->second;
    auto req = requests_.find(r.request);
    if (req == requests_.end() || req->second.version_ != r.table_version) {
        return KvCacheError::RequestConflict;
    }
    std::uint16_t const tail_tokens = r.candidate.entries_.back().valid_tokens;
    Page* target = r.target.isStructurallyValid() ? page(r.target) : nullptr;
    Page* in_place = r.in_place.isStructurallyValid() ? page(r.in_place) : nullptr;
    Page const* replaced = r.replaced_tail.isStructurallyValid() ? page(r.replaced_tail) : nullptr;
    if ((target != nullptr && (target->state != PageState::CopyTarget || target->ref_count != 0))
        || (in_place != nullptr
            && (in_place->state != PageState::Mutable || in_place->ref_count != 1
                || in_place->owner != r.request))
        || (replaced != nullptr && (replaced->state != PageState::Sealed || replaced->ref_count == 0))) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (r.replaced_tail.isStructurallyValid()) {
        KvCacheError const e = dropReference(r.replaced_tail);
        if (e != KvCacheError::None) {
            return e;
        }
    }
    if (in_place != nullptr) {
        in_place->valid_tokens = tail_tokens;
        if (tail_tokens == page_tokens_) {
            in_place->state = PageState::Sealed;
            in_place->owner = kInvalidRequestId;
        }
    }
    if (target != nullptr) {
        publish(*target, tail_tokens, r.request);
    }
    req->second = std::move(r.candidate);
    by_request_.erase(r.request);
    reservations_.erase(found);
    return KvCacheError::None;
}

KvCacheError FixedPageManager::rollbackTokenReservation(KvTokenReservationId reservation_id)
{
    if (reservation_id == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = reservations_.find(reservation_id);
    if (found == reservations_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    if (found->second.target.isStructurallyValid()) {
        KvCacheError const e = freePage(found->second.target);
        if (e != KvCacheError::None) {
            return e;
        }
    }
    by_request_.erase(found->second.request);
    reservations_.erase(found);
    return KvCacheError::None;
}

KvCacheError FixedPageManager::sealTail(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (reserved(request_id)) {
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
    if (p->state != PageState::Mutable || p->ref_count != 1 || p->owner != request_id) {
        return KvCacheError::InvalidState;
    }
    // The mapping is unchanged, so the table version stays.
    p->state = PageState::Sealed;
    p->owner = kInvalidRequestId;
    return KvCacheError::None;
}

KvCacheError FixedPageManager::forkRequest(RequestId source_request_id, RequestId child_request_id)
{
    if (source_request_id == kInvalidRequestId || child_request_id == kInvalidRequestId
        || source_request_id == child_request_id) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto source = requests_.find(source_request_id);
    if (source == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (reserved(source_request_id)) {
        return KvCacheError::RequestConflict;
    }
    if (requests_.count(child_request_id) != 0) {
        return KvCacheError::RequestAlreadyExists;
    }
    std::vector<MappingEntry> const& entries = source->second.entries_;
    for (std::size_t i = 0; i < entries.size(); ++i) {
        Page const* p = page(entries[i].handle);
        if (p == nullptr || p->valid_tokens != entries[i].valid_tokens || p->ref_count == 0
            || p->ref_count == std::numeric_limits<std::uint32_t>::max()) {
            return KvCacheError::InternalInvariantViolation;
        }
        if (p->state == PageState::Mutable) {
            if (i + 1 != entries.size() || p->ref_count != 1 || p->owner != source_request_id) {
                return KvCacheError::InternalInvariantViolation;
            }
        } else if (p->state != PageState::Sealed) {
            return KvCacheError::InvalidState;
        }
    }
    BlockTable child = source->second;
    child.version_ = child.entries_.empty() ? 0 : 1;
    // The emplace may rehash: keep no iterator into requests_ across it.
    auto const inserted = requests_.emplace(child_request_id, std::move(child));
    if (!inserted.second) {
        return KvCacheError::RequestAlreadyExists;
    }
    // Both tables now share every page; a shared tail is sealed so the next
    // write on either side copies it.
    for (MappingEntry const& e : inserted.first->second.entries_) {
        Page* p = page(e.handle);
        if (p->state == PageState::Mutable) {
            p->state = PageState::Sealed;
            p->owner = kInvalidRequestId;
        }
        ++p->ref_count;
    }
    return KvCacheError::None;
}

KvCacheError FixedPageManager::releaseRequest(RequestId request_id)
{
    if (request_id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return KvCacheError::RequestNotFound;
    }
    if (reserved(request_id)) {
        return KvCacheError::RequestConflict;
    }
    for (MappingEntry const& e : found->second.entries_) {
        Page const* p = page(e.handle);
        if (p == nullptr || p->state == PageState::Free || p->state == PageState::CopyTarget
            || p->ref_count == 0) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    for (MappingEntry const& e : found->second.entries_) {
        KvCacheError const err = dropReference(e.handle);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    requests_.erase(found);
    return KvCacheError::None;
}

std::optional<BlockTable> FixedPageManager::blockTable(RequestId request_id) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    auto found = requests_.find(request_id);
    if (found == requests_.end()) {
        return std::nullopt;
    }
    return found->second;
}

FixedPageManagerSnapshot FixedPageManager::snapshot() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    FixedPageManagerSnapshot s;
    s.request_count = requests_.size();
    s.pool = pool_.snapshot();
    s.successful_allocations = s.pool.successful_allocations;
    s.peak_allocated_pages = peak_allocated_;
    s.token_reservation_count = reservations_.size();
    return s;
}

bool FixedPageManager::checkInvariants() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return consistent();
}

// Cross-checks the three views of the state: request tables, per-page
// records and the pool. References counted from the tables must equal each
// page's ref_count; a CopyTarget page must belong to exactly one pending
// reservation; the pool's allocated count must equal the non-Free pages.
bool FixedPageManager::consistent() const
{
    if (!pool_.checkInvariants() || reservations_.size() != by_request_.size()) {
        return false;
    }
    std::vector<std::uint32_t> refs(pages_.size(), 0);
    for (auto const& [rid, table] : requests_) {
        if (rid == kInvalidRequestId || !table.checkInvariants(page_tokens_)) {
            return false;
        }
        std::vector<MappingEntry> const& entries = table.entries_;
        for (std::size_t i = 0; i < entries.size(); ++i) {
            MappingEntry const& e = entries[i];
            Page const* p = page(e.handle);
            if (e.kind != PageKind::Micro || e.valid_tokens == 0 || e.valid_tokens > page_tokens_
                || p == nullptr || p->valid_tokens != e.valid_tokens
                || refs[e.handle.slot] == std::numeric_limits<std::uint32_t>::max()) {
                return false;
            }
            bool const tail = i + 1 == entries.size();
            if (p->state == PageState::Mutable) {
                if (!tail || p->ref_count != 1 || p->owner != rid) {
                    return false;
                }
            } else if (p->state != PageState::Sealed) {
                return false;
            }
            ++refs[e.handle.slot];
        }
    }
    std::vector<std::uint8_t> targets(pages_.size(), 0);
    for (auto const& [id, r] : reservations_) {
        auto const req = requests_.find(r.request);
        auto const back = by_request_.find(r.request);
        if (id == kInvalidKvTokenReservationId || req == requests_.end() || back == by_request_.end()
            || back->second != id || !r.candidate.checkInvariants(page_tokens_)
            || r.candidate.tokenCount() != req->second.tokenCount() + 1
            || r.candidate.version() != req->second.version() + 1) {
            return false;
        }
        if (r.target.isStructurallyValid() == r.in_place.isStructurallyValid()) {
            return false;  // exactly one way of placing the token
        }
        BlockTable const& committed = req->second;
        if (r.target.isStructurallyValid()) {
            Page const* t = page(r.target);
            if (t == nullptr || t->state != PageState::CopyTarget || t->ref_count != 0
                || targets[r.target.slot] != 0) {
                return false;
            }
            std::uint16_t const copied = r.replaced_tail.isStructurallyValid()
                ? static_cast<std::uint16_t>(r.candidate.entries_.back().valid_tokens - 1)
                : 0;
            if (t->valid_tokens != copied) {
                return false;
            }
            targets[r.target.slot] = 1;
        } else {
            Page const* p = page(r.in_place);
            if (p == nullptr || p->state != PageState::Mutable || p->ref_count != 1 || p->owner != r.request
                || committed.entries_.empty() || committed.entries_.back().handle != r.in_place) {
                return false;
            }
        }
        if (r.replaced_tail.isStructurallyValid()) {
            Page const* p = page(r.replaced_tail);
            if (p == nullptr || p->state != PageState::Sealed || p->ref_count == 0
                || committed.entries_.empty() || committed.entries_.back().handle != r.replaced_tail) {
                return false;
            }
        }
    }
    std::uint32_t in_use = 0;
    for (std::size_t slot = 0; slot < pages_.size(); ++slot) {
        Page const& p = pages_[slot];
        bool ok = true;
        switch (p.state) {
        case PageState::Free:
            if (p.valid_tokens != 0 || p.ref_count != 0 || p.owner != kInvalidRequestId || refs[slot] != 0) {
                return false;
            }
            continue;
        case PageState::Mutable: ok = p.ref_count == 1 && p.owner != kInvalidRequestId; break;
        case PageState::Sealed: ok = p.ref_count != 0 && p.owner == kInvalidRequestId; break;
        case PageState::CopyTarget:
            ok = p.ref_count == 0 && p.owner == kInvalidRequestId && targets[slot] != 0
                && p.valid_tokens < page_tokens_;
            break;
        default: ok = false;
        }
        if (!ok || p.valid_tokens > page_tokens_
            || (p.valid_tokens == 0 && p.state != PageState::CopyTarget)
            || p.generation == PageHandle::kInvalidGeneration || p.ref_count != refs[slot]
            || pool_.validate(PageHandle{PageKind::Micro, static_cast<std::uint32_t>(slot), p.generation})
                != PagePoolError::None) {
            return false;
        }
        ++in_use;
    }
    PagePoolSnapshot const ps = pool_.snapshot();
    return ps.allocated_slots == in_use && ps.capacityBalanced();
}

} // namespace kimkvcache
