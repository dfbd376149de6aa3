// The page-table engine shared by the two KV metadata runtimes (see
// paged_tables.h). Reference semantics: src/runtime/kv_cache_append.cpp,
// token_reservation.cpp, kv_cache_lifecycle.cpp and kv_cache_invariants.cpp
// for the two-pool runtime, src/fixed/*.cpp for the fixed-page one.
#include "paged_tables.h"

#include <algorithm>
#include <limits>
#include <stdexcept>

namespace kimkvcache {

namespace {
constexpr std::uint32_t kMaxU32 = std::numeric_limits<std::uint32_t>::max();
constexpr std::uint64_t kMaxU64 = std::numeric_limits<std::uint64_t>::max();
constexpr std::size_t kNoEntry = std::numeric_limits<std::size_t>::max();
} // namespace

PageSlots::PageSlots(PageKind k, std::uint32_t capacity, std::uint16_t tokens)
    : kind(k), page_tokens(tokens), pool(k, capacity), state(capacity, PageState::Free)
    , generation(capacity, 0), valid(capacity, 0), refs(capacity, 0), pins(capacity, 0)
    , readers(capacity, 0), owner(capacity, kInvalidRequestId)
{
}

void PageSlots::clear(std::uint32_t slot) noexcept
{
    state[slot] = PageState::Free;
    valid[slot] = 0;
    refs[slot] = 0;
    pins[slot] = 0;
    readers[slot] = 0;
    owner[slot] = kInvalidRequestId;
}

TableEngine::TableEngine(std::uint16_t micro_tokens, std::uint32_t micro_capacity,
    std::uint32_t extent_capacity)
    : micro_(PageKind::Micro, micro_capacity,
          micro_tokens != 0 ? micro_tokens
                            : throw std::invalid_argument("page token capacity must be greater than zero"))
{
    if (extent_capacity != 0) {
        extent_ = std::make_unique<PageSlots>(PageKind::Extent, extent_capacity, kExtentPageTokenCapacity);
    }
}

std::pair<PageSlots*, std::uint32_t> TableEngine::find(PageHandle h) noexcept
{
    auto const [s, slot] = static_cast<TableEngine const*>(this)->find(h);
    return {const_cast<PageSlots*>(s), slot};
}

std::pair<PageSlots const*, std::uint32_t> TableEngine::find(PageHandle h) const noexcept
{
    PageSlots const* s = poolOf(h);
    std::int64_t const slot = s != nullptr ? s->slotOf(h) : -1;
    if (slot < 0) {
        return {nullptr, 0};
    }
    return {s, static_cast<std::uint32_t>(slot)};
}

// ---- page transitions -------------------------------------------------------------

KvCacheError TableEngine::stage(PageKind kind, std::uint16_t tokens, PageHandle& out)
{
    out = PageHandle::invalid();
    if (kind == PageKind::Extent && extent_ == nullptr) {
        return KvCacheError::InternalInvariantViolation;
    }
    PageSlots& s = slots(kind);
    // A staged micro page is never full: a full page is published Sealed.
    if (kind == PageKind::Micro && tokens >= s.page_tokens) {
        return KvCacheError::InvalidArgument;
    }
    PageAllocationResult const got = s.pool.allocate();
    if (!got.ok()) {
        return got.error == PagePoolError::Exhausted ? KvCacheError::ResourceExhausted
                                                     : KvCacheError::InternalInvariantViolation;
    }
    std::uint32_t const slot = got.handle.slot;
    if (slot >= s.size() || s.state[slot] != PageState::Free || s.refs[slot] != 0 || s.pins[slot] != 0
        || s.readers[slot] != 0) {
        static_cast<void>(s.pool.release(got.handle));
        return KvCacheError::InternalInvariantViolation;
    }
    s.state[slot] = PageState::CopyTarget;
    s.generation[slot] = got.handle.generation;
    s.valid[slot] = tokens;
    s.owner[slot] = kInvalidRequestId;
    peak_allocated_ = std::max<std::uint64_t>(peak_allocated_, s.pool.snapshot().allocated_slots);
    out = got.handle;
    return KvCacheError::None;
}

KvCacheError TableEngine::retire(PageHandle h)
{
    auto const [s, slot] = find(h);
    if (s == nullptr || s->state[slot] == PageState::Free) {
        return KvCacheError::InternalInvariantViolation;
    }
    if (s->refs[slot] != 0) {
        return KvCacheError::InvalidState;
    }
    s->owner[slot] = kInvalidRequestId;
    if (s->pins[slot] != 0 || s->readers[slot] != 0) {
        s->state[slot] = PageState::Retiring;  // freed by the last unpin / lease release
        return KvCacheError::None;
    }
    if (s->pool.validate(h) != PagePoolError::None || s->pool.release(h) != PagePoolError::None) {
        return KvCacheError::InternalInvariantViolation;
    }
    s->clear(slot);
    return KvCacheError::None;
}

KvCacheError TableEngine::unref(PageHandle h)
{
    auto const [s, slot] = find(h);
    if (s == nullptr || s->refs[slot] == 0
        || (s->state[slot] != PageState::Mutable && s->state[slot] != PageState::Sealed
            && s->state[slot] != PageState::Retiring)) {
        return KvCacheError::InternalInvariantViolation;
    }
    return --s->refs[slot] == 0 ? retire(h) : KvCacheError::None;
}

// ---- table edits -----------------------------------------------------------------------

bool TableEngine::tableWellFormed(BlockTable const& t) const
{
    return extent_ != nullptr ? t.checkInvariants() : t.checkInvariants(micro_.page_tokens);
}

KvCacheError TableEngine::grow(RequestId owner, BlockTable const& from, std::uint32_t tokens, TableEdit& e)
{
    e = TableEdit{};
    e.table = from;
    std::vector<MappingEntry>& entries = e.table.entries_;
    std::uint16_t const cap = micro_.page_tokens;
    entries.reserve(entries.size() + tokens / cap + 2);
    // The entry that takes tokens first: the tail when it is a partial micro
    // page, written in place when the request owns it Mutable, copied to a
    // staged page when it is sealed (possibly shared with a fork).
    std::size_t open = kNoEntry;
    if (!entries.empty()) {
        MappingEntry& tail = entries.back();
        auto const [s, slot] = find(tail.handle);
        if (s == nullptr || s->valid[slot] != tail.valid_tokens) {
            return KvCacheError::InternalInvariantViolation;
        }
        bool const partial = tail.kind == PageKind::Micro && tail.valid_tokens < cap;
        if (!partial) {
            if (s->state[slot] != PageState::Sealed) {
                return KvCacheError::InternalInvariantViolation;
            }
        } else if (s->state[slot] == PageState::Mutable) {
            if (s->refs[slot] != 1 || s->owner[slot] != owner) {
                return KvCacheError::InternalInvariantViolation;
            }
            e.grown = tail.handle;
            open = entries.size() - 1;
        } else if (s->state[slot] == PageState::Sealed) {
            PageHandle copy;
            KvCacheError const err = stage(PageKind::Micro, tail.valid_tokens, copy);
            if (err != KvCacheError::None) {
                return err;
            }
            e.replaced = tail.handle;
            tail.handle = copy;
            open = entries.size() - 1;
            e.staged.emplace_back(copy, open);
        } else {
            return KvCacheError::InvalidState;
        }
    }
    std::uint32_t end = from.tokenCount();
    for (std::uint32_t left = tokens; left != 0;) {
        if (open == kNoEntry) {
            PageHandle fresh;
            KvCacheError const err = stage(PageKind::Micro, 0, fresh);
            if (err != KvCacheError::None) {
                discard(e);
                return err;
            }
            open = entries.size();
            entries.push_back(MappingEntry{end, 0, PageKind::Micro, fresh});
            e.staged.emplace_back(fresh, open);
        }
        MappingEntry& m = entries[open];
        std::uint32_t const n = std::min<std::uint32_t>(left, cap - m.valid_tokens);
        m.valid_tokens = static_cast<std::uint16_t>(m.valid_tokens + n);
        end += n;
        left -= n;
        if (m.valid_tokens == cap) {
            open = kNoEntry;
        }
    }
    e.table.version_ = from.version_ + 1;
    if (!tableWellFormed(e.table) || !editIntact(owner, e)) {
        discard(e);
        return KvCacheError::InternalInvariantViolation;
    }
    return KvCacheError::None;
}

bool TableEngine::editIntact(RequestId owner, TableEdit const& e) const
{
    for (auto const& [h, index] : e.staged) {
        auto const [s, slot] = find(h);
        if (s == nullptr || s->state[slot] != PageState::CopyTarget || s->refs[slot] != 0
            || index >= e.table.entries_.size() || e.table.entries_[index].handle != h) {
            return false;
        }
    }
    if (e.grown.isStructurallyValid()) {
        auto const [s, slot] = find(e.grown);
        if (s == nullptr || s->state[slot] != PageState::Mutable || s->refs[slot] != 1
            || s->owner[slot] != owner) {
            return false;
        }
    }
    if (e.replaced.isStructurallyValid()) {
        auto const [s, slot] = find(e.replaced);
        if (s == nullptr || s->state[slot] != PageState::Sealed || s->refs[slot] == 0) {
            return false;
        }
    }
    return true;
}

KvCacheError TableEngine::apply(RequestId owner, TableEdit const& e)
{
    if (e.replaced.isStructurallyValid()) {
        KvCacheError const err = unref(e.replaced);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    std::uint16_t const cap = micro_.page_tokens;
    // The grown tail is the table's last page that is not staged.
    if (e.grown.isStructurallyValid()) {
        auto const [s, slot] = find(e.grown);
        auto const m = std::find_if(e.table.entries_.rbegin(), e.table.entries_.rend(),
            [&](MappingEntry const& x) { return x.handle == e.grown; });
        s->valid[slot] = m->valid_tokens;
        if (m->valid_tokens == cap) {
            s->state[slot] = PageState::Sealed;
            s->owner[slot] = kInvalidRequestId;
        }
    }
    for (auto const& [h, index] : e.staged) {
        auto const [s, slot] = find(h);
        std::uint16_t const n = e.table.entries_[index].valid_tokens;
        bool const full = n == cap;
        s->valid[slot] = n;
        s->refs[slot] = 1;
        s->state[slot] = full ? PageState::Sealed : PageState::Mutable;
        s->owner[slot] = full ? kInvalidRequestId : owner;
    }
    return KvCacheError::None;
}

void TableEngine::discard(TableEdit const& e) noexcept
{
    // Newest first: the pool's LIFO free stack ends as it was before.
    for (auto it = e.staged.rbegin(); it != e.staged.rend(); ++it) {
        auto const [s, slot] = find(it->first);
        if (s != nullptr && s->state[slot] == PageState::CopyTarget && s->refs[slot] == 0) {
            static_cast<void>(retire(it->first));
        }
    }
}

// ---- requests ------------------------------------------------------------------------------

BlockTable* TableEngine::table(RequestId id) noexcept
{
    auto const f = tables_.find(id);
    return f == tables_.end() ? nullptr : &f->second;
}

BlockTable const* TableEngine::table(RequestId id) const noexcept
{
    auto const f = tables_.find(id);
    return f == tables_.end() ? nullptr : &f->second;
}

PendingToken const* TableEngine::reservation(KvTokenReservationId id) const noexcept
{
    auto const f = pending_.find(id);
    return f == pending_.end() ? nullptr : &f->second;
}

KvCacheError TableEngine::create(RequestId id)
{
    if (id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    return tables_.emplace(id, BlockTable{}).second ? KvCacheError::None : KvCacheError::RequestAlreadyExists;
}

KvCacheError TableEngine::append(RequestId id, std::uint32_t tokens)
{
    if (id == kInvalidRequestId || tokens == 0) {
        return KvCacheError::InvalidArgument;
    }
    BlockTable* t = table(id);
    if (t == nullptr) {
        return KvCacheError::RequestNotFound;
    }
    if (pending(id)) {
        return KvCacheError::RequestConflict;
    }
    if (tokens > kMaxU32 - t->tokenCount()) {
        return KvCacheError::InvalidArgument;
    }
    TableEdit e;
    KvCacheError err = grow(id, *t, tokens, e);
    if (err == KvCacheError::None && (err = apply(id, e)) != KvCacheError::None) {
        discard(e);
    }
    if (err == KvCacheError::None) {
        *t = std::move(e.table);
    }
    return err;
}

TokenReservationResult TableEngine::reserve(RequestId id, std::uint32_t expected_tokens, bool busy)
{
    TokenReservationResult r;
    r.request_id = id;
    r.logical_token_position = expected_tokens;
    BlockTable const* t = id == kInvalidRequestId ? nullptr : table(id);
    if (id == kInvalidRequestId) {
        r.error = KvCacheError::InvalidArgument;
    } else if (t == nullptr) {
        r.error = KvCacheError::RequestNotFound;
    } else if (pending(id) || busy) {
        r.error = KvCacheError::RequestConflict;
    } else if (t->tokenCount() != expected_tokens || t->version_ == kMaxU64 || expected_tokens == kMaxU32) {
        r.error = KvCacheError::InvalidState;
    }
    if (r.error != KvCacheError::None) {
        return r;
    }
    PendingToken p{id, t->version_, {}};
    r.error = grow(id, *t, 1, p.edit);
    if (r.error != KvCacheError::None) {
        return r;
    }
    KvTokenReservationId const rid = reservation_ids_.next(pending_);
    if (rid == kInvalidKvTokenReservationId) {
        discard(p.edit);
        r.error = KvCacheError::InternalInvariantViolation;
        return r;
    }
    r.before = *t;
    r.reserved = p.edit.table;
    pending_.emplace(rid, std::move(p));
    pending_of_.emplace(id, rid);
    r.reservation_id = rid;
    return r;
}

KvCacheError TableEngine::commit(KvTokenReservationId rid)
{
    if (rid == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    auto const f = pending_.find(rid);
    if (f == pending_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    PendingToken& p = f->second;
    BlockTable* t = table(p.request);
    if (t == nullptr || t->version_ != p.base_version) {
        return KvCacheError::RequestConflict;
    }
    if (!editIntact(p.request, p.edit)) {
        return KvCacheError::InternalInvariantViolation;
    }
    KvCacheError const err = apply(p.request, p.edit);
    if (err != KvCacheError::None) {
        return err;
    }
    *t = std::move(p.edit.table);
    pending_of_.erase(p.request);
    pending_.erase(f);
    return KvCacheError::None;
}

KvCacheError TableEngine::rollback(KvTokenReservationId rid)
{
    if (rid == kInvalidKvTokenReservationId) {
        return KvCacheError::InvalidArgument;
    }
    auto const f = pending_.find(rid);
    if (f == pending_.end()) {
        return KvCacheError::TokenReservationNotFound;
    }
    // A reservation stages at most one page; a lease taken on it keeps the
    // page Retiring until released.
    for (auto const& staged : f->second.edit.staged) {
        KvCacheError const err = retire(staged.first);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    pending_of_.erase(f->second.request);
    pending_.erase(f);
    return KvCacheError::None;
}

KvCacheError TableEngine::seal(RequestId id)
{
    if (id == kInvalidRequestId) {
        return KvCacheError::InvalidArgument;
    }
    BlockTable const* t = table(id);
    if (t == nullptr) {
        return KvCacheError::RequestNotFound;
    }
    if (pending(id)) {
        return KvCacheError::RequestConflict;
    }
    if (t->entries_.empty()) {
        return KvCacheError::InvalidState;
    }
    MappingEntry const& tail = t->entries_.back();
    auto const [s, slot] = find(tail.handle);
    if (s == nullptr || s->valid[slot] != tail.valid_tokens) {
        return KvCacheError::InternalInvariantViolation;
    }
    switch (s->state[slot]) {
    case PageState::Sealed:
        return KvCacheError::None;
    case PageState::Mutable:
        if (s->refs[slot] == 1 && s->owner[slot] == id) {
            // Same mapping, so the table version does not move.
            s->state[slot] = PageState::Sealed;
            s->owner[slot] = kInvalidRequestId;
            return KvCacheError::None;
        }
        return KvCacheError::InvalidState;
    default:
        return KvCacheError::InvalidState;
    }
}

KvCacheError TableEngine::fork(RequestId source, RequestId child)
{
    if (source == kInvalidRequestId || child == kInvalidRequestId || source == child) {
        return KvCacheError::InvalidArgument;
    }
    BlockTable const* t = table(source);
    if (t == nullptr) {
        return KvCacheError::RequestNotFound;
    }
    if (pending(source)) {
        return KvCacheError::RequestConflict;
    }
    if (table(child) != nullptr) {
        return KvCacheError::RequestAlreadyExists;
    }
    std::vector<MappingEntry> const& entries = t->entries_;
    for (std::size_t i = 0; i < entries.size(); ++i) {
        auto const [s, slot] = find(entries[i].handle);
        if (s == nullptr || s->valid[slot] != entries[i].valid_tokens || s->refs[slot] == 0
            || s->refs[slot] == kMaxU32) {
            return KvCacheError::InternalInvariantViolation;
        }
        PageState const st = s->state[slot];
        bool const owned_tail = st == PageState::Mutable && i + 1 == entries.size() && s->refs[slot] == 1
            && s->owner[slot] == source;
        if (st == PageState::Mutable && !owned_tail) {
            return KvCacheError::InternalInvariantViolation;
        }
        if (st != PageState::Mutable && st != PageState::Sealed) {
            return KvCacheError::InvalidState;
        }
    }
    BlockTable copy = *t;
    copy.version_ = copy.entries_.empty() ? 0 : 1;
    // The emplace may rehash: the source table is not touched after it.
    auto const inserted = tables_.emplace(child, std::move(copy));
    // Every page is now shared; a Mutable tail is sealed so that the next
    // write on either side copies it.
    for (MappingEntry const& m : inserted.first->second.entries_) {
        auto const [s, slot] = find(m.handle);
        if (s->state[slot] == PageState::Mutable) {
            s->state[slot] = PageState::Sealed;
            s->owner[slot] = kInvalidRequestId;
        }
        ++s->refs[slot];
    }
    return KvCacheError::None;
}

KvCacheError TableEngine::release(RequestId id)
{
    auto const f = tables_.find(id);
    if (f == tables_.end()) {
        return KvCacheError::RequestNotFound;
    }
    for (MappingEntry const& m : f->second.entries_) {
        auto const [s, slot] = find(m.handle);
        if (s == nullptr || s->refs[slot] == 0 || s->state[slot] == PageState::Free
            || s->state[slot] == PageState::CopyTarget) {
            return KvCacheError::InternalInvariantViolation;
        }
    }
    for (MappingEntry const& m : f->second.entries_) {
        KvCacheError const err = unref(m.handle);
        if (err != KvCacheError::None) {
            return err;
        }
    }
    tables_.erase(f);
    return KvCacheError::None;
}

// ---- audit -------------------------------------------------------------------------------

bool TableEngine::auditTables(ExpectedCounts& micro, ExpectedCounts* extent) const
{
    std::uint16_t const cap = micro_.page_tokens;
    for (auto const& [rid, t] : tables_) {
        if (rid == kInvalidRequestId || !tableWellFormed(t)) {
            return false;
        }
        for (std::size_t i = 0; i < t.entries_.size(); ++i) {
            MappingEntry const& m = t.entries_[i];
            auto const [s, slot] = find(m.handle);
            ExpectedCounts* x = m.kind == PageKind::Extent ? extent : &micro;
            if (s == nullptr || x == nullptr || s->valid[slot] != m.valid_tokens || s->refs[slot] == 0
                || x->refs[slot] == kMaxU32) {
                return false;
            }
            PageState const st = s->state[slot];
            bool const ok = st == PageState::Sealed
                ? s->owner[slot] == kInvalidRequestId
                : st == PageState::Mutable && i + 1 == t.entries_.size() && m.kind == PageKind::Micro
                    && s->refs[slot] == 1 && s->owner[slot] == rid && s->valid[slot] != 0
                    && s->valid[slot] < cap;
            if (!ok) {
                return false;
            }
            ++x->refs[slot];
        }
    }
    if (pending_.size() != pending_of_.size()) {
        return false;
    }
    for (auto const& [rid, p] : pending_) {
        BlockTable const* t = table(p.request);
        auto const back = pending_of_.find(p.request);
        if (rid == kInvalidKvTokenReservationId || t == nullptr || back == pending_of_.end()
            || back->second != rid || !tableWellFormed(p.edit.table) || t->version_ != p.base_version
            || p.edit.table.version_ != t->version_ + 1 || p.edit.table.tokenCount() != t->tokenCount() + 1) {
            return false;
        }
        // The token goes either into the request's Mutable tail or onto one
        // staged page (a fresh page, or the copy of a sealed tail).
        bool const staged = p.edit.staged.size() == 1;
        if (staged == p.edit.grown.isStructurallyValid() || p.edit.staged.size() > 1) {
            return false;
        }
        if (!editIntact(p.request, p.edit)) {
            return false;
        }
        if (staged) {
            PageHandle const h = p.edit.staged.front().first;
            auto const [s, slot] = find(h);
            std::uint16_t const copied = p.edit.replaced.isStructurallyValid()
                ? static_cast<std::uint16_t>(p.edit.table.entries_.back().valid_tokens - 1) : 0;
            if (h.kind != PageKind::Micro || micro.staged[slot] != 0 || s->pins[slot] != 0
                || s->valid[slot] != copied) {
                return false;
            }
            micro.staged[slot] = 1;
        }
        for (PageHandle const h : {p.edit.grown, p.edit.replaced}) {
            if (h.isStructurallyValid() && (t->entries_.empty() || t->entries_.back().handle != h)) {
                return false;
            }
        }
    }
    return true;
}

bool TableEngine::auditSlots(PageSlots const& s, ExpectedCounts const& x) const
{
    if (!s.pool.checkInvariants()) {
        return false;
    }
    std::uint32_t in_use = 0;
    for (std::uint32_t i = 0; i < s.size(); ++i) {
        PageState const st = s.state[i];
        bool const counted = x.refs[i] != 0 || x.pins[i] != 0 || x.readers[i] != 0 || x.staged[i] != 0;
        if (st == PageState::Free) {
            if (counted || s.valid[i] != 0 || s.refs[i] != 0 || s.pins[i] != 0 || s.readers[i] != 0
                || s.owner[i] != kInvalidRequestId) {
                return false;
            }
            continue;
        }
        ++in_use;
        if (s.generation[i] == PageHandle::kInvalidGeneration || s.pool.validate(s.handleOf(i)) != PagePoolError::None
            || s.refs[i] != x.refs[i] || s.pins[i] != x.pins[i] || s.readers[i] != x.readers[i]) {
            return false;
        }
        bool const target = x.staged[i] != 0;
        bool const ownerless = s.owner[i] == kInvalidRequestId;
        bool ok = false;
        switch (st) {
        case PageState::Mutable:
            ok = s.kind == PageKind::Micro && s.refs[i] == 1 && s.valid[i] != 0 && s.valid[i] < s.page_tokens
                && !ownerless && s.pins[i] == 0 && !target;
            break;
        case PageState::Sealed:
            ok = s.refs[i] != 0 && s.valid[i] != 0 && s.valid[i] <= s.page_tokens && ownerless && !target;
            break;
        case PageState::CopyTarget:
            ok = target && s.refs[i] == 0 && s.pins[i] == 0 && ownerless
                && (s.kind == PageKind::Extent ? s.valid[i] == s.page_tokens : s.valid[i] < s.page_tokens);
            break;
        case PageState::Retiring:
            ok = s.refs[i] == 0 && ownerless && !target && (s.pins[i] != 0 || s.readers[i] != 0);
            break;
        default:
            break;
        }
        if (!ok) {
            return false;
        }
    }
    PagePoolSnapshot const snap = s.pool.snapshot();
    return snap.allocated_slots == in_use && snap.capacityBalanced();
}

} // namespace kimkvcache
