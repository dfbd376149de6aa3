// The page-table engine behind both KV metadata runtimes.
//
// KvCacheManager (8-token micro pages + 64-token extent pages, promotion,
// leases) and FixedPageManager (one pool of tokens_per_page pages) are two
// configurations of this engine. It owns:
//
//  * one PageSlots per pool: the slot allocator plus every slot's record
//    kept as parallel arrays (state, last issued generation, valid tokens,
//    table references, promotion pins, in-flight readers, mutable owner);
//  * the committed block table of every request;
//  * pending token reservations.
//
// Every mutation of a table goes through a TableEdit: a candidate table plus
// the pages staged for it (taken from the pool as unreferenced CopyTarget
// pages, in allocation order), the request's own Mutable tail if the edit
// grows it in place, and the sealed tail the edit replaces by a copy. An
// edit is built by grow() (append of n tokens = reservation of 1 token with
// n = 1), then either applied (no-fail: page states published, the replaced
// tail unreferenced) or discarded (staged pages returned newest first, which
// restores the pool's free stack). Promotion and leases live in
// KvCacheManager on top of the same records.
//
// Observable behaviour (error precedence, slot numbers and generations,
// versions, counters) is that of the reference runtime
// (src/runtime/*.cpp, src/fixed/*.cpp); the parity tests replay identical
// op streams on both.
#pragma once

#include "kv_types.h"
#include "page_pool.h"

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <unordered_map>
#include <utility>
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

// Ids handed out from a counter that wraps and never yields 0 or an id that
// is still live in `live`.
class IdSequence final {
public:
    template <typename Map>
    [[nodiscard]] std::uint64_t next(Map const& live)
    {
        // Among live.size() + 1 consecutive non-zero candidates one is free.
        for (std::size_t tries = live.size() + 1; tries != 0; --tries) {
            std::uint64_t const id = counter_;
            counter_ = counter_ + 1 == 0 ? 1 : counter_ + 1;
            if (id != 0 && live.count(id) == 0) {
                return id;
            }
        }
        return 0;
    }

private:
    std::uint64_t counter_{1};
};

// One pool's slots: allocator + per-slot records as parallel arrays.
class PageSlots final {
public:
    PageSlots(PageKind kind, std::uint32_t capacity, std::uint16_t page_tokens);

    [[nodiscard]] std::uint32_t size() const noexcept { return static_cast<std::uint32_t>(state.size()); }
    // Slot of a handle whose generation is the slot's last issued one (its
    // record may be Free again); -1 otherwise.
    [[nodiscard]] std::int64_t slotOf(PageHandle h) const noexcept
    {
        if (!h.isStructurallyValid() || h.kind != kind || h.slot >= size()
            || generation[h.slot] != h.generation) {
            return -1;
        }
        return h.slot;
    }
    [[nodiscard]] PageHandle handleOf(std::uint32_t slot) const noexcept
    {
        return PageHandle{kind, slot, generation[slot]};
    }
    // Slot back to the Free record (the generation stays: it names the last
    // handle issued for the slot).
    void clear(std::uint32_t slot) noexcept;

    PageKind kind;
    std::uint16_t page_tokens;
    PagePool pool;
    std::vector<PageState> state;
    std::vector<std::uint32_t> generation;
    std::vector<std::uint16_t> valid;
    std::vector<std::uint32_t> refs;
    std::vector<std::uint32_t> pins;
    std::vector<std::uint32_t> readers;
    std::vector<RequestId> owner;
};

// A pending change of one request's table.
struct TableEdit final {
    BlockTable table{};                                       // candidate
    std::vector<std::pair<PageHandle, std::size_t>> staged{};  // page, entry index
    PageHandle grown{PageHandle::invalid()};                  // Mutable tail grown in place
    PageHandle replaced{PageHandle::invalid()};               // sealed tail replaced by a copy
};

struct PendingToken final {
    RequestId request{kInvalidRequestId};
    std::uint64_t base_version{0};
    TableEdit edit{};
};

// Reference counts recomputed from the tables, reservations, promotions and
// leases, compared with the slot records by TableEngine::audit.
struct ExpectedCounts final {
    std::vector<std::uint32_t> refs, pins, readers;
    std::vector<std::uint8_t> staged;
    explicit ExpectedCounts(std::uint32_t n) : refs(n, 0), pins(n, 0), readers(n, 0), staged(n, 0) {}
};

class TableEngine final {
public:
    // extent_capacity 0: a single-pool (fixed-page) engine. Throws
    // std::invalid_argument for a zero micro capacity or page size.
    TableEngine(std::uint16_t micro_tokens, std::uint32_t micro_capacity, std::uint32_t extent_capacity);

    [[nodiscard]] std::uint16_t microTokens() const noexcept { return micro_.page_tokens; }
    [[nodiscard]] PageSlots& slots(PageKind k) noexcept { return k == PageKind::Extent ? *extent_ : micro_; }
    [[nodiscard]] PageSlots const& slots(PageKind k) const noexcept
    {
        return k == PageKind::Extent ? *extent_ : micro_;
    }
    [[nodiscard]] bool hasExtents() const noexcept { return extent_ != nullptr; }
    // Slots of the pool a handle names, or null (a fixed engine has no extents).
    [[nodiscard]] PageSlots const* poolOf(PageHandle h) const noexcept
    {
        return h.kind == PageKind::Extent ? extent_.get() : (h.kind == PageKind::Micro ? &micro_ : nullptr);
    }
    [[nodiscard]] PageSlots* poolOf(PageHandle h) noexcept
    {
        return const_cast<PageSlots*>(static_cast<TableEngine const*>(this)->poolOf(h));
    }
    // The live record of a handle: (pool, slot), or (null, 0).
    [[nodiscard]] std::pair<PageSlots*, std::uint32_t> find(PageHandle h) noexcept;
    [[nodiscard]] std::pair<PageSlots const*, std::uint32_t> find(PageHandle h) const noexcept;

    // ---- page transitions ----
    // A fresh unreferenced CopyTarget page holding `valid` tokens.
    [[nodiscard]] KvCacheError stage(PageKind kind, std::uint16_t valid, PageHandle& out);
    // An unreferenced page leaves: Retiring while pinned or read, else back
    // to its pool.
    [[nodiscard]] KvCacheError retire(PageHandle h);
    // One table reference less; the last one retires the page.
    [[nodiscard]] KvCacheError unref(PageHandle h);

    // ---- table edits ----
    [[nodiscard]] KvCacheError grow(RequestId owner, BlockTable const& from, std::uint32_t tokens,
        TableEdit& edit);
    // Checks that the pages an edit touches are still as grow() left them.
    [[nodiscard]] bool editIntact(RequestId owner, TableEdit const& edit) const;
    // Publishes the page states of an intact edit; the caller installs the table.
    [[nodiscard]] KvCacheError apply(RequestId owner, TableEdit const& edit);
    void discard(TableEdit const& edit) noexcept;
    [[nodiscard]] bool tableWellFormed(BlockTable const& t) const;

    // ---- requests ----
    [[nodiscard]] BlockTable* table(RequestId id) noexcept;
    [[nodiscard]] BlockTable const* table(RequestId id) const noexcept;
    [[nodiscard]] bool pending(RequestId id) const noexcept { return pending_of_.count(id) != 0; }

    [[nodiscard]] KvCacheError create(RequestId id);
    [[nodiscard]] KvCacheError append(RequestId id, std::uint32_t tokens);
    // `busy`: the caller knows of other work on the request (a pending
    // promotion) that forbids a reservation.
    [[nodiscard]] TokenReservationResult reserve(RequestId id, std::uint32_t expected_tokens, bool busy);
    [[nodiscard]] KvCacheError commit(KvTokenReservationId id);
    [[nodiscard]] KvCacheError rollback(KvTokenReservationId id);
    [[nodiscard]] KvCacheError seal(RequestId id);
    [[nodiscard]] KvCacheError fork(RequestId source, RequestId child);
    // Drops the request's references (its pending promotions already undone).
    [[nodiscard]] KvCacheError release(RequestId id);

    [[nodiscard]] PendingToken const* reservation(KvTokenReservationId id) const noexcept;
    [[nodiscard]] std::size_t requestCount() const noexcept { return tables_.size(); }
    [[nodiscard]] std::size_t reservationCount() const noexcept { return pending_.size(); }
    [[nodiscard]] std::uint64_t peakAllocated() const noexcept { return peak_allocated_; }
    [[nodiscard]] std::unordered_map<RequestId, BlockTable> const& tables() const noexcept { return tables_; }

    // Recounts references from the tables and staged pages from the pending
    // reservations into `expect` (one per pool, indexed by PageKind), then
    // checks every slot record against them and against its pool.
    [[nodiscard]] bool auditTables(ExpectedCounts& micro, ExpectedCounts* extent) const;
    [[nodiscard]] bool auditSlots(PageSlots const& s, ExpectedCounts const& expect) const;

private:
    PageSlots micro_;
    std::unique_ptr<PageSlots> extent_;
    std::unordered_map<RequestId, BlockTable> tables_;
    std::unordered_map<KvTokenReservationId, PendingToken> pending_;
    std::unordered_map<RequestId, KvTokenReservationId> pending_of_;
    IdSequence reservation_ids_;
    std::uint64_t peak_allocated_{0};
};

} // namespace kimkvcache
