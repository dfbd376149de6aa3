// Block table lookup and structural checks
// (reference: src/core/block_table.cpp:12-130).
#include "kv_types.h"

#include <algorithm>
#include <cstdint>
#include <limits>
#include <tuple>
#include <vector>

namespace kimkvcache {
namespace {

bool tableIsWellFormed(std::vector<MappingEntry> const& entries,
    std::uint16_t uniform_capacity)
{
    std::uint64_t next_begin = 0;
    std::uint32_t max_slot = 0;
    for (std::size_t i = 0; i < entries.size(); ++i) {
        MappingEntry const& entry = entries[i];
        if (!entry.handle.isStructurallyValid() || entry.kind != entry.handle.kind) {
            return false;
        }
        std::uint16_t const capacity = uniform_capacity != 0
            ? uniform_capacity : pageTokenCapacity(entry.kind);
        if (capacity == 0 || entry.valid_tokens == 0 || entry.valid_tokens > capacity) {
            return false;
        }
        if (entry.logical_token_begin != next_begin) {
            return false;
        }
        next_begin += entry.valid_tokens;
        if (next_begin > std::numeric_limits<std::uint32_t>::max()) {
            return false;
        }
        max_slot = std::max(max_slot, entry.handle.slot);
    }
    // One physical page mapped twice: the same verdict as comparing every
    // pair of entries. Tables of a few thousand tokens hold tens of entries
    // and are checked on every token reservation, so the common case marks
    // each (kind, slot) in a per-thread bitmap and clears the marks again:
    // a table whose slots are all distinct has no equal handles. A slot seen
    // twice (possibly with another generation, which is not a duplicate)
    // or a slot beyond the bitmap falls back to sorting the full handles.
    constexpr std::uint32_t kBitmapSlots = 1u << 22;
    thread_local std::vector<std::uint64_t> tls_marks[2];
    std::vector<std::uint64_t>* const marks = tls_marks;  // one TLS lookup
    bool distinct = max_slot < kBitmapSlots;
    std::size_t marked = 0;
    if (distinct) {
        std::size_t const words = (max_slot >> 6) + 1;
        for (int k = 0; k < 2; ++k) {
            if (marks[k].size() < words) {
                marks[k].resize(words, 0);
            }
        }
        std::uint64_t* const bits[2] = {marks[0].data(), marks[1].data()};
        // Consecutive entries usually sit in neighbouring slots of one word:
        // the word being filled stays in a register and is written back
        // when the next entry moves to another word.
        std::uint64_t* cur = nullptr;
        std::uint64_t cur_bits = 0;
        for (; marked < entries.size(); ++marked) {
            PageHandle const h = entries[marked].handle;
            std::uint64_t* const word = bits[h.kind == PageKind::Micro ? 0 : 1] + (h.slot >> 6);
            if (word != cur) {
                if (cur != nullptr) {
                    *cur = cur_bits;
                }
                cur = word;
                cur_bits = *word;
            }
            std::uint64_t const bit = std::uint64_t{1} << (h.slot & 63);
            if (cur_bits & bit) {
                distinct = false;
                break;
            }
            cur_bits |= bit;
        }
        if (cur != nullptr) {
            *cur = cur_bits;
        }
        // Every mark in a touched word belongs to this table: clear whole words.
        for (std::size_t i = 0; i < marked; ++i) {
            PageHandle const h = entries[i].handle;
            bits[h.kind == PageKind::Micro ? 0 : 1][h.slot >> 6] = 0;
        }
    }
    if (distinct) {
        return true;
    }
    std::vector<PageHandle> handles;
    handles.reserve(entries.size());
    for (MappingEntry const& entry : entries) {
        handles.push_back(entry.handle);
    }
    std::sort(handles.begin(), handles.end(), [](PageHandle a, PageHandle b) {
        return std::tie(a.kind, a.slot, a.generation) < std::tie(b.kind, b.slot, b.generation);
    });
    return std::adjacent_find(handles.begin(), handles.end()) == handles.end();
}

} // namespace

MappingEntry const* BlockTable::find(std::uint32_t logical_token) const noexcept
{
    auto const after = std::upper_bound(entries_.begin(), entries_.end(), logical_token,
        [](std::uint32_t token, MappingEntry const& e) { return token < e.logical_token_begin; });
    if (after == entries_.begin()) {
        return nullptr;
    }
    MappingEntry const& candidate = *(after - 1);
    return logical_token < candidate.logicalTokenEnd() ? &candidate : nullptr;
}

bool BlockTable::checkInvariants() const
{
    return tableIsWellFormed(entries_, 0);
}

bool BlockTable::checkInvariants(std::uint16_t uniform_page_token_capacity) const
{
    return uniform_page_token_capacity != 0
        && tableIsWellFormed(entries_, uniform_page_token_capacity);
}

} // namespace kimkvcache
