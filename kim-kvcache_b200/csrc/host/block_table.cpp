// Block table lookup and structural checks
// (reference: src/core/block_table.cpp:12-130).
#include "kv_types.h"

#include <algorithm>
#include <cstdint>
#include <vector>

namespace kimkvcache {
namespace {

bool tableIsWellFormed(std::vector<MappingEntry> const& entries,
    std::uint16_t uniform_capacity)
{
    std::uint64_t next_begin = 0;
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
    }
    // One physical page mapped twice: the same verdict as comparing every
    // pair of entries, from a sorted copy of the handles (tables of a few
    // thousand tokens hold tens of entries and are checked on every token
    // reservation, where the pairwise scan dominated the host time).
    std::uint64_t local[128];
    std::vector<std::uint64_t> heap;
    std::uint64_t* keys = local;
    if (entries.size() > 128) {
        heap.resize(entries.size());
        keys = heap.data();
    }
    std::size_t n = 0;
    for (MappingEntry const& entry : entries) {
        // kind (8 bits) | slot (32 bits) | generation (24 low bits): equal
        // keys only for equal handles when generations fit 24 bits; larger
        // generations fall back to the exact pairwise comparison below.
        if (entry.handle.generation >= (1u << 24)) {
            for (std::size_t i = 1; i < entries.size(); ++i) {
                for (std::size_t j = 0; j < i; ++j) {
                    if (entries[j].handle == entries[i].handle) {
                        return false;
                    }
                }
            }
            return true;
        }
        keys[n++] = (static_cast<std::uint64_t>(static_cast<std::uint8_t>(entry.handle.kind)) << 56)
            | (static_cast<std::uint64_t>(entry.handle.slot) << 24) | entry.handle.generation;
    }
    std::sort(keys, keys + n);
    return std::adjacent_find(keys, keys + n) == keys + n;
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
