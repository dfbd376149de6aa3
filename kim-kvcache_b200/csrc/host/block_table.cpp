// Block table lookup and structural checks
// (reference: src/core/block_table.cpp:12-130).
#include "kv_types.h"

#include <algorithm>

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
        for (std::size_t j = 0; j < i; ++j) {
            if (entries[j].handle == entry.handle) {
                return false;  // one physical page mapped twice
            }
        }
    }
    return true;
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
