// Property test of the block-table structure check: on random tables built to
// collide (shared slots, equal slots with other generations, slots on both
// sides of the per-thread bitmap's limit, both page kinds), the verdict of
// BlockTable's check must equal the definition it implements: contiguous
// entries from token 0, kinds and capacities valid, and no page handle twice
// (every pair compared). Each table is checked twice, so marks left behind by
// one call would show up as a wrong verdict on the next.
#include "block_table.cpp"

#include <cstdio>
#include <random>

using namespace kimkvcache;

namespace {

bool byDefinition(std::vector<MappingEntry> const& e)
{
    std::uint64_t next = 0;
    for (MappingEntry const& x : e) {
        if (!x.handle.isStructurallyValid() || x.kind != x.handle.kind) {
            return false;
        }
        std::uint16_t const cap = pageTokenCapacity(x.kind);
        if (cap == 0 || x.valid_tokens == 0 || x.valid_tokens > cap || x.logical_token_begin != next) {
            return false;
        }
        next += x.valid_tokens;
    }
    for (std::size_t i = 1; i < e.size(); ++i) {
        for (std::size_t j = 0; j < i; ++j) {
            if (e[i].handle == e[j].handle) {
                return false;
            }
        }
    }
    return true;
}

} // namespace

int main(int argc, char** argv)
{
    long const tables = argc > 1 ? std::atol(argv[1]) : 100000;
    std::mt19937_64 rng(7);
    long mismatches = 0, well_formed = 0;
    for (long it = 0; it < tables; ++it) {
        std::size_t const len = rng() % 200;
        std::uint32_t const range = it % 4 == 0 ? 8u : it % 4 == 1 ? 300u : it % 4 == 2 ? (1u << 23) : 100000u;
        std::uint32_t const gens = it % 3 == 0 ? 1u : 3u;
        std::vector<MappingEntry> e;
        std::uint32_t begin = 0;
        for (std::size_t i = 0; i < len; ++i) {
            PageKind const k = (rng() & 1) ? PageKind::Micro : PageKind::Extent;
            std::uint16_t const n = static_cast<std::uint16_t>(k == PageKind::Micro ? 1 + rng() % 8 : 1 + rng() % 64);
            std::uint32_t const slot = it % 5 == 0 ? static_cast<std::uint32_t>(rng() % range) + (1u << 22) - 4
                                                   : static_cast<std::uint32_t>(rng() % range);
            e.push_back(MappingEntry{begin, n, k, PageHandle{k, slot, 1 + static_cast<std::uint32_t>(rng() % gens)}});
            begin += n;
        }
        bool const expected = byDefinition(e);
        well_formed += expected;
        mismatches += tableIsWellFormed(e, 0) != expected;
        mismatches += tableIsWellFormed(e, 0) != expected;
    }
    std::printf("tables %ld well_formed %ld mismatches %ld\n", tables, well_formed, mismatches);
    return mismatches == 0 && well_formed > tables / 10 && well_formed < tables ? 0 : 1;
}
