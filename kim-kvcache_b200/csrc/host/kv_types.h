// Core paging vocabulary of the token loop: page kinds, handles, states,
// error codes, the per-page [layer][K/V][token][head][dim] layout and the
// request block table.
//
// Names and numeric values mirror the reference runtime so that callers of
// kim-kvcache compile unchanged against this library:
//   include/kim-kv/core/page_types.h:8-67     (PageKind, PagePoolError)
//   include/kim-kv/core/page_handle.h:10-47   (PageHandle)
//   include/kim-kv/core/page_state.h:9-98     (capacities, PageState, KvCacheError)
//   include/kim-kv/core/kv_layout.h:19-106    (KvLayout)
//   include/kim-kv/core/block_table.h:13-72   (MappingEntry, BlockTable)
#pragma once

#include <cstddef>
#include <cstdint>
#include <limits>
#include <string_view>
#include <vector>

namespace kimkvcache {

enum class PageKind : std::uint8_t { Micro, Extent };

[[nodiscard]] constexpr bool isKnownPageKind(PageKind kind) noexcept
{
    return kind == PageKind::Micro || kind == PageKind::Extent;
}

[[nodiscard]] constexpr std::string_view toString(PageKind kind) noexcept
{
    return kind == PageKind::Micro ? "micro"
        : kind == PageKind::Extent ? "extent" : "unknown";
}

enum class PagePoolError : std::uint8_t {
    None,
    Exhausted,
    InvalidHandle,
    WrongKind,
    OutOfRange,
    StaleGeneration,
    AlreadyFree,
};

// A physical page: pool kind + slot + allocation generation. Generation 0 is
// reserved for "never valid", so a default handle is structurally invalid.
struct PageHandle final {
    static constexpr std::uint32_t kInvalidSlot =
        std::numeric_limits<std::uint32_t>::max();
    static constexpr std::uint32_t kInvalidGeneration = 0;

    PageKind kind{PageKind::Micro};
    std::uint32_t slot{kInvalidSlot};
    std::uint32_t generation{kInvalidGeneration};

    [[nodiscard]] static constexpr PageHandle invalid() noexcept { return {}; }

    [[nodiscard]] constexpr bool isStructurallyValid() const noexcept
    {
        return isKnownPageKind(kind) && slot != kInvalidSlot
            && generation != kInvalidGeneration;
    }

    friend constexpr bool operator==(PageHandle a, PageHandle b) noexcept
    {
        return a.kind == b.kind && a.slot == b.slot
            && a.generation == b.generation;
    }
    friend constexpr bool operator!=(PageHandle a, PageHandle b) noexcept
    {
        return !(a == b);
    }
};

constexpr std::uint16_t kMicroPageTokenCapacity = 8;
constexpr std::uint16_t kExtentPageTokenCapacity = 64;

[[nodiscard]] constexpr std::uint16_t pageTokenCapacity(PageKind kind) noexcept
{
    return kind == PageKind::Micro ? kMicroPageTokenCapacity
        : kind == PageKind::Extent ? kExtentPageTokenCapacity : 0;
}

enum class PageState : std::uint8_t { Free, Mutable, Sealed, CopyTarget, Retiring };

enum class KvCacheError : std::uint8_t {
    None,
    InvalidArgument,
    RequestNotFound,
    RequestAlreadyExists,
    RequestConflict,
    ResourceExhausted,
    InvalidState,
    TokenReservationNotFound,
    PromotionNotEligible,
    PromotionNotFound,
    PromotionConflict,
    InternalInvariantViolation,
};

[[nodiscard]] std::string_view toString(KvCacheError error) noexcept;
[[nodiscard]] std::string_view toString(PageState state) noexcept;

// FP16 bit pattern; host code never needs the CUDA half type.
using KvScalar = std::uint16_t;

enum class KvComponent : std::uint8_t { Key = 0, Value = 1 };

// Element layout of one page: [layer][K/V][token][head][dim]. A page holds
// every layer of its tokens, so per layer a micro page's K (or V) block is
// 8 tokens x heads x dim contiguous elements.
struct KvLayout final {
    std::uint32_t layer_count{0};
    std::uint32_t kv_head_count{0};
    std::uint32_t head_dimension{0};

    [[nodiscard]] constexpr bool valid() const noexcept
    {
        return layer_count != 0 && kv_head_count != 0 && head_dimension != 0;
    }

    [[nodiscard]] bool elementsPerToken(std::size_t& out) const noexcept
    {
        if (!valid()) {
            return false;
        }
        return mul(layer_count, 2, out) && mul(out, kv_head_count, out)
            && mul(out, head_dimension, out);
    }

    [[nodiscard]] bool elementsForTokens(
        std::uint32_t tokens, std::size_t& out) const noexcept
    {
        std::size_t per = 0;
        return elementsPerToken(per) && mul(per, tokens, out);
    }

    [[nodiscard]] bool bytesForTokens(
        std::uint32_t tokens, std::size_t& out) const noexcept
    {
        std::size_t elements = 0;
        return elementsForTokens(tokens, elements)
            && mul(elements, sizeof(KvScalar), out);
    }

    [[nodiscard]] bool pageElements(PageKind kind, std::size_t& out) const noexcept
    {
        return elementsForTokens(pageTokenCapacity(kind), out);
    }

    [[nodiscard]] std::size_t offset(std::uint32_t layer, KvComponent component,
        std::uint32_t token, std::uint32_t head, std::uint32_t dim,
        std::uint32_t token_capacity) const noexcept
    {
        std::size_t index = static_cast<std::size_t>(layer) * 2
            + static_cast<std::size_t>(component);
        index = index * token_capacity + token;
        index = index * kv_head_count + head;
        return index * head_dimension + dim;
    }

private:
    static bool mul(std::size_t a, std::size_t b, std::size_t& out) noexcept
    {
        if (a != 0 && b > std::numeric_limits<std::size_t>::max() / a) {
            return false;
        }
        out = a * b;
        return true;
    }
};

// One logical run [logical_token_begin, +valid_tokens) of a request mapped to
// one physical page.
struct MappingEntry final {
    std::uint32_t logical_token_begin{0};
    std::uint16_t valid_tokens{0};
    PageKind kind{PageKind::Micro};
    PageHandle handle{PageHandle::invalid()};

    [[nodiscard]] constexpr std::uint32_t logicalTokenEnd() const noexcept
    {
        return logical_token_begin + valid_tokens;
    }

    friend constexpr bool operator==(MappingEntry const& a, MappingEntry const& b) noexcept
    {
        return a.logical_token_begin == b.logical_token_begin
            && a.valid_tokens == b.valid_tokens && a.kind == b.kind
            && a.handle == b.handle;
    }
    friend constexpr bool operator!=(MappingEntry const& a, MappingEntry const& b) noexcept
    {
        return !(a == b);
    }
};

class KvCacheManager;

// A request's page table: entries are contiguous from token 0, each entry's
// kind equals its handle's kind, no handle appears twice, and the version
// counts every committed change of the mapping.
class BlockTable final {
public:
    BlockTable() = default;

    [[nodiscard]] std::uint64_t version() const noexcept { return version_; }
    [[nodiscard]] std::uint32_t tokenCount() const noexcept
    {
        return entries_.empty() ? 0 : entries_.back().logicalTokenEnd();
    }
    [[nodiscard]] bool empty() const noexcept { return entries_.empty(); }
    [[nodiscard]] std::vector<MappingEntry> const& entries() const noexcept
    {
        return entries_;
    }

    // Entry covering a logical token (binary search), nullptr when unmapped.
    [[nodiscard]] MappingEntry const* find(std::uint32_t logical_token) const noexcept;

    [[nodiscard]] bool checkInvariants() const;
    [[nodiscard]] bool checkInvariants(std::uint16_t uniform_page_token_capacity) const;

private:
    friend class KvCacheManager;
    friend class FixedPageManager;
    friend class TableEngine;
    std::vector<MappingEntry> entries_;
    std::uint64_t version_{0};
};

} // namespace kimkvcache
