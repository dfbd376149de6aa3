// Slot allocator for one page kind (reference: include/kim-kv/core/page_pool.h:42-99,
// src/core/page_pool.cpp:8-265).
//
// Allocation order is part of the observable contract (slot numbers appear in
// page tables and device addresses): the free list is a LIFO stack seeded so
// that a fresh pool hands out slots 0, 1, 2, ...; a released slot is the next
// one handed out. Every allocation bumps the slot's generation (skipping the
// reserved value 0) so stale handles are detected.
#pragma once

#include "kv_types.h"

#include <cstdint>
#include <mutex>
#include <vector>

namespace kimkvcache {

struct PageAllocationResult final {
    PagePoolError error{PagePoolError::None};
    PageHandle handle{PageHandle::invalid()};

    [[nodiscard]] constexpr bool ok() const noexcept { return error == PagePoolError::None; }
    [[nodiscard]] explicit constexpr operator bool() const noexcept { return ok(); }
};

struct PagePoolSnapshot final {
    PageKind kind{PageKind::Micro};
    std::uint32_t total_slots{0};
    std::uint32_t free_slots{0};
    std::uint32_t allocated_slots{0};
    std::uint64_t successful_allocations{0};
    std::uint64_t successful_releases{0};
    std::uint64_t failed_allocations{0};
    std::uint64_t rejected_releases{0};

    [[nodiscard]] constexpr bool capacityBalanced() const noexcept
    {
        return total_slots == free_slots + allocated_slots;
    }
};

class PagePool final {
public:
    // Throws std::invalid_argument for an unknown kind or zero capacity.
    PagePool(PageKind kind, std::uint32_t capacity);

    PagePool(PagePool const&) = delete;
    PagePool& operator=(PagePool const&) = delete;

    [[nodiscard]] PageKind kind() const noexcept { return kind_; }
    [[nodiscard]] std::uint32_t capacity() const noexcept { return capacity_; }

    [[nodiscard]] PageAllocationResult allocate();
    [[nodiscard]] PagePoolError release(PageHandle handle);
    [[nodiscard]] PagePoolError validate(PageHandle handle) const;
    [[nodiscard]] PagePoolSnapshot snapshot() const;
    [[nodiscard]] bool checkInvariants() const;

private:
    [[nodiscard]] PagePoolError check(PageHandle handle) const noexcept;

    PageKind kind_;
    std::uint32_t capacity_;
    std::vector<std::uint32_t> generation_;   // per slot, last issued generation
    std::vector<std::uint8_t> in_use_;        // per slot
    std::vector<std::uint32_t> free_stack_;   // top = back()
    std::uint32_t in_use_count_{0};
    std::uint64_t allocations_{0};
    std::uint64_t releases_{0};
    std::uint64_t failed_allocations_{0};
    std::uint64_t rejected_releases_{0};
    mutable std::mutex mutex_;
};

} // namespace kimkvcache
