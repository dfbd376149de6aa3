#include "page_pool.h"

#include <stdexcept>

namespace kimkvcache {

std::string_view toString(KvCacheError error) noexcept
{
    static constexpr std::string_view names[] = {
        "none", "invalid_argument", "request_not_found",
        "request_already_exists", "request_conflict", "resource_exhausted",
        "invalid_state", "token_reservation_not_found",
        "promotion_not_eligible", "promotion_not_found",
        "promotion_conflict", "internal_invariant_violation",
    };
    auto const index = static_cast<std::size_t>(error);
    return index < sizeof(names) / sizeof(names[0]) ? names[index] : "unknown";
}

std::string_view toString(PageState state) noexcept
{
    static constexpr std::string_view names[] = {
        "free", "mutable", "sealed", "copy_target", "retiring",
    };
    auto const index = static_cast<std::size_t>(state);
    return index < 5 ? names[index] : "unknown";
}

PagePool::PagePool(PageKind kind, std::uint32_t capacity)
    : kind_(kind), capacity_(capacity)
{
    if (!isKnownPageKind(kind)) {
        throw std::invalid_argument("page pool kind must be micro or extent");
    }
    if (capacity == 0) {
        throw std::invalid_argument("page pool capacity must be positive");
    }
    generation_.assign(capacity, 0);
    in_use_.assign(capacity, 0);
    free_stack_.resize(capacity);
    // Highest slot at the bottom of the stack: pops yield 0, 1, 2, ...
    for (std::uint32_t i = 0; i < capacity; ++i) {
        free_stack_[i] = capacity - 1 - i;
    }
}

PageAllocationResult PagePool::allocate()
{
    std::lock_guard<std::mutex> lock(mutex_);
    if (free_stack_.empty()) {
        ++failed_allocations_;
        return {PagePoolError::Exhausted, PageHandle::invalid()};
    }
    std::uint32_t const slot = free_stack_.back();
    if (slot >= capacity_ || in_use_[slot] != 0 || in_use_count_ >= capacity_) {
        throw std::logic_error("page pool free stack is corrupt");
    }
    free_stack_.pop_back();
    std::uint32_t generation = generation_[slot] + 1;
    if (generation == PageHandle::kInvalidGeneration) {
        generation = 1;  // wrap past the reserved invalid generation
    }
    generation_[slot] = generation;
    in_use_[slot] = 1;
    ++in_use_count_;
    ++allocations_;
    return {PagePoolError::None, PageHandle{kind_, slot, generation}};
}

PagePoolError PagePool::check(PageHandle handle) const noexcept
{
    if (!handle.isStructurallyValid()) {
        return PagePoolError::InvalidHandle;
    }
    if (handle.kind != kind_) {
        return PagePoolError::WrongKind;
    }
    if (handle.slot >= capacity_) {
        return PagePoolError::OutOfRange;
    }
    // A recycled slot reports a stale generation before "already free".
    if (handle.generation != generation_[handle.slot]) {
        return PagePoolError::StaleGeneration;
    }
    if (in_use_[handle.slot] == 0) {
        return PagePoolError::AlreadyFree;
    }
    return PagePoolError::None;
}

PagePoolError PagePool::release(PageHandle handle)
{
    std::lock_guard<std::mutex> lock(mutex_);
    PagePoolError const error = check(handle);
    if (error != PagePoolError::None) {
        ++rejected_releases_;
        return error;
    }
    if (in_use_count_ == 0 || free_stack_.size() >= capacity_) {
        throw std::logic_error("page pool accounting is corrupt");
    }
    free_stack_.push_back(handle.slot);
    in_use_[handle.slot] = 0;
    --in_use_count_;
    ++releases_;
    return PagePoolError::None;
}

PagePoolError PagePool::validate(PageHandle handle) const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return check(handle);
}

PagePoolSnapshot PagePool::snapshot() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    return PagePoolSnapshot{kind_, capacity_,
        static_cast<std::uint32_t>(free_stack_.size()), in_use_count_,
        allocations_, releases_, failed_allocations_, rejected_releases_};
}

bool PagePool::checkInvariants() const
{
    std::lock_guard<std::mutex> lock(mutex_);
    if (generation_.size() != capacity_ || in_use_.size() != capacity_
        || free_stack_.size() + in_use_count_ != capacity_) {
        return false;
    }
    std::vector<std::uint8_t> on_stack(capacity_, 0);
    for (std::uint32_t slot : free_stack_) {
        if (slot >= capacity_ || on_stack[slot] != 0 || in_use_[slot] != 0) {
            return false;
        }
        on_stack[slot] = 1;
    }
    std::uint32_t used = 0;
    for (std::uint32_t slot = 0; slot < capacity_; ++slot) {
        if (in_use_[slot] != 0) {
            if (generation_[slot] == PageHandle::kInvalidGeneration || on_stack[slot] != 0) {
                return false;
            }
            ++used;
        } else if (on_stack[slot] == 0) {
            return false;
        }
    }
    return used == in_use_count_ && releases_ <= allocations_
        && allocations_ - releases_ == in_use_count_;
}

} // namespace kimkvcache
