// SHA-256 (FIPS 180-4) for verifying weight archives at model load.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <string>

namespace kimkvcache {

class Sha256 final {
public:
    Sha256() noexcept;
    void update(void const* data, std::size_t size) noexcept;
    // Lower-case hex digest; the object must not be updated afterwards.
    [[nodiscard]] std::string hexDigest() noexcept;

private:
    void block(std::uint8_t const* p) noexcept;

    std::array<std::uint32_t, 8> h_{};
    std::array<std::uint8_t, 64> buf_{};
    std::size_t used_{0};
    std::uint64_t total_{0};
};

} // namespace kimkvcache
