// Host FP16 <-> FP32 conversion with IEEE-754 round-to-nearest-even, the same
// rounding the device uses (__float2half_rn). Public names follow the
// reference (include/kim-kv/reference/kv_reference.h:10-13); the bit
// arithmetic below is derived directly from the binary16/binary32 formats.
#pragma once

#include "kv_types.h"

#include <cstdint>
#include <cstring>

namespace kimkvcache {

[[nodiscard]] inline KvScalar floatToKvScalar(float value) noexcept
{
    std::uint32_t x = 0;
    std::memcpy(&x, &value, sizeof(x));
    std::uint32_t const sign = (x >> 16) & 0x8000u;
    x &= 0x7fffffffu;
    if (x >= 0x7f800000u) {                       // Inf stays Inf; NaN -> quiet NaN
        return static_cast<KvScalar>(sign | (x == 0x7f800000u ? 0x7c00u : 0x7e00u));
    }
    std::uint32_t const exponent = x >> 23;       // biased binary32 exponent
    std::uint32_t mantissa = x & 0x7fffffu;
    int const half_exponent = static_cast<int>(exponent) - 112;  // rebias 127 -> 15
    if (half_exponent >= 31) {
        return static_cast<KvScalar>(sign | 0x7c00u);
    }
    if (half_exponent <= 0) {
        // Result is subnormal (or zero): count units of 2^-24.
        std::uint32_t const shift = static_cast<std::uint32_t>(126 - static_cast<int>(exponent));
        if (shift > 24) {
            return static_cast<KvScalar>(sign);
        }
        mantissa |= 0x800000u;
        std::uint32_t q = mantissa >> shift;
        std::uint32_t const rest = mantissa & ((1u << shift) - 1u);
        std::uint32_t const tie = 1u << (shift - 1u);
        if (rest > tie || (rest == tie && (q & 1u) != 0)) {
            ++q;                                   // may carry into the smallest normal
        }
        return static_cast<KvScalar>(sign | q);
    }
    std::uint32_t q = (static_cast<std::uint32_t>(half_exponent) << 10) | (mantissa >> 13);
    std::uint32_t const rest = mantissa & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (q & 1u) != 0)) {
        ++q;                                       // carry may reach the Inf encoding
    }
    return static_cast<KvScalar>(sign | q);
}

[[nodiscard]] inline float kvScalarToFloat(KvScalar value) noexcept
{
    std::uint32_t const sign = static_cast<std::uint32_t>(value & 0x8000u) << 16;
    std::uint32_t const exponent = (value >> 10) & 0x1fu;
    std::uint32_t mantissa = value & 0x3ffu;
    std::uint32_t bits = 0;
    if (exponent == 0x1fu) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else if (exponent != 0) {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    } else if (mantissa != 0) {
        // Subnormal: normalise the leading one into the implicit bit.
        int e = 113;
        while ((mantissa & 0x400u) == 0) {
            mantissa <<= 1;
            --e;
        }
        bits = sign | (static_cast<std::uint32_t>(e) << 23) | ((mantissa & 0x3ffu) << 13);
    } else {
        bits = sign;
    }
    float out = 0.0f;
    std::memcpy(&out, &bits, sizeof(out));
    return out;
}

} // namespace kimkvcache
