// SHA-256 written from the FIPS 180-4 specification (section 6.2).
#include "sha256.h"

#include <cstring>

namespace kimkvcache {
namespace {

// First 32 bits of the fractional parts of the cube roots of the first 64 primes.
constexpr std::uint32_t kRound[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
    0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
    0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
    0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
    0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
    0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
    0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
    0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2,
};

constexpr std::uint32_t rotr(std::uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

} // namespace

Sha256::Sha256() noexcept
    // First 32 bits of the fractional parts of the square roots of the first 8 primes.
    : h_{0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab,
          0x5be0cd19}
{
}

void Sha256::block(std::uint8_t const* p) noexcept
{
    std::uint32_t w[64];
    for (int i = 0; i < 16; ++i) {
        w[i] = (std::uint32_t(p[4 * i]) << 24) | (std::uint32_t(p[4 * i + 1]) << 16)
            | (std::uint32_t(p[4 * i + 2]) << 8) | std::uint32_t(p[4 * i + 3]);
    }
    for (int i = 16; i < 64; ++i) {
        std::uint32_t const s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        std::uint32_t const s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    std::uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3];
    std::uint32_t e = h_[4], f = h_[5], g = h_[6], h = h_[7];
    for (int i = 0; i < 64; ++i) {
        std::uint32_t const S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        std::uint32_t const ch = (e & f) ^ (~e & g);
        std::uint32_t const t1 = h + S1 + ch + kRound[i] + w[i];
        std::uint32_t const S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        std::uint32_t const maj = (a & b) ^ (a & c) ^ (b & c);
        std::uint32_t const t2 = S0 + maj;
        h = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d;
    h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
}

void Sha256::update(void const* data, std::size_t size) noexcept
{
    auto const* p = static_cast<std::uint8_t const*>(data);
    total_ += size;
    if (used_ != 0) {
        std::size_t const take = size < 64 - used_ ? size : 64 - used_;
        std::memcpy(buf_.data() + used_, p, take);
        used_ += take;
        p += take;
        size -= take;
        if (used_ == 64) {
            block(buf_.data());
            used_ = 0;
        }
    }
    while (size >= 64) {
        block(p);
        p += 64;
        size -= 64;
    }
    if (size != 0) {
        std::memcpy(buf_.data(), p, size);
        used_ = size;
    }
}

std::string Sha256::hexDigest() noexcept
{
    std::uint64_t const bits = total_ * 8;
    std::uint8_t pad[72] = {0x80};
    std::size_t const pad_len = (used_ < 56 ? 56 - used_ : 120 - used_);
    update(pad, pad_len);
    std::uint8_t len[8];
    for (int i = 0; i < 8; ++i) {
        len[i] = static_cast<std::uint8_t>(bits >> (56 - 8 * i));
    }
    update(len, 8);
    static constexpr char kHex[] = "0123456789abcdef";
    std::string out(64, '0');
    for (int i = 0; i < 8; ++i) {
        for (int j = 0; j < 4; ++j) {
            std::uint8_t const byte = static_cast<std::uint8_t>(h_[i] >> (24 - 8 * j));
            out[8 * i + 2 * j] = kHex[byte >> 4];
            out[8 * i + 2 * j + 1] = kHex[byte & 15];
        }
    }
    return out;
}

} // namespace kimkvcache
