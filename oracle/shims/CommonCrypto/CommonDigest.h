// Test-infrastructure shim: the reference hashes files with Apple CommonCrypto's
// CC_SHA256_* (src/core/io.cpp:111-122). This header provides the same three calls
// over a SHA-256 written from FIPS 180-4 (sections 4.1.2, 4.2.2, 5.1.1, 6.2), so
// the reference CPU path builds on Linux. Hashes only feed file fingerprints,
// never the GRPO arithmetic.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstring>

typedef std::uint32_t CC_LONG;
struct CC_SHA256_CTX {
    std::uint32_t h[8];
    std::uint64_t length; // bytes hashed so far
    unsigned char block[64];
    std::size_t used;
};

namespace mini_mla_shim {
inline std::uint32_t rotr(std::uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
inline void sha256_compress(std::uint32_t* h, const unsigned char* p) {
    // Round constants: the first 32 bits of the fractional parts of the cube roots
    // of the first 64 primes (FIPS 180-4, 4.2.2).
    static const std::uint32_t k[64] = {
        0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
        0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
        0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
        0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
        0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
        0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
        0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
        0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
        0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
        0xc67178f2};
    std::uint32_t w[64];
    for (int t = 0; t < 16; ++t)
        w[t] = (std::uint32_t(p[4 * t]) << 24) | (std::uint32_t(p[4 * t + 1]) << 16) |
               (std::uint32_t(p[4 * t + 2]) << 8) | std::uint32_t(p[4 * t + 3]);
    for (int t = 16; t < 64; ++t) {
        std::uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
        std::uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
        w[t] = w[t - 16] + s0 + w[t - 7] + s1;
    }
    std::uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int t = 0; t < 64; ++t) {
        std::uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) +
                           k[t] + w[t];
        std::uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
        hh = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += hh;
}
} // namespace mini_mla_shim

inline int CC_SHA256_Init(CC_SHA256_CTX* c) {
    // Initial hash value: fractional parts of the square roots of the first 8 primes.
    static const std::uint32_t init[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                          0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    std::memcpy(c->h, init, sizeof(init));
    c->length = 0;
    c->used = 0;
    return 1;
}
inline int CC_SHA256_Update(CC_SHA256_CTX* c, const void* data, CC_LONG len) {
    const auto* p = static_cast<const unsigned char*>(data);
    c->length += len;
    while (len > 0) {
        std::size_t take = 64 - c->used;
        if (take > len)
            take = len;
        std::memcpy(c->block + c->used, p, take);
        c->used += take;
        p += take;
        len -= static_cast<CC_LONG>(take);
        if (c->used == 64) {
            mini_mla_shim::sha256_compress(c->h, c->block);
            c->used = 0;
        }
    }
    return 1;
}
inline int CC_SHA256_Final(unsigned char* out, CC_SHA256_CTX* c) {
    std::uint64_t bits = c->length * 8;
    unsigned char pad = 0x80;
    CC_SHA256_Update(c, &pad, 1);
    unsigned char zero = 0;
    while (c->used != 56)
        CC_SHA256_Update(c, &zero, 1);
    unsigned char len_be[8];
    for (int i = 0; i < 8; ++i)
        len_be[i] = static_cast<unsigned char>(bits >> (56 - 8 * i));
    CC_SHA256_Update(c, len_be, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = static_cast<unsigned char>(c->h[i] >> 24);
        out[4 * i + 1] = static_cast<unsigned char>(c->h[i] >> 16);
        out[4 * i + 2] = static_cast<unsigned char>(c->h[i] >> 8);
        out[4 * i + 3] = static_cast<unsigned char>(c->h[i]);
    }
    return 1;
}
