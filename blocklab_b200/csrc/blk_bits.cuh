// Bit-level helpers shared by the tile kernel and the region relight: level
// bit planes to nibbles, row masks of 32-row words, byte tests.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace blk {

// Rows r of 32 as 4-bit levels given as bit planes (bit r of p_k = bit k of the
// level of row r): nibble j of n_k = level of row 4j + k. Pairs bits of even and
// odd rows, then pairs of pairs (a bit-matrix transpose by masked shifts).
__device__ inline void level_nibbles(uint32_t p0, uint32_t p1, uint32_t p2, uint32_t p3, uint32_t& n0, uint32_t& n1,
    uint32_t& n2, uint32_t& n3)
{
    const uint32_t e01 = (p0 & 0x55555555u) | ((p1 << 1) & 0xAAAAAAAAu); // pair i: row 2i, bits 0, 1
    const uint32_t o01 = ((p0 >> 1) & 0x55555555u) | (p1 & 0xAAAAAAAAu); // pair i: row 2i + 1
    const uint32_t e23 = (p2 & 0x55555555u) | ((p3 << 1) & 0xAAAAAAAAu);
    const uint32_t o23 = ((p2 >> 1) & 0x55555555u) | (p3 & 0xAAAAAAAAu);
    n0 = (e01 & 0x33333333u) | ((e23 << 2) & 0xCCCCCCCCu);
    n2 = ((e01 >> 2) & 0x33333333u) | (e23 & 0xCCCCCCCCu);
    n1 = (o01 & 0x33333333u) | ((o23 << 2) & 0xCCCCCCCCu);
    n3 = ((o01 >> 2) & 0x33333333u) | (o23 & 0xCCCCCCCCu);
}

// Bits j of the word starting at row ybase where ybase + j > top.
__device__ inline uint32_t above_mask(int32_t ybase, int32_t top)
{
    // ~0 << k for the first open bit k, clamped to 0..32 (the funnel shift
    // clamps shifts above 32: k >= 32 gives 0).
    return __funnelshift_lc(0u, 0xFFFFFFFFu, static_cast<uint32_t>(max(top - ybase + 1, 0)));
}

// 0x80 in every byte of x that is zero (bytes below 0x80: adding 0x7F carries
// into bit 7 exactly when the byte is non-zero, and never into the next byte).
__device__ inline uint32_t zero_bytes(uint32_t x) { return ((x + 0x7F7F7F7Fu) & 0x80808080u) ^ 0x80808080u; }
// Bit 7 of each byte -> 4 packed bits.
__device__ inline uint32_t pack4_hi(uint32_t m) { return ((m >> 7) * 0x10204080u) >> 28; }

} // namespace blk
