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

// Light bytes of 32 rows from block level bit planes b and sky level bit
// planes s: out[q] holds rows 4q .. 4q + 3, one byte each (sky << 4 | block).
// The nibbles of both floods are interleaved into bytes (l: rows 8m + k, h:
// rows 8m + 4 + k in byte m of l[k], h[k]), then each group of four words is
// transposed bytewise.
__device__ inline void planes_to_bytes(const uint32_t (&b)[4], const uint32_t (&s)[4], uint32_t (&out)[8])
{
    uint32_t n[4], m[4], l[4], h[4];
    level_nibbles(b[0], b[1], b[2], b[3], n[0], n[1], n[2], n[3]);
    level_nibbles(s[0], s[1], s[2], s[3], m[0], m[1], m[2], m[3]);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        l[k] = (n[k] & 0x0F0F0F0Fu) | ((m[k] << 4) & 0xF0F0F0F0u);
        h[k] = ((n[k] >> 4) & 0x0F0F0F0Fu) | (m[k] & 0xF0F0F0F0u);
    }
    const uint32_t la = __byte_perm(l[0], l[1], 0x5140), lb = __byte_perm(l[0], l[1], 0x7362);
    const uint32_t lc = __byte_perm(l[2], l[3], 0x5140), ld = __byte_perm(l[2], l[3], 0x7362);
    const uint32_t ha = __byte_perm(h[0], h[1], 0x5140), hb = __byte_perm(h[0], h[1], 0x7362);
    const uint32_t hc = __byte_perm(h[2], h[3], 0x5140), hd = __byte_perm(h[2], h[3], 0x7362);
    out[0] = __byte_perm(la, lc, 0x5410);
    out[2] = __byte_perm(la, lc, 0x7632);
    out[4] = __byte_perm(lb, ld, 0x5410);
    out[6] = __byte_perm(lb, ld, 0x7632);
    out[1] = __byte_perm(ha, hc, 0x5410);
    out[3] = __byte_perm(ha, hc, 0x7632);
    out[5] = __byte_perm(hb, hd, 0x5410);
    out[7] = __byte_perm(hb, hd, 0x7632);
}

// Asynchronous global -> shared copies (cp.async): 4 and 16 bytes, and the
// wait for all of this thread's copies.
__device__ inline void cp_async4(void* smem, const void* gmem)
{
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(d), "l"(gmem) : "memory");
}
__device__ inline void cp_async16(void* smem, const void* gmem)
{
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem) : "memory");
}
__device__ inline void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

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
