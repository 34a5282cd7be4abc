// Fused world generation + exact sky/block light for one 32x32-column tile
// per CTA step, and the same kernel in relight mode over the dirty tiles of
// relight regions too large for the region kernels (blk_relight.cu).
//
// Light model (reference: src/world/WorldGenerator.cu:364-588). The reference
// runs one breadth-first search per light source over a 29^3 cube and
// max-merges with global atomics. Its result is the least fixed point
//     L(v) = opaque(v) ? 0 : max(src(v), max_{n in N6(v)} L(n) - 1, 0)
// with src = 15 at torches (block light) and at every cell above the height
// map (sky light; the reference's cave-entrance seeds, :506-588, are exactly
// the lit cells from which every dark open cell is reached first, so seeding
// all lit cells gives the same field). Out-of-region cells are opaque.
//
// This kernel computes that fixed point with bit-sliced level sets: with
// S_k = {v : L(v) >= k}, S_15 = sources and
//     S_k = S_{k+1} | (open & dilate6(S_{k+1}))        k = 14 .. 1,
// one bit per cell, 32 consecutive y cells of a column per 32-bit word. A
// thread keeps its own columns' level-set words and open masks in registers;
// the y neighbours are shifts across a column's words, the x/z neighbours are
// the adjacent columns' words read from a shared plane. The planes ping-pong
// between two buffers, one barrier per level. L(v) is accumulated into four
// bit planes (bit0 = xor of all S_k, bit1 = xor of even k, bit2 = xor of
// k % 4 == 0, bit3 = S_8), exact because the sets are nested.
//
// A tile is 32x32 output columns plus a 14-column halo (60x60 columns): light
// reaches 14 cells, so the halo holds every source and obstacle that can
// affect the tile. At level step s only columns within L1 distance 14 - s of
// the tile interior are updated (the "cone"), which is all the interior needs.
// Each thread owns its interior column plus up to two halo columns (the 1976
// halo columns with cone distance <= 13), handed out in order of cone distance
// so that whole warps drop out of later steps. In y only the band of rows that
// can hold non-trivial light is processed (torch rows +-14 for block light,
// dark open rows +-14 for sky light), in words that start at the band's first
// row, at most 3 words at a time (taller bands in windows of 64 output rows);
// every other row has block light 0 and trivial sky light (15 above the
// height map, 0 at or below it).
//
// Per-column inputs of generation (terrain surface, final top, the column's
// override list or its lone override inline, torch and dark rows) are
// summarised once per column by column_summary_kernel; a tile reads one
// 16-byte summary per ext column. The kernel is persistent (one CTA per SM
// walking the tiles), and every warp writes its 32 finished columns
// (contiguous in memory) with coalesced 16-byte stores from a shared staging
// area.
#include "blk_bits.cuh"
#include "blk_internal.h"

namespace blk {
namespace {

constexpr int kTile = 32;
constexpr int kExt = kTile + 2 * kHalo;             // 60
constexpr int kExtCols = kExt * kExt;               // 3600
constexpr int kHaloCols = kExtCols - kTile * kTile; // 2576
constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kSlots = 3;                           // interior + up to 2 halo columns per thread
constexpr int kColIters = (kExtCols + kThreads - 1) / kThreads;
constexpr uint32_t kCntSat = 31;                    // packed override count saturates here
constexpr uint32_t kOvrInline = 0x80000000u;        // packed list holds its single entry: y << 8 | block
// Halo slot without a column: ext column (1, 1) (cone distance 26, never in
// reach, and neither are its neighbours) with a cone distance no step reaches.
constexpr int kDummySlot = (1 * kExt + 1) | (0x7FFF << 16);

struct TileArgs {
    uint8_t* ids;
    uint8_t* light;
    int16_t* hmap;
    const int16_t* terrain_top;     // [env][z][x] local terrain surface clamped to [-1, H+4]
    const uint16_t* halo_order;     // halo ext columns sorted by cone distance
    const uint32_t* col_offset;
    const uint64_t* entries;
    const uint4* col_summary;       // generation: per column summary (column_summary_kernel)
    const uint32_t* dirty_list;
    const uint32_t* dirty_window;
    const uint32_t* dirty_count;
    uint32_t* flags;
    uint32_t* park;                 // per-CTA scratch for block planes during a sky flood
    const int4* origins;            // [env] world coordinates of each env's local (0, 0, 0)
    uint32_t n_tiles;
    int32_t W, D;
    int32_t tiles_x, tiles_z;
    uint64_t env_stride;
    uint64_t columns;
    int32_t mode; // 0 = generate, 1 = relight dirty tiles from the resident ids
    int32_t listed; // mode 0: tiles from dirty_list (0xFFFFFFFF = skip) instead of all
    const uint32_t* list_count;     // mode 0 listed: device-side entry count of dirty_list (else n_tiles)
    uint32_t* fallback_list;        // surface kernel: tiles it leaves to the tile kernel
    uint32_t* fallback_count;
    uint32_t* tile_cursor;          // surface kernel: next list position to take
};

// Rows a tile lights (see plan_tile in process_tile).
struct TilePlan {
    int32_t r_lo, r_hi, w_lo, nb;
    int32_t b_lo, b_hi, s_lo, s_hi;
    uint32_t o_chunks;
    int n_win;
    bool whole;
};

template <int NW>
struct Smem {
    // Max words of one flood band: 3 keeps the flood's registers unspilled;
    // taller bands are lit in windows.
    static constexpr int kBand = NW < 3 ? NW : 3;
    static constexpr int kPlane = kBand * kExtCols;                   // words per plane
    static constexpr int kPitch = 32 * NW + 16;                       // staging bytes per column
    // Output staging: every warp at once when its rows fit in 198 KB (with the
    // column summaries the CTA stays within 227 KB), else half of the warps per round.
    static constexpr int kStageWarps = kWarps * kTile * kPitch <= 198 * 1024 ? kWarps : kWarps / 2;
    static constexpr int kRounds = kWarps / kStageWarps;
    static constexpr int kStageWords = kStageWarps * kTile * kPitch / 4;
    static constexpr int kPoolWords = 3 * kPlane > kStageWords ? 3 * kPlane : kStageWords;
    // O | B0 | B1 during the floods; output staging otherwise.
    uint32_t pool[kPoolWords];
    int16_t top_t[kExtCols];   // terrain surface (local, clamped to [-1, H+4]); unused in relight mode
    int16_t top_f[kExtCols];   // final highest opaque local y, -1 none, -2 outside the world
    uint32_t ovr[kExtCols];    // override list: begin << 5 | min(count, 31)
    int32_t tmin, tmax, dmin, dmax;
    int32_t omin;              // generation: lowest open row of the ext region (rows below are opaque everywhere)
    TilePlan plan;             // the tile's plan, computed once per tile by thread 0

    __device__ int32_t terrain_top(int c) const { return top_t[c]; }
    __device__ uint32_t* O() { return pool; }
    __device__ uint32_t* B(int i) { return pool + (1 + i) * kPlane; }
};

// Light bytes of 32 rows (out[q] holds rows 4q .. 4q + 3, one byte each) from
// the block level bit planes b and either the sky level bit planes s
// (sky = true) or, for trivial sky light, level 15 above row `topf` (r0 = row
// of bit 0).
__device__ inline void light_bytes(const uint32_t (&b)[4], const uint32_t (&s)[4], bool sky, int32_t topf, int32_t r0,
    uint32_t (&out)[8])
{
    if (!sky && !__any_sync(__activemask(), (b[0] | b[1] | b[2] | b[3]) != 0u)) {
        // No block light in this word for any active lane: sky bytes only.
        const int32_t t8 = 8 * (topf - r0 + 1);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            out[q] = __funnelshift_lc(0u, 0xF0F0F0F0u, static_cast<uint32_t>(max(t8 - 32 * q, 0)));
        return;
    }
    uint32_t n[4], l[4], h[4];
    level_nibbles(b[0], b[1], b[2], b[3], n[0], n[1], n[2], n[3]);
    if (sky) {
        uint32_t m[4];
        level_nibbles(s[0], s[1], s[2], s[3], m[0], m[1], m[2], m[3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            l[k] = (n[k] & 0x0F0F0F0Fu) | ((m[k] << 4) & 0xF0F0F0F0u);
            h[k] = ((n[k] >> 4) & 0x0F0F0F0Fu) | (m[k] & 0xF0F0F0F0u);
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            l[k] = n[k] & 0x0F0F0F0Fu;        // byte m: row 8m + k
            h[k] = (n[k] >> 4) & 0x0F0F0F0Fu; // byte m: row 8m + 4 + k
        }
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
    if (!sky) {
        // Rows of this word at or below topf keep sky 0: 8 bits of shift per
        // such row (the funnel shift clamps at 32).
        const int32_t t8 = 8 * (topf - r0 + 1);
#pragma unroll
        for (int q = 0; q < 8; ++q)
            out[q] |= __funnelshift_lc(0u, 0xF0F0F0F0u, static_cast<uint32_t>(max(t8 - 32 * q, 0)));
    }
}

__device__ inline uint32_t entry_y(uint64_t e) { return static_cast<uint32_t>(e >> 40); }
__device__ inline uint8_t entry_block(uint64_t e) { return static_cast<uint8_t>(e & 0xFF); }

// Bits j of the word starting at row ybase with ybase + j < H.
__device__ inline uint32_t inside_mask(int32_t ybase, int32_t H)
{
    return ~above_mask(ybase, H - 1);
}

// Rows [lo, hi] of the word starting at ybase.
__device__ inline uint32_t rows_mask(int32_t ybase, int32_t lo, int32_t hi)
{
    const int32_t a = max(lo - ybase, 0), b = min(hi - ybase, 31);
    if (a > b)
        return 0u;
    const uint32_t upper = b == 31 ? 0xFFFFFFFFu : ((1u << (b + 1)) - 1u);
    return upper & ~((1u << a) - 1u);
}

// Per byte of a little-endian word: 0xFF where the byte equals `v`.
__device__ inline uint32_t bytes_eq(uint32_t x, uint32_t v) { return __vcmpeq4(x, v * 0x01010101u); }
// Low bit of each byte -> 4 packed bits.
__device__ inline uint32_t pack4(uint32_t m) { return ((m & 0x01010101u) * 0x10204080u) >> 28; }

__device__ inline int cone_distance(int c)
{
    const int ex = c % kExt, ez = c / kExt;
    const int dx = max(0, max(kHalo - ex, ex - (kHalo + kTile - 1)));
    const int dz = max(0, max(kHalo - ez, ez - (kHalo + kTile - 1)));
    return dx + dz;
}

__device__ inline bool in_world(const TileArgs& a, int gx, int gz) { return gx >= 0 && gz >= 0 && gx < a.W && gz < a.D; }

// Open-cell and torch bits of the 32 rows held in v (two 16-byte chunks of a
// resident id column, ids 0..4): open = Air or Torch (id & ~4 == 0).
__device__ inline void id_bits(const uint4 (&v)[2], uint32_t& open, uint32_t& torch)
{
    open = 0u;
    torch = 0u;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint32_t w[4] = { v[q].x, v[q].y, v[q].z, v[q].w };
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            open |= pack4_hi(zero_bytes(w[j] & 0xFBFBFBFBu)) << (16 * q + 4 * j);
            torch |= pack4_hi(zero_bytes(w[j] ^ 0x04040404u)) << (16 * q + 4 * j);
        }
    }
}

// ---- pieces shared by the tile kernel and the surface kernel ---------------
// SM is a tile's shared-memory layout: output staging in `pool` (kPitch bytes
// per column, kStageWarps warps at a time, kRounds rounds), and per ext column
// the final top top_f and the packed override list ovr (begin << 5 |
// min(count, 31), or kOvrInline | y << 8 | block); terrain_top(c) is the
// terrain surface of ext column c.

// Calls fn(y, block) for the winning override of every y of ext column c whose
// y lies in [ylo, yhi] (entries sorted by y, then input order; the last of a y
// run wins).
template <class SM, class Fn>
__device__ inline void ext_for_each_winner(const TileArgs& a, const SM& s, int c, int x0, int z0, uint64_t env_col0,
    int32_t ylo, int32_t yhi, Fn&& fn)
{
    const uint32_t packed = s.ovr[c];
    if (packed & kOvrInline) {
        const int32_t y = static_cast<int32_t>((packed >> 8) & 0x1FFu);
        if (y >= ylo && y <= yhi)
            fn(y, static_cast<uint8_t>(packed & 0xFFu));
        return;
    }
    uint32_t n = packed & kCntSat;
    uint32_t beg = packed >> 5;
    if (n == kCntSat) {
        // Long list: reread its bounds.
        const int gx = x0 - kHalo + c % kExt, gz = z0 - kHalo + c / kExt;
        const uint64_t col = env_col0 + static_cast<uint64_t>(gz) * a.W + gx;
        beg = __ldg(a.col_offset + col);
        n = __ldg(a.col_offset + col + 1) - beg;
    }
    const uint64_t* e = a.entries + beg;
    for (uint32_t i = 0; i < n; ++i) {
        const uint64_t v = __ldg(e + i);
        const int32_t y = static_cast<int32_t>(entry_y(v));
        if (y < ylo || y > yhi)
            continue;
        if (i + 1 < n && static_cast<int32_t>(entry_y(__ldg(e + i + 1))) == y)
            continue;
        fn(y, entry_block(v));
    }
}

// Output staging: each warp owns one z row of 32 columns, contiguous in
// memory. A lane builds its column's bytes in its staging column, then the
// warp stores the row with coalesced 16-byte stores.
template <class SM>
__device__ inline uint8_t* stage_column(SM& s)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    return reinterpret_cast<uint8_t*>(s.pool) + (warp % SM::kStageWarps) * (kTile * SM::kPitch) + lane * SM::kPitch;
}

// Copies the warp's staged 16-row chunks selected by `mask` (bit ch = rows
// 16ch..) of its 32 columns to dst (the row's first column).
template <int H, class SM>
__device__ inline void copy_staged(const TileArgs& a, const SM& s, int x0, uint8_t* dst, uint32_t mask)
{
    constexpr int kChunks = H / 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint8_t* stage = reinterpret_cast<const uint8_t*>(s.pool) + (warp % SM::kStageWarps) * (kTile * SM::kPitch);
    const int ncols = min(kTile, a.W - x0);
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const int idx = i * 32 + lane;
        const int col = idx / kChunks, ch = idx - col * kChunks;
        if (col < ncols && ((mask >> ch) & 1u))
            *reinterpret_cast<uint4*>(dst + static_cast<size_t>(col) * H + ch * 16)
                = *reinterpret_cast<const uint4*>(stage + col * SM::kPitch + ch * 16);
    }
}

// One 16-row chunk of trivial light bytes: sky 15 above the final top topf,
// 0 at or below it, no block light.
__device__ inline void stage_trivial_chunk(uint8_t* my, int32_t topf, int r0)
{
    uint32_t wv[4];
    // Bytes of rows at or below topf keep sky 0: shift by 8 bits per such row
    // of the word (the funnel shift clamps at 32).
    const int32_t t8 = 8 * (topf - r0 + 1);
#pragma unroll
    for (int q = 0; q < 4; ++q)
        wv[q] = __funnelshift_lc(0u, 0xF0F0F0F0u, static_cast<uint32_t>(max(t8 - 32 * q, 0)));
    *reinterpret_cast<uint4*>(my + r0) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
}

// Generation: block ids (layer rule, then the winning overrides) and the height
// map of the tile's 32 x 32 columns; c0 = this thread's interior ext column.
template <int NW, class SM>
__device__ void ids_pass(const TileArgs& a, SM& s, uint32_t env, int x0, int z0, int c0, int32_t origin_y)
{
    constexpr int H = 32 * NW;
    constexpr int kChunks = H / 16;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t env_col0 = static_cast<uint64_t>(env) * a.columns;
    uint8_t* env_ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
    for (int round = 0; round < SM::kRounds; ++round) {
        __syncthreads();
        if (warp / SM::kStageWarps != round)
            continue;
        const int gx = x0 + lane, gz = z0 + warp;
        if (in_world(a, gx, gz)) {
            const int32_t top = s.terrain_top(c0);
            uint8_t* my = stage_column(s);
            a.hmap[env_col0 + static_cast<uint64_t>(gz) * a.W + gx] = static_cast<int16_t>(s.top_f[c0] + origin_y);
            // Layer rule: id = [y <= top] + [y <= top-1] + [y <= top-4]
            // = 3 - (number of those thresholds below y). U(t) holds 0x01 in
            // the bytes of a 4-row word whose row is above t: 0x01010101
            // shifted by 8 bits per row at or below t (clamped at 32).
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch) {
                const int r0 = ch * 16;
                uint32_t wv[4];
                if (r0 > top) {
                    wv[0] = wv[1] = wv[2] = wv[3] = 0u;
                } else if (r0 + 15 <= top - 4) {
                    wv[0] = wv[1] = wv[2] = wv[3] = 0x03030303u;
                } else {
                    const int32_t a0 = 8 * (top - r0 + 1);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int32_t sh = a0 - 32 * q;
                        wv[q] = 0x03030303u - __funnelshift_lc(0u, 0x01010101u, static_cast<uint32_t>(max(sh, 0)))
                            - __funnelshift_lc(0u, 0x01010101u, static_cast<uint32_t>(max(sh - 8, 0)))
                            - __funnelshift_lc(0u, 0x01010101u, static_cast<uint32_t>(max(sh - 32, 0)));
                    }
                }
                *reinterpret_cast<uint4*>(my + r0) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
            // Winning overrides (latest of each y) replace the terrain bytes.
            if ((s.ovr[c0] & (kOvrInline | kCntSat)) != 0u)
                ext_for_each_winner(a, s, c0, x0, z0, env_col0, 0, H - 1, [&](int32_t y, uint8_t b) { my[y] = b; });
        }
        __syncwarp();
        if (z0 + warp < a.D)
            copy_staged<H>(a, s, x0, env_ids + (static_cast<uint64_t>(z0 + warp) * a.W + x0) * H, 0xFFFFFFFFu);
    }
}

// 14 dilation steps of S over NB band words. Plane O holds the open cells and
// plane B0 the level-15 sources of every ext column. A thread keeps its slot
// columns' words in registers for the whole flood. Accumulates the level bit
// planes of the interior column (slot 0) into cnt[w][p]. slot[k] packs the
// ext column (low 16 bits) and its cone distance (high bits); kDummySlot = unused.
template <int NW, int NB>
__device__ void flood(Smem<NW>& s, const int (&slot)[kSlots], uint32_t (&cnt)[Smem<NW>::kBand][4])
{
    constexpr int KB = Smem<NW>::kBand;
    constexpr int P = Smem<NW>::kPlane;
    const uint32_t* O = s.O();
    uint32_t own[kSlots][NB];
#pragma unroll
    for (int k = 0; k < kSlots; ++k)
#pragma unroll
        for (int w = 0; w < NB; ++w)
            own[k][w] = s.B(0)[w * kExtCols + (slot[k] & 0xFFFF)];
    // Open masks of the slot columns stay in registers for the whole flood.
    uint32_t open0[NB], openh[kSlots][NB];
#pragma unroll
    for (int w = 0; w < NB; ++w)
        open0[w] = O[w * kExtCols + (slot[0] & 0xFFFF)];
#pragma unroll
    for (int k = 1; k < kSlots; ++k)
#pragma unroll
        for (int w = 0; w < NB; ++w)
            openh[k][w] = O[w * kExtCols + (slot[k] & 0xFFFF)];
#pragma unroll
    for (int w = 0; w < KB; ++w) {
        cnt[w][0] = w < NB ? own[0][w < NB ? w : 0] : 0u;
        cnt[w][1] = 0;
        cnt[w][2] = 0;
        cnt[w][3] = 0;
    }
    // Fully unrolled: plane pointers, cone reach and counter updates are
    // compile-time per step.
#pragma unroll
    for (int step = 1; step <= kMaxDistance; ++step) {
        const uint32_t* cur = s.pool + (1 + ((step - 1) & 1)) * P;
        uint32_t* nxt = s.pool + (1 + (step & 1)) * P;
        const int reach = kMaxDistance - step;
        const int level = 15 - step;
#pragma unroll
        for (int k = 0; k < kSlots; ++k) {
            // A warp updates a halo slot while any of its lanes' columns is in
            // reach; the lanes beyond reach update too. That is harmless: a
            // column beyond reach at step s is only read by neighbours that are
            // beyond reach themselves at step s + 1 and later.
            if (k > 0 && !__any_sync(0xFFFFFFFFu, (slot[k] >> 16) <= reach))
                continue; // the whole warp skips this slot
            const int c = slot[k] & 0xFFFF;
            uint32_t v[NB];
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                const uint32_t* Bw = cur + w * kExtCols + c;
                const uint32_t below = w > 0 ? own[k][w > 0 ? w - 1 : 0] : 0u;
                const uint32_t above = w + 1 < NB ? own[k][w + 1 < NB ? w + 1 : w] : 0u;
                const uint32_t up = __funnelshift_l(below, own[k][w], 1); // cell y takes y-1
                const uint32_t dn = __funnelshift_r(own[k][w], above, 1); // cell y takes y+1
                const uint32_t n = up | dn | Bw[-1] | Bw[1] | Bw[-kExt] | Bw[kExt];
                v[w] = own[k][w] | ((k == 0 ? open0[w] : openh[k][w]) & n);
            }
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                own[k][w] = v[w];
                nxt[w * kExtCols + c] = v[w];
            }
            if (k == 0) {
#pragma unroll
                for (int w = 0; w < NB; ++w) {
                    cnt[w][0] ^= v[w];
                    if ((level & 1) == 0)
                        cnt[w][1] ^= v[w];
                    if ((level & 3) == 0)
                        cnt[w][2] ^= v[w];
                    if (level == 8)
                        cnt[w][3] = v[w];
                }
            }
        }
        __syncthreads();
    }
}

template <int NW>
__device__ void flood_any(int nb, Smem<NW>& s, const int (&slot)[kSlots], uint32_t (&cnt)[Smem<NW>::kBand][4])
{
    constexpr int KB = Smem<NW>::kBand;
    switch (nb) {
    case 1:
        flood<NW, 1>(s, slot, cnt);
        break;
    case 2:
        if constexpr (KB >= 2)
            flood<NW, KB >= 2 ? 2 : 1>(s, slot, cnt);
        break;
    case 3:
        if constexpr (KB >= 3)
            flood<NW, KB >= 3 ? 3 : 1>(s, slot, cnt);
        break;
    default:
        if constexpr (KB >= 4)
            flood<NW, KB>(s, slot, cnt);
        break;
    }
}

template <int NW, int MODE>
__device__ void process_tile(const TileArgs& a, Smem<NW>& s, uint32_t env, int x0, int z0, int32_t wlo_rows,
    int32_t whi_rows)
{
    constexpr int H = 32 * NW;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint64_t env_col0 = static_cast<uint64_t>(env) * a.columns;
    uint8_t* env_ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
    const int32_t origin_y = __ldg(&a.origins[env].y);

    if (tid == 0) {
        s.tmin = 1 << 20;
        s.tmax = -(1 << 20);
        s.dmin = 1 << 20;
        s.dmax = -(1 << 20);
        s.omin = 1 << 20;
    }

    // ---- phase A: per-column summary -----------------------------------
    // Generation reads each ext column's precomputed summary (one 16-byte
    // load); relight reads the height map. All loads are issued before use.
    uint4 pa[kColIters];
#pragma unroll
    for (int it = 0; it < kColIters; ++it) {
        const int c = tid + it * kThreads;
        pa[it] = make_uint4(0u, 0u, 0u, 0u);
        if (c < kExtCols) {
            const int gx = x0 - kHalo + c % kExt, gz = z0 - kHalo + c / kExt;
            if (in_world(a, gx, gz)) {
                const uint64_t col = env_col0 + static_cast<uint64_t>(gz) * a.W + gx;
                if (MODE == 0)
                    pa[it] = __ldg(a.col_summary + col);
                else
                    pa[it].x = static_cast<uint16_t>(__ldg(a.hmap + col));
            }
        }
    }
    __syncthreads();
    int32_t open_lo = 1 << 20; // lowest open row among this thread's ext columns
#pragma unroll
    for (int it = 0; it < kColIters; ++it) {
        const int c = tid + it * kThreads;
        if (c >= kExtCols)
            break;
        const int ex = c % kExt, ez = c / kExt;
        const int gx = x0 - kHalo + ex, gz = z0 - kHalo + ez;
        const bool interior = ex >= kHalo && ex < kHalo + kTile && ez >= kHalo && ez < kHalo + kTile;
        if (!in_world(a, gx, gz)) {
            s.top_t[c] = -1;
            s.top_f[c] = -2;
            s.ovr[c] = 0;
            continue;
        }
        if (MODE == 0) {
            const uint4 v = pa[it];
            s.top_t[c] = static_cast<int16_t>(v.x & 0xFFFFu);
            s.top_f[c] = static_cast<int16_t>(v.x >> 16);
            s.ovr[c] = v.y;
            const int32_t tlo = static_cast<int16_t>(v.z & 0xFFFFu), thi = static_cast<int16_t>(v.z >> 16);
            if (tlo <= thi) {
                atomicMin(&s.tmin, tlo);
                atomicMax(&s.tmax, thi);
            }
            const int32_t dlo = static_cast<int16_t>(v.w & 0xFFFFu), dhi = static_cast<int16_t>(v.w >> 16);
            if (interior && dlo <= dhi) {
                atomicMin(&s.dmin, dlo);
                atomicMax(&s.dmax, dhi);
            }
            // Open cells of the column: every row above the final top, and the
            // dark rows below it.
            open_lo = min(open_lo, static_cast<int32_t>(static_cast<int16_t>(v.x >> 16)) + 1);
            if (dlo <= dhi)
                open_lo = min(open_lo, dlo);
        } else {
            s.top_t[c] = -1;
            s.top_f[c] = static_cast<int16_t>(clamp_top(static_cast<int16_t>(pa[it].x) - origin_y, H));
            s.ovr[c] = 0;
        }
    }
    if (MODE == 0) {
        open_lo = __reduce_min_sync(0xFFFFFFFFu, open_lo);
        if (lane == 0)
            atomicMin(&s.omin, open_lo);
    }
    __syncthreads();

    // ---- slot ownership for the flood ------------------------------------
    // Slot 0: the thread's interior column. Slots 1..2: halo columns in order
    // of cone distance; slot 2 runs the warps in reverse so every warp gets a
    // similar amount of work at each step.
    int slot[kSlots];
    slot[0] = (kHalo + tid / kTile) * kExt + kHalo + tid % kTile;
#pragma unroll
    for (int k = 1; k < kSlots; ++k) {
        const int wk = (k == 2) ? (kWarps - 1 - warp) : warp;
        const int r = (k - 1) * kThreads + wk * 32 + lane;
        slot[k] = kDummySlot;
        if (r < kHaloCols) {
            const int c = __ldg(a.halo_order + r);
            const int d = cone_distance(c);
            if (d < kMaxDistance)
                slot[k] = c | (d << 16);
        }
    }

    // Calls fn(y, block) for the winning override of every y of ext column c
    // whose y lies in [ylo, yhi].
    auto for_each_winner = [&](int c, int32_t ylo, int32_t yhi, auto&& fn) {
        ext_for_each_winner(a, s, c, x0, z0, env_col0, ylo, yhi, fn);
    };

    // Generation: open-cell and source bits of ext column c for the 32 rows
    // from ybase. source: 0 = torches, 1 = lit cells (above the final top).
    auto column_bits = [&](int c, int ybase, int source, uint32_t& open, uint32_t& src) {
        const int32_t topf = s.top_f[c];
        open = 0u;
        src = 0u;
        if (topf < -1)
            return; // outside the world
        const uint32_t inside = inside_mask(ybase, H); // bands start at row >= 0
        open = above_mask(ybase, min(static_cast<int32_t>(s.top_t[c]), H - 1));
        if ((s.ovr[c] & (kOvrInline | kCntSat)) != 0u)
            for_each_winner(c, ybase, ybase + 31, [&](int32_t y, uint8_t b) {
                const uint32_t bit = 1u << (y - ybase);
                open = is_opaque(b) ? (open & ~bit) : (open | bit);
                if (source == 0 && b == Torch)
                    src |= bit;
            });
        if (source == 1)
            src = above_mask(ybase, topf);
        open &= inside;
        src &= inside & open;
    };

    // Builds planes O (open cells) and B0 (level-15 sources) of every ext
    // column over nb words from row blo.
    auto build = [&](int blo, int nb, int source) {
        uint32_t* O = s.O();
        uint32_t* B0 = s.B(0);
        if (MODE != 0) {
            // Relight: from the resident ids. Each word's loads for all of this
            // thread's ext columns are in flight before any is decoded. Window
            // words start on 16-row chunks, so a word is two aligned chunks.
            constexpr int kInFlight = 2; // columns whose loads are in flight together
            for (int w = 0; w < nb; ++w) {
                const int ybase = blo + 32 * w;
                const uint32_t inside = inside_mask(ybase, H);
#pragma unroll
                for (int it0 = 0; it0 < kColIters; it0 += kInFlight) {
                    uint4 v[kInFlight][2];
#pragma unroll
                    for (int k = 0; k < kInFlight; ++k) {
                        const int c = tid + (it0 + k) * kThreads;
                        v[k][0] = v[k][1] = make_uint4(0u, 0u, 0u, 0u);
                        if (c < kExtCols && s.top_f[c] >= -1) {
                            const int gx = x0 - kHalo + c % kExt, gz = z0 - kHalo + c / kExt;
                            const uint8_t* col = env_ids + (static_cast<uint64_t>(gz) * a.W + gx) * H + ybase;
                            v[k][0] = __ldg(reinterpret_cast<const uint4*>(col));
                            if (ybase + 16 < H)
                                v[k][1] = __ldg(reinterpret_cast<const uint4*>(col + 16));
                        }
                    }
#pragma unroll
                    for (int k = 0; k < kInFlight; ++k) {
                        const int c = tid + (it0 + k) * kThreads;
                        if (c >= kExtCols)
                            break;
                        uint32_t open = 0u, src = 0u;
                        const int32_t topf = s.top_f[c];
                        if (topf >= -1) {
                            uint32_t t;
                            id_bits(v[k], open, t);
                            open &= inside;
                            src = (source == 0 ? t : above_mask(ybase, topf)) & open;
                        }
                        O[w * kExtCols + c] = open;
                        B0[w * kExtCols + c] = src;
                    }
                }
            }
            return;
        }
        for (int c = tid; c < kExtCols; c += kThreads) {
#pragma unroll
            for (int w = 0; w < Smem<NW>::kBand; ++w)
                if (w < nb) {
                    uint32_t o, src;
                    column_bits(c, blo + 32 * w, source, o, src);
                    O[w * kExtCols + c] = o;
                    B0[w * kExtCols + c] = src;
                }
        }
    };

    // Plane B0 of the sky flood from an already built plane O: every open cell
    // above its column's final top is a source (cells outside the region are
    // not open in O).
    auto sky_sources = [&](int blo, int nb) {
        const uint32_t* O = s.O();
        uint32_t* B0 = s.B(0);
        for (int w = 0; w < nb; ++w)
            for (int c = tid; c < kExtCols; c += kThreads)
                B0[w * kExtCols + c] = O[w * kExtCols + c] & above_mask(blo + 32 * w, s.top_f[c]);
    };

    // ---- output staging helpers ----------------------------------------------
    // Each warp owns one z row of 32 columns, contiguous in memory. A lane
    // builds its column's bytes in the warp's staging area (the flood planes),
    // then the warp stores the row with coalesced 16-byte stores. All warps
    // stage at once up to H = 160, half of them per round above. The helpers
    // derive everything from tid, the tile
    // origin and shared memory, so nothing of theirs stays live across a flood.
    constexpr int kChunks = H / 16;
    constexpr int KB = Smem<NW>::kBand;
    // Output rows of one window when a tile needs several: with margins of 16
    // rows below and 14 above they fill KB words.
    constexpr int kWinRows = ((32 * KB - 30) / 16) * 16;
    auto stage_of = [&]() { return stage_column(s); };
    auto row_offset = [&]() { return (static_cast<uint64_t>(z0 + warp) * a.W + x0) * H; };
    auto copy_out = [&](uint8_t* dst, uint32_t mask) { copy_staged<H>(a, s, x0, dst, mask); };
    auto emit_trivial = [&](uint8_t* my, int32_t topf, int r0) { stage_trivial_chunk(my, topf, r0); };
    // One band word (32 rows from r0): block levels from b, sky levels from s
    // (sky) or trivial; writes the 16-row halves selected by lo_on / hi_on.
    auto emit_word = [&](uint8_t* my, int32_t topf, int r0, const uint32_t (&b)[4], const uint32_t (&sv)[4], bool sky,
                         bool lo_on, bool hi_on) {
        uint32_t o[8];
        light_bytes(b, sv, sky, topf, r0, o);
        if (lo_on)
            *reinterpret_cast<uint4*>(my + r0) = make_uint4(o[0], o[1], o[2], o[3]);
        if (hi_on)
            *reinterpret_cast<uint4*>(my + r0 + 16) = make_uint4(o[4], o[5], o[6], o[7]);
    };

    // ---- block ids and height map (generation) -------------------------------
    if (MODE == 0)
        ids_pass<NW>(a, s, env, x0, z0, slot[0], origin_y);

    // ---- light: rows that can hold non-trivial light ---------------------------
    // Block band: torch rows +-14; sky band: rows of dark open cells +-14.
    // Output rows o = the bands' hull rounded to 16-row chunks (relight: the
    // dirty window). They are lit in windows of at most KB words: a window's
    // flood covers its output rows +-14 so that every path of length <= 14
    // that ends in them stays inside. Mode 0 bands already carry that margin:
    // one window of the output rows when they fit. Otherwise windows of kWinRows
    // output rows with a margin of 16 rows below (every window starts on a
    // 16-row chunk, so its band words split into whole chunks) and 14 above.
    // The plan reads shared memory only, so it is recomputed after each flood
    // instead of being held in registers across it.
    using Plan = TilePlan;
    auto compute_plan = [&](Plan& p) {
        int32_t o_lo = 0, o_hi = -1;
        p.b_lo = H;
        p.b_hi = -1;
        p.s_lo = H;
        p.s_hi = -1;
        if (MODE == 0) {
            const int32_t tmin = s.tmin, tmax = s.tmax, dmin = s.dmin, dmax = s.dmax;
            if (tmin <= tmax) {
                p.b_lo = max(tmin - kMaxDistance, 0);
                p.b_hi = min(tmax + kMaxDistance, H - 1);
            }
            if (dmin <= dmax) {
                p.s_lo = max(dmin - kMaxDistance, 0);
                p.s_hi = min(dmax + kMaxDistance, H - 1);
            }
            // Rows below the lowest open row of the ext region are opaque in
            // every column: their light is 0 and they carry none, so the band
            // starts no lower than that row. Sources are open cells, so the
            // band stays non-empty.
            const int32_t u_lo = max(min(p.b_lo, p.s_lo), s.omin), u_hi = max(p.b_hi, p.s_hi);
            if (u_lo <= u_hi) {
                o_lo = u_lo & ~15;
                o_hi = min(u_hi | 15, H - 1);
            }
        } else {
            o_lo = wlo_rows;
            o_hi = whi_rows;
            p.b_lo = p.s_lo = max(o_lo - kMaxDistance, 0);
            p.b_hi = p.s_hi = min(o_hi + kMaxDistance, H - 1);
        }
        p.whole = o_lo <= o_hi
            && ((MODE == 0 && o_hi - o_lo + 1 <= 32 * KB)
                || (min(o_hi + kMaxDistance, H - 1) - max(o_lo - 16, 0) + 1 <= 32 * KB));
        p.n_win = o_lo > o_hi ? 0 : (p.whole ? 1 : (o_hi - o_lo + kWinRows) / kWinRows);
        p.o_chunks = o_lo > o_hi ? 0u : (((2u << (o_hi >> 4)) - 1u) & ~((1u << (o_lo >> 4)) - 1u));
        p.r_lo = o_lo;
        p.r_hi = o_hi;
    };
    // Generation: every thread reads the tile's plan from shared memory
    // (computed once by thread 0) instead of keeping it in registers across the
    // floods. Relight (one short box per change) recomputes it per thread,
    // which costs less than the extra barrier.
    auto plan_tile = [&](Plan& p) {
        if (MODE == 0)
            p = s.plan;
        else
            compute_plan(p);
    };
    auto plan_window = [&](Plan& p, int wi) {
        plan_tile(p);
        const int32_t o_lo = p.r_lo, o_hi = p.r_hi;
        int32_t w_hi;
        if (p.whole) {
            p.w_lo = MODE == 0 ? o_lo : max(o_lo - 16, 0);
            w_hi = MODE == 0 ? o_hi : min(o_hi + kMaxDistance, H - 1);
        } else {
            p.r_lo = o_lo + kWinRows * wi;
            p.r_hi = min(p.r_lo + kWinRows - 1, o_hi);
            p.w_lo = max(p.r_lo - 16, 0);
            w_hi = min(p.r_hi + kMaxDistance, H - 1);
        }
        p.nb = (w_hi - p.w_lo) / 32 + 1;
    };

    uint32_t* park = a.park + static_cast<uint64_t>(blockIdx.x) * (KB * 4 * kThreads);
    constexpr uint32_t kAllChunks = (1u << kChunks) - 1u;
    if (MODE == 0) {
        if (tid == 0)
            compute_plan(s.plan);
        __syncthreads();
    }
    int n_win;
    {
        Plan p;
        plan_tile(p);
        n_win = p.n_win;
    }
    // Pass wi < n_win lights window wi. When one window covers the output
    // rows (always for H <= 128) its pass also writes the trivial chunks;
    // otherwise a last pass writes them (generation only).
    for (int wi = 0; wi < max(n_win, 1); ++wi) {
        uint32_t cb[KB][4], cs[KB][4];
        bool have_block = false, have_sky = false;
        if (n_win > 0) {
            Plan p;
            plan_window(p, wi);
            const bool do_block = p.b_lo <= p.b_hi && p.b_lo <= p.r_hi && p.b_hi >= p.r_lo;
            const bool do_sky = p.s_lo <= p.s_hi && p.s_lo <= p.r_hi && p.s_hi >= p.r_lo;
            bool open_ready = false; // plane O of this window is built (floods only read it)
            if (do_block) {
                __syncthreads();
                build(p.w_lo, p.nb, 0);
                open_ready = true;
                __syncthreads();
                bool go = true;
                if (MODE == 1) {
                    // Any torch in the window? (generation knows from the override lists.)
                    bool any = false;
                    for (int idx = tid; idx < p.nb * kExtCols; idx += kThreads)
                        any |= s.B(0)[idx] != 0u;
                    go = __syncthreads_or(any) != 0;
                }
                if (go) {
                    flood_any<NW>(p.nb, s, slot, cb);
                    have_block = true;
                }
            }
            if (do_sky) {
                plan_window(p, wi);
                __syncthreads();
                if (open_ready)
                    sky_sources(p.w_lo, p.nb);
                else
                    build(p.w_lo, p.nb, 1);
                __syncthreads();
                bool go = true;
                if (MODE == 1) {
                    // Needed if an interior column has an open cell at or below
                    // its top inside the output rows.
                    bool dark = false;
                    const int32_t topf = s.top_f[slot[0]];
                    if (topf >= 0) {
#pragma unroll
                        for (int w = 0; w < KB; ++w)
                            if (w < p.nb) {
                                const int ybase = p.w_lo + 32 * w;
                                dark |= (s.O()[w * kExtCols + slot[0]] & ~above_mask(ybase, topf)
                                            & rows_mask(ybase, p.r_lo, p.r_hi))
                                    != 0u;
                            }
                    }
                    go = __syncthreads_or(dark) != 0;
                }
                if (go) {
                    // The block planes wait in this CTA's global scratch slice while
                    // the sky flood uses the registers (rare: needs dark open cells).
#pragma unroll
                    for (int j = 0; j < KB; ++j)
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            park[(j * 4 + q) * kThreads + tid] = have_block ? cb[j][q] : 0u;
                            cb[j][q] = 0u; // the sky path reads the parked copy
                        }
                    flood_any<NW>(p.nb, s, slot, cs);
                    have_sky = true;
                }
            }
        }

        // Stage and store the pass's light chunks. Band word j, half h holds
        // the 16-row chunk from row w_lo + 32j + 16h (w_lo is chunk aligned).
        for (int round = 0; round < Smem<NW>::kRounds; ++round) {
            __syncthreads();
            if (warp / Smem<NW>::kStageWarps != round)
                continue;
            Plan p;
            uint32_t mask = kAllChunks, band_chunks = 0u;
            if (n_win > 0) {
                plan_window(p, wi);
                const uint32_t r_chunks = ((2u << (p.r_hi >> 4)) - 1u) & ~((1u << (p.r_lo >> 4)) - 1u);
                mask = p.whole ? (MODE == 0 ? kAllChunks : r_chunks) : r_chunks;
                band_chunks = (have_block || have_sky) ? r_chunks : 0u;
            } else {
                p.w_lo = 0;
            }
            const int gx = x0 + lane, gz = z0 + warp;
            if (in_world(a, gx, gz)) {
                uint8_t* my = stage_of();
                const int32_t topf = s.top_f[slot[0]];
                const uint32_t trivial = mask & ~band_chunks;
#pragma unroll
                for (int ch = 0; ch < kChunks; ++ch)
                    if ((trivial >> ch) & 1u)
                        emit_trivial(my, topf, ch * 16);
                if (band_chunks != 0u) {
#pragma unroll
                    for (int j = 0; j < KB; ++j) {
                        const int r0 = p.w_lo + 32 * j;
                        const bool lo_on = r0 < H && ((band_chunks >> (r0 >> 4)) & 1u);
                        const bool hi_on = r0 + 16 < H && ((band_chunks >> ((r0 >> 4) + 1)) & 1u);
                        if (!lo_on && !hi_on)
                            continue;
                        if (!have_sky) {
                            emit_word(my, topf, r0, cb[j], cb[j], false, lo_on, hi_on);
                        } else {
                            const uint32_t* pk = park + j * 4 * kThreads + tid;
                            const uint32_t bp[4] = { pk[0], pk[kThreads], pk[2 * kThreads], pk[3 * kThreads] };
                            emit_word(my, topf, r0, bp, cs[j], true, lo_on, hi_on);
                        }
                    }
                }
            }
            __syncwarp();
            if (gz < a.D)
                copy_out(a.light + static_cast<uint64_t>(env) * a.env_stride + row_offset(), mask);
        }
    }

    // Several windows: the chunks outside the output rows (generation only).
    if (MODE == 0 && n_win > 1) {
        for (int round = 0; round < Smem<NW>::kRounds; ++round) {
            __syncthreads();
            if (warp / Smem<NW>::kStageWarps != round)
                continue;
            Plan p;
            plan_tile(p);
            const uint32_t mask = kAllChunks & ~p.o_chunks;
            const int gx = x0 + lane, gz = z0 + warp;
            if (in_world(a, gx, gz)) {
                uint8_t* my = stage_of();
                const int32_t topf = s.top_f[slot[0]];
#pragma unroll
                for (int ch = 0; ch < kChunks; ++ch)
                    if ((mask >> ch) & 1u)
                        emit_trivial(my, topf, ch * 16);
            }
            __syncwarp();
            if (gz < a.D)
                copy_out(a.light + static_cast<uint64_t>(env) * a.env_stride + row_offset(), mask);
        }
    }
}

// Persistent: one CTA per SM walks the tiles.
template <int NW, int MODE>
__global__ void __launch_bounds__(kThreads, 1) tile_kernel(TileArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem<NW>& s = *reinterpret_cast<Smem<NW>*>(smem_raw);
    // Relight works on the dirty tiles (regions too large for the region
    // kernels). Every CTA reads the same count.
    const uint32_t n = MODE != 0 ? *a.dirty_count : (a.list_count ? *a.list_count : a.n_tiles);
    const uint32_t tiles_per_env = static_cast<uint32_t>(a.tiles_x * a.tiles_z);
    for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
        int32_t wlo_rows = 0, whi_rows = 32 * NW - 1;
        uint32_t win = 0;
        const uint32_t tile_id = MODE == 0 && !a.listed ? i : a.dirty_list[i];
        if (tile_id == 0xFFFFFFFFu)
            continue; // uniform over the CTA
        const uint32_t env = tile_id / tiles_per_env;
        const uint32_t t_in_env = tile_id % tiles_per_env;
        const int x0 = static_cast<int>(t_in_env % a.tiles_x) * kTile;
        const int z0 = static_cast<int>(t_in_env / a.tiles_x) * kTile;
        if (MODE != 0)
            win = a.dirty_window[tile_id];
        if (MODE != 0) {
            wlo_rows = static_cast<int32_t>(win & 0xFFFFu) & ~15;
            whi_rows = min(static_cast<int32_t>(win >> 16) | 15, 32 * NW - 1);
        }
        process_tile<NW, MODE>(a, s, env, x0, z0, wlo_rows, whi_rows);
        __syncthreads();
    }
}

// ---- surface kernel: generation with one light word per column ---------------
//
// On terrain worlds the open cells of a column are the rows above its final
// top, and block light reaches at most 14 rows above a torch, less its
// horizontal distance; torches stand on the surface. So the rows of a column
// that can hold block light start at its own first open row b = top_f + 1 and
// span far fewer than 32 rows (the benchmark's reset worlds: at most 29, 11 on
// average), while one band over the 60 x 60 ext columns of varied terrain needs
// two or three 32-row words. This kernel floods ONE word per column, based at
// that column's own first open row. A column's word is kept in its 64-bit plane
// entry at bit offset 16 (lo = w << 16, hi = w >> 16); the rows [b, b + 31] of a
// neighbour with first open row b_n are that entry shifted right by
// 16 - (b_n - b), one funnel shift, for |b_n - b| <= 16.
//
// Exactness. The word flood is the exact flood of the world in which every
// open cell above its column's word is made opaque ("truncated"). That world
// has the real world's light if no truncated cell is lit in the real world,
// and that holds if no cell next to a truncated cell is lit in the word flood:
// its light is then a solution of the real world's equation, whose solution is
// unique. The cells next to truncated ones are the top bits of a word: bit 31
// (the cell above) and bits >= 32 + (b_n - b) for a neighbour whose word ends
// lower. After the flood every column of the cone tests its level set against
// those bits (a halo column at cone distance d ends with S_{1+d}, which holds
// every cell a path into the interior can use there: a path that enters a
// truncated cell x at cone distance d_x came through a neighbour of level
// >= 2 + d_x); torches of the outer ring are tested before it. A tile that
// fails a test, or holds open cells under a column top (caves and overhangs,
// which need the sky flood), a torch 16 or more rows above its column's first
// open row, or neighbouring first open rows more than 16 apart, is appended to
// fallback_list and generated by the tile kernel, which handles every world.

template <int NW>
struct SurfSmem {
    static constexpr int kPitch = 32 * NW + 16;
    static constexpr int kStageWarps = kWarps * kTile * kPitch <= 198 * 1024 ? kWarps : kWarps / 2;
    static constexpr int kRounds = kWarps / kStageWarps;
    static constexpr int kStageWords = kStageWarps * kTile * kPitch / 4;
    static constexpr int kPoolWords = 4 * kExtCols > kStageWords ? 4 * kExtCols : kStageWords;
    // Two planes of one uint2 entry per ext column during the flood; output
    // staging otherwise.
    uint32_t pool[kPoolWords];
    uint32_t ovr[kExtCols];
    int16_t top_f[kExtCols];
    int16_t top_t[kTile * kTile]; // terrain surface of the interior columns
    uint32_t flags;               // kSurfFallback | kSurfTorch
    int32_t top_lo, top_hi;       // final tops of the cone's columns in the world

    __device__ uint2* P(int i) { return reinterpret_cast<uint2*>(pool) + i * kExtCols; }
    __device__ int32_t terrain_top(int c) const { return top_t[(c / kExt - kHalo) * kTile + c % kExt - kHalo]; }
};

constexpr uint32_t kSurfFallback = 1u; // the tile is left to the tile kernel
constexpr uint32_t kSurfTorch = 2u;    // a torch lies in the cone
constexpr int kSurfPad = 16;           // bit offset of a word in its plane entry; largest |b_n - b|
// Tiles whose cone spans more rows of final tops than this mostly carry light
// above some column's word, so they go to the tile kernel before any work here.
// (The reset worlds' cones span at most 52 rows and all but 3 of their 8192
// tiles pass; the scale-out worlds' (amplitude 120) span 74 at the median and
// most of them failed the exactness test after the flood.)
constexpr int kSurfRelief = 56;

__device__ inline uint2 surf_entry(uint32_t w) { return make_uint2(w << kSurfPad, w >> (32 - kSurfPad)); }
// Rows [b, b + 31] of a neighbour's entry, amt = 16 - (b_n - b) in 0..32.
__device__ inline uint32_t surf_window(uint2 e, uint32_t amt) { return __funnelshift_rc(e.x, e.y, amt); }

// Generates one tile; returns false (uniformly over the CTA) when the tile must
// be generated by the tile kernel instead (its light is then not written).
// Thread 0 takes the CTA's next list position from the shared cursor into
// *next once this tile's column loads are in flight.
template <int NW>
__device__ bool process_surface_tile(const TileArgs& a, SurfSmem<NW>& s, uint32_t env, int x0, int z0, uint32_t* next)
{
    constexpr int H = 32 * NW;
    constexpr int kChunks = H / 16;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint64_t env_col0 = static_cast<uint64_t>(env) * a.columns;
    const int32_t origin_y = __ldg(&a.origins[env].y);

    if (tid == 0) {
        s.flags = 0u;
        s.top_lo = 1 << 20;
        s.top_hi = -(1 << 20);
    }
    // ---- column summaries and the conditions of this path -------------------
    uint4 pa[kColIters];
#pragma unroll
    for (int it = 0; it < kColIters; ++it) {
        const int c = tid + it * kThreads;
        pa[it] = make_uint4(0u, 0u, 0u, 0u);
        if (c < kExtCols) {
            const int gx = x0 - kHalo + c % kExt, gz = z0 - kHalo + c / kExt;
            if (in_world(a, gx, gz))
                pa[it] = __ldg(a.col_summary + env_col0 + static_cast<uint64_t>(gz) * a.W + gx);
        }
    }
    if (tid == 0)
        *next = atomicAdd(a.tile_cursor, 1u);
    __syncthreads();
    uint32_t fl = 0u;
    int32_t lo = 1 << 20, hi = -(1 << 20);
#pragma unroll
    for (int it = 0; it < kColIters; ++it) {
        const int c = tid + it * kThreads;
        if (c >= kExtCols)
            break;
        const int gx = x0 - kHalo + c % kExt, gz = z0 - kHalo + c / kExt;
        if (!in_world(a, gx, gz)) {
            s.top_f[c] = -2;
            s.ovr[c] = 0;
            continue;
        }
        const uint4 v = pa[it];
        const int32_t topf = static_cast<int16_t>(v.x >> 16);
        const int ex = c % kExt - kHalo, ez = c / kExt - kHalo;
        if (ex >= 0 && ex < kTile && ez >= 0 && ez < kTile)
            s.top_t[ez * kTile + ex] = static_cast<int16_t>(v.x & 0xFFFFu);
        s.top_f[c] = static_cast<int16_t>(topf);
        s.ovr[c] = v.y;
        if (cone_distance(c) <= kMaxDistance) {
            lo = min(lo, topf);
            hi = max(hi, topf);
            const int32_t tlo = static_cast<int16_t>(v.z & 0xFFFFu), thi = static_cast<int16_t>(v.z >> 16);
            const int32_t dlo = static_cast<int16_t>(v.w & 0xFFFFu), dhi = static_cast<int16_t>(v.w >> 16);
            if (dlo <= dhi)
                fl |= kSurfFallback; // open cells under the top
            if (tlo <= thi) {
                fl |= kSurfTorch;
                if (thi - (topf + 1) >= kSurfPad)
                    fl |= kSurfFallback;
            }
        }
    }
    fl = __reduce_or_sync(0xFFFFFFFFu, fl);
    lo = __reduce_min_sync(0xFFFFFFFFu, lo);
    hi = __reduce_max_sync(0xFFFFFFFFu, hi);
    if (lane == 0) {
        if (fl != 0u)
            atomicOr(&s.flags, fl);
        atomicMin(&s.top_lo, lo);
        atomicMax(&s.top_hi, hi);
    }
    __syncthreads();
    const uint32_t tf = s.flags;
    if ((tf & kSurfFallback) || s.top_hi - s.top_lo > kSurfRelief)
        return false;

    // ---- slot ownership (as in process_tile) -----------------------------------
    int slot[kSlots];
    slot[0] = (kHalo + tid / kTile) * kExt + kHalo + tid % kTile;
#pragma unroll
    for (int k = 1; k < kSlots; ++k) {
        const int wk = (k == 2) ? (kWarps - 1 - warp) : warp;
        const int r = (k - 1) * kThreads + wk * 32 + lane;
        slot[k] = kDummySlot;
        if (r < kHaloCols) {
            const int c = __ldg(a.halo_order + r);
            const int d = cone_distance(c);
            if (d < kMaxDistance)
                slot[k] = c | (d << 16);
        }
    }

    ids_pass<NW>(a, s, env, x0, z0, slot[0], origin_y);

    // Level bit planes of the interior column's word (rows b .. b + 31).
    uint32_t cnt[4] = { 0u, 0u, 0u, 0u };
    if (tf & kSurfTorch) {
        __syncthreads(); // every warp has copied its staged ids out of the pool
        // Plane 0: the torches of every ext column (rows b .. b + 15 after the
        // check above); plane 1: zero, so that a column updated beyond its
        // reach reads older values of its neighbours, never stale garbage.
        for (int c = tid; c < kExtCols; c += kThreads) {
            const int32_t b = s.top_f[c] + 1;
            uint32_t src = 0u;
            if (b >= 0 && (s.ovr[c] & (kOvrInline | kCntSat)) != 0u)
                ext_for_each_winner(a, s, c, x0, z0, env_col0, b, b + kSurfPad - 1, [&](int32_t y, uint8_t blk) {
                    if (blk == Torch)
                        src |= 1u << (y - b);
                });
            s.P(0)[c] = surf_entry(src);
            s.P(1)[c] = make_uint2(0u, 0u);
        }
        __syncthreads();

        // Per slot: its word, its rows inside the region and the shift amount
        // of each neighbour (x - 1, x + 1, z - 1, z + 1).
        uint32_t own[kSlots], inside[kSlots], amt[kSlots][4];
        int last[kSlots];
        bool bad = false;
#pragma unroll
        for (int k = 0; k < kSlots; ++k) {
            const int c = slot[k] & 0xFFFF;
            const int d = slot[k] >> 16;
            const int32_t tc = s.top_f[c];
            const int32_t b = tc + 1;
            inside[k] = tc < -1 ? 0u : inside_mask(b, H); // 0 for b >= H too
            own[k] = surf_window(s.P(0)[c], kSurfPad);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int32_t tn = s.top_f[c + (j == 0 ? -1 : j == 1 ? 1 : j == 2 ? -kExt : kExt)];
                int32_t dlt = 0; // any amount for a neighbour or column without open rows
                if (tc >= -1 && tn >= -1 && b < H && tn + 1 < H) {
                    dlt = tn - tc;
                    if (d < kMaxDistance && (dlt < -kSurfPad || dlt > kSurfPad))
                        bad = true;
                    dlt = max(-kSurfPad, min(kSurfPad, dlt));
                }
                amt[k][j] = static_cast<uint32_t>(kSurfPad - dlt);
            }
            // Last step of this slot for its warp: the nearest lane's reach.
            last[k] = k == 0 ? kMaxDistance : kMaxDistance - __reduce_min_sync(0xFFFFFFFFu, d);
        }
        if (__syncthreads_or(bad))
            return false;

        cnt[0] = own[0];
        uint32_t s2 = 0u; // S_2 of the interior column: the cells a truncation could change
        // S_k = S_{k+1} | (open & dilate6(S_{k+1})), open = the rows of the word
        // inside the region; the level bit planes accumulate as in flood().
#pragma unroll
        for (int step = 1; step <= kMaxDistance; ++step) {
            const uint2* cur = s.P((step - 1) & 1);
            uint2* nxt = s.P(step & 1);
            const int level = 15 - step;
#pragma unroll
            for (int k = 0; k < kSlots; ++k) {
                if (k > 0 && step > last[k])
                    continue; // uniform over the warp
                const int c = slot[k] & 0xFFFF;
                const uint32_t lat = surf_window(cur[c - 1], amt[k][0]) | surf_window(cur[c + 1], amt[k][1])
                    | surf_window(cur[c - kExt], amt[k][2]) | surf_window(cur[c + kExt], amt[k][3]);
                const uint32_t w = own[k];
                const uint32_t v = (w | (w << 1) | (w >> 1) | lat) & inside[k];
                own[k] = v;
                nxt[c] = surf_entry(v);
                if (k == 0) {
                    cnt[0] ^= v;
                    if ((level & 1) == 0)
                        cnt[1] ^= v;
                    if ((level & 3) == 0)
                        cnt[2] ^= v;
                    if (level == 8)
                        cnt[3] = v;
                    if (level == 2)
                        s2 = v;
                }
            }
            __syncthreads();
        }

        // No cell of level >= 2 next to a truncated one (bits >= g: g = 32 +
        // the lowest neighbour offset b_n - b below zero; bit 31 always). The
        // interior column tests S_2; a halo column its last set, S_{1+d} or
        // a part of a later one.
#pragma unroll
        for (int k = 0; k < kSlots; ++k) {
            if ((slot[k] >> 16) >= kMaxDistance)
                continue; // no column
            const uint32_t amax = max(max(amt[k][0], amt[k][1]), max(amt[k][2], amt[k][3]));
            const uint32_t g = min(31u, 48u - amax);
            bad |= ((k == 0 ? s2 : own[k]) & (0xFFFFFFFFu << g)) != 0u;
        }
        if (__syncthreads_or(bad))
            return false;
    }

    // ---- light bytes: 0 up to the final top, sky 15 above it, block levels of
    // the word's rows -------------------------------------------------------------
    for (int round = 0; round < SurfSmem<NW>::kRounds; ++round) {
        __syncthreads();
        if (warp / SurfSmem<NW>::kStageWarps != round)
            continue;
        const int gx = x0 + lane, gz = z0 + warp;
        if (in_world(a, gx, gz)) {
            uint8_t* my = stage_column(s);
            const int32_t topf = s.top_f[slot[0]];
#pragma unroll
            for (int ch = 0; ch < kChunks; ++ch)
                stage_trivial_chunk(my, topf, ch * 16);
            if ((cnt[0] | cnt[1] | cnt[2] | cnt[3]) != 0u) {
                // Rows b .. b + 31 (all open: sky 15) as bytes, written as the
                // 4-byte words from b & ~3: rows below b keep 0, rows above
                // b + 31 sky 15 without block light.
                const uint32_t sky[4] = { 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu };
                uint32_t o[8];
                planes_to_bytes(cnt, sky, o);
                const int32_t b = topf + 1;
                const uint32_t sh = 8u * static_cast<uint32_t>(b & 3);
                const int base = b & ~3;
                uint32_t prev = 0u;
#pragma unroll
                for (int q = 0; q <= 8; ++q) {
                    const uint32_t cur = q < 8 ? o[q] : 0xF0F0F0F0u;
                    if (base + 4 * q < H)
                        *reinterpret_cast<uint32_t*>(my + base + 4 * q) = __funnelshift_l(prev, cur, sh);
                    prev = cur;
                }
            }
        }
        __syncwarp();
        if (gz < a.D)
            copy_staged<H>(a, s, x0,
                a.light + static_cast<uint64_t>(env) * a.env_stride + (static_cast<uint64_t>(gz) * a.W + x0) * H,
                0xFFFFFFFFu);
    }
    return true;
}

// Persistent: one CTA per SM takes the tiles (all, or the listed ones) from a
// shared cursor, so that the CTAs end together although tiles differ in cost.
template <int NW>
__global__ void __launch_bounds__(kThreads, 1) surface_kernel(TileArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ uint32_t next;
    SurfSmem<NW>& s = *reinterpret_cast<SurfSmem<NW>*>(smem_raw);
    const uint32_t tiles_per_env = static_cast<uint32_t>(a.tiles_x * a.tiles_z);
    if (threadIdx.x == 0)
        next = atomicAdd(a.tile_cursor, 1u);
    __syncthreads();
    uint32_t i = next;
    while (i < a.n_tiles) {
        __syncthreads(); // every thread has read `next` before it is rewritten
        const uint32_t tile_id = a.listed ? a.dirty_list[i] : i;
        if (tile_id == 0xFFFFFFFFu) {
            if (threadIdx.x == 0)
                next = atomicAdd(a.tile_cursor, 1u);
        } else {
            const uint32_t env = tile_id / tiles_per_env;
            const uint32_t t_in_env = tile_id % tiles_per_env;
            const int x0 = static_cast<int>(t_in_env % a.tiles_x) * kTile;
            const int z0 = static_cast<int>(t_in_env / a.tiles_x) * kTile;
            const bool done = process_surface_tile<NW>(a, s, env, x0, z0, &next);
            if (!done && threadIdx.x == 0)
                a.fallback_list[atomicAdd(a.fallback_count, 1u)] = tile_id;
        }
        __syncthreads();
        i = next;
    }
}

// Terrain surface of every column of every env (local y, clamped to
// [-1, H+4], which preserves the layer rule inside the region).
__global__ void terrain_kernel(const uint32_t* seeds, const int4* origins, TerrainParams t, int32_t W, int32_t D,
    uint64_t total, const uint8_t* env_mask, int16_t* out)
{
    const uint64_t columns = static_cast<uint64_t>(W) * D;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t env = static_cast<uint32_t>(i / columns);
        if (env_mask && !env_mask[env])
            continue;
        const uint64_t col = i - env * columns;
        const int32_t x = static_cast<int32_t>(col % W), z = static_cast<int32_t>(col / W);
        const int4 org = origins[env];
        int32_t top = terrain_top_local(t, seeds[env], org.x + x, org.z + z, org.y);
        top = top < -1 ? -1 : (top > t.height + 4 ? t.height + 4 : top);
        out[i] = static_cast<int16_t>(top);
    }
}

// fBm surfaces, one CTA per 64 x 64 columns of one env at a time: each
// octave's lattice values over the block (at most 10 x 10: a 64-column span
// meets at most 64 / 8 + 1 cells) are hashed once into shared memory instead
// of four times per column; the per-column arithmetic is fbm()'s.
constexpr int kFbmBlock = 64;
// Generation summary of one column from its terrain surface `top` and its
// override CSR slice (see column_summary_kernel for the fields).
__device__ inline uint4 summarize_column(int32_t top, uint64_t col, const uint32_t* col_offset, const uint64_t* entries,
    int32_t H)
{
    constexpr uint32_t kEmpty = 0x7FFFu | (0x8000u << 16);
    const int32_t tc = min(top, H - 1);
    const uint32_t beg = col_offset[col];
    const uint32_t n = col_offset[col + 1] - beg;
    int32_t topf = tc;
    int32_t tlo = 1 << 20, thi = -(1 << 20), dlo = 1 << 20, dhi = -(1 << 20);
    if (n > 0) {
        const uint64_t* e = entries + beg;
        int32_t hi_opaque = -1;
        // Winners: the last entry of each y run (entries sorted by y, then input order).
        for (uint32_t i = 0; i < n; ++i) {
            const uint64_t v = e[i];
            const int32_t y = static_cast<int32_t>(entry_y(v));
            if (i + 1 < n && static_cast<int32_t>(entry_y(e[i + 1])) == y)
                continue;
            const uint8_t b = entry_block(v);
            if (is_opaque(b))
                hi_opaque = max(hi_opaque, y);
            if (b == Torch) {
                tlo = min(tlo, y);
                thi = max(thi, y);
            }
        }
        // Terrain part of the height map: walk down through cells whose
        // winning override is non-opaque.
        int32_t yt = tc;
        int32_t i = static_cast<int32_t>(n) - 1;
        while (yt >= 0) {
            while (i >= 0 && static_cast<int32_t>(entry_y(e[i])) > yt)
                --i;
            if (i >= 0 && static_cast<int32_t>(entry_y(e[i])) == yt && !is_opaque(entry_block(e[i]))) {
                --yt;
                continue;
            }
            break;
        }
        topf = max(hi_opaque, yt);
        // Open cells below the final top: non-opaque overrides there, and the
        // rows of terrain air between the terrain surface and the final top
        // that no opaque override fills (r: the next row above the surface not
        // yet known to be filled, walking the winners upwards).
        int32_t r = tc + 1;
        for (uint32_t k = 0; k < n; ++k) {
            const uint64_t v = e[k];
            const int32_t y = static_cast<int32_t>(entry_y(v));
            if (k + 1 < n && static_cast<int32_t>(entry_y(e[k + 1])) == y)
                continue;
            const bool opaque = is_opaque(entry_block(v));
            if (!opaque && y < topf) {
                dlo = min(dlo, y);
                dhi = max(dhi, y);
            }
            if (opaque && y >= r && y < topf) {
                if (y > r) {
                    dlo = min(dlo, r);
                    dhi = max(dhi, y - 1);
                }
                r = y + 1;
            }
        }
        if (r < topf) {
            dlo = min(dlo, r);
            dhi = max(dhi, topf - 1);
        }
    }
    uint4 r;
    r.x = static_cast<uint32_t>(static_cast<uint16_t>(top)) | (static_cast<uint32_t>(static_cast<uint16_t>(topf)) << 16);
    // A single override (a torch, mostly) is stored inline: its cell needs no
    // entry load later.
    r.y = n == 1 ? kOvrInline | (entry_y(entries[beg]) << 8) | entry_block(entries[beg])
                 : (beg << 5) | (n < kCntSat ? n : kCntSat);
    r.z = tlo <= thi ? static_cast<uint32_t>(static_cast<uint16_t>(tlo)) | (static_cast<uint32_t>(thi) << 16) : kEmpty;
    r.w = dlo <= dhi ? static_cast<uint32_t>(static_cast<uint16_t>(dlo)) | (static_cast<uint32_t>(dhi) << 16) : kEmpty;
    return r;
}

// With `summary` set it also writes each column's generation summary
// (summarize_column), which needs the override CSR built first.
__global__ void __launch_bounds__(256) terrain_fbm_kernel(const uint32_t* seeds, const int4* origins,
    TerrainParams t, int32_t W, int32_t D, uint32_t num_envs, const uint8_t* env_mask, int16_t* out,
    const uint32_t* col_offset, const uint64_t* entries, uint4* summary)
{
    __shared__ float lat[4][100];
    __shared__ int32_t lat_ix[4], lat_iz[4], lat_nx[4], lat_nz[4];
    // Per octave and block row z: the row's offset into lat and its weight.
    __shared__ int32_t row_off[4][kFbmBlock];
    __shared__ float row_w[4][kFbmBlock];
    static_assert(kFbmBlock * 4 == 256, "one block of threads covers four rows of columns per pass");
    const int bx = blockIdx.x * kFbmBlock, bz = blockIdx.y * kFbmBlock;
    const int ex = min(bx + kFbmBlock - 1, W - 1), ez = min(bz + kFbmBlock - 1, D - 1);
    // A thread keeps one column x of the block and walks its rows z.
    const int xx = threadIdx.x % kFbmBlock;
    for (uint32_t env = blockIdx.z; env < num_envs; env += gridDim.z) {
        if (env_mask && !env_mask[env])
            continue; // uniform over the block
        const uint32_t seed = seeds[env];
        const int4 org = origins[env];
        __syncthreads();
        if (threadIdx.x < 4) {
            // Lattice cells of octave o met by the block's columns (world x, z).
            const int o = threadIdx.x;
            int32_t i0, i1, k0, k1;
            float w;
            fbm_cell(o, org.x + bx, i0, w);
            fbm_cell(o, org.x + ex, i1, w);
            fbm_cell(o, org.z + bz, k0, w);
            fbm_cell(o, org.z + ez, k1, w);
            lat_ix[o] = i0;
            lat_iz[o] = k0;
            lat_nx[o] = i1 - i0 + 2; // corners ix .. ix + 1 of every cell met
            lat_nz[o] = k1 - k0 + 2;
        }
        __syncthreads();
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            const uint32_t so = fbm_octave_seed(seed, o);
            const int nx = lat_nx[o], nz = lat_nz[o];
            for (int k = threadIdx.x; k < nx * nz; k += blockDim.x)
                lat[o][k] = fbm_lattice(so, lat_ix[o] + k % nx, lat_iz[o] + k / nx);
        }
        {
            // Row tables: thread t covers octave t / 64, row t % 64.
            const int o = threadIdx.x / kFbmBlock, zz = threadIdx.x % kFbmBlock;
            int32_t iz;
            float wz;
            fbm_cell(o, org.z + bz + zz, iz, wz);
            row_off[o][zz] = (iz - lat_iz[o]) * lat_nx[o];
            row_w[o][zz] = wz;
        }
        // This thread's column: per octave its lattice offset and weight.
        int32_t col_off[4];
        float col_w[4];
#pragma unroll
        for (int o = 0; o < 4; ++o) {
            int32_t ix;
            fbm_cell(o, org.x + bx + xx, ix, col_w[o]);
            col_off[o] = ix - lat_ix[o];
        }
        __syncthreads();
        const uint64_t env_col0 = static_cast<uint64_t>(env) * W * D;
        const int x = bx + xx;
        for (int zz = threadIdx.x / kFbmBlock; zz < kFbmBlock; zz += 4) {
            const int z = bz + zz;
            if (x >= W || z >= D)
                continue;
            float acc = 0.0f;
            float amp = 1.0f;
#pragma unroll
            for (int o = 0; o < 4; ++o) {
                const int nx = lat_nx[o];
                const float* L = lat[o] + row_off[o][zz] + col_off[o];
                const float n = fbm_mix(L[0], L[1], L[nx], L[nx + 1], col_w[o], row_w[o][zz]);
                acc = __fadd_rn(acc, __fmul_rn(amp, n));
                amp = __fmul_rn(amp, 0.5f);
            }
            const float f = __fdiv_rn(acc, 1.875f);
            int32_t top = t.base + static_cast<int32_t>(roundf(__fmul_rn(t.amplitude, f))) - org.y;
            top = top < -1 ? -1 : (top > t.height + 4 ? t.height + 4 : top);
            const uint64_t col = env_col0 + static_cast<uint64_t>(z) * W + x;
            out[col] = static_cast<int16_t>(top);
            if (summary)
                summary[col] = summarize_column(top, col, col_offset, entries, t.height);
        }
    }
}

template <int NW, int MODE>
int launch_mode(blk_ctx* ctx, const TileArgs& a, uint32_t n_tiles, cudaStream_t stream)
{
    static bool attr_set[64] = {};
    static int sm_count[64] = {};
    const int dev = ctx->device;
    if (dev < 0 || dev >= 64) {
        set_error("device index out of range");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tile_kernel<NW, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(sizeof(Smem<NW>)));
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaFuncSetAttribute(tile_kernel)");
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(multiprocessor count)");
        attr_set[dev] = true;
    }
    if (n_tiles == 0)
        return BLK_OK;
    uint32_t grid = n_tiles < static_cast<uint32_t>(sm_count[dev]) ? n_tiles : static_cast<uint32_t>(sm_count[dev]);
    if (grid > ctx->park_ctas)
        grid = ctx->park_ctas;
    tile_kernel<NW, MODE><<<grid, kThreads, sizeof(Smem<NW>), stream>>>(a);
    return cuda_fail(cudaGetLastError(), "tile_kernel launch");
}

template <int NW>
int launch_surface_nw(blk_ctx* ctx, const TileArgs& a, uint32_t n_tiles, cudaStream_t stream)
{
    static bool attr_set[64] = {};
    static int sm_count[64] = {};
    const int dev = ctx->device;
    if (dev < 0 || dev >= 64) {
        set_error("device index out of range");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(surface_kernel<NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(sizeof(SurfSmem<NW>)));
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaFuncSetAttribute(surface_kernel)");
        e = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute(multiprocessor count)");
        attr_set[dev] = true;
    }
    if (n_tiles == 0)
        return BLK_OK;
    uint32_t grid = n_tiles < static_cast<uint32_t>(sm_count[dev]) ? n_tiles : static_cast<uint32_t>(sm_count[dev]);
    surface_kernel<NW><<<grid, kThreads, sizeof(SurfSmem<NW>), stream>>>(a);
    return cuda_fail(cudaGetLastError(), "surface_kernel launch");
}

// Generation and relight are separate kernels: each gets the registers of its
// own code path.
template <int NW>
int launch_nw(blk_ctx* ctx, const TileArgs& a, uint32_t n_tiles, cudaStream_t stream)
{
    return a.mode == 0 ? launch_mode<NW, 0>(ctx, a, n_tiles, stream) : launch_mode<NW, 1>(ctx, a, n_tiles, stream);
}

} // namespace

// Halo columns of the extended tile in the order threads take them: nearest
// cone distance first, 32 at a time (one warp), each group of 32 using 32
// distinct shared-memory banks (ext column index mod 32) so that a warp's
// plane accesses, and those of its +-1 / +-60 neighbours, are conflict-free.
// Within a group, each half-warp holds distinct columns mod 16, so that the
// surface kernel's 8-byte plane entries (served a half-warp at a time) are
// conflict-free too.
void halo_order_table(uint16_t* out)
{
    // Lanes of one group: the two columns of a residue mod 16 go to different
    // halves; residues with one column fill the emptier half.
    auto place = [&](const std::vector<int>& grp, int at) {
        std::vector<int> half[2];
        std::vector<int> by_res[16];
        for (int c : grp)
            by_res[c & 15].push_back(c);
        for (int r = 0; r < 16; ++r) {
            for (int c : by_res[r]) {
                const bool has0 = std::any_of(half[0].begin(), half[0].end(), [&](int x) { return (x & 15) == r; });
                const bool has1 = std::any_of(half[1].begin(), half[1].end(), [&](int x) { return (x & 15) == r; });
                int h = half[0].size() <= half[1].size() ? 0 : 1;
                if ((h == 0 && has0 && !has1) || (h == 1 && has1 && !has0))
                    h ^= 1;
                if (half[h].size() >= 16)
                    h ^= 1;
                half[h].push_back(c);
            }
        }
        int n = at;
        for (int h = 0; h < 2; ++h)
            for (int c : half[h])
                out[n++] = static_cast<uint16_t>(c);
    };
    std::vector<int> rest;
    for (int d = 1; d <= 2 * kHalo; ++d)
        for (int c = 0; c < kExtCols; ++c) {
            const int ex = c % kExt, ez = c / kExt;
            const int dx = std::max(0, std::max(kHalo - ex, ex - (kHalo + kTile - 1)));
            const int dz = std::max(0, std::max(kHalo - ez, ez - (kHalo + kTile - 1)));
            if (dx + dz == d)
                rest.push_back(c);
        }
    int n = 0;
    std::vector<char> taken(rest.size(), 0);
    size_t first = 0;
    while (n < kHaloCols) {
        uint32_t banks = 0;
        std::vector<int> grp;
        for (size_t i = first; i < rest.size() && grp.size() < 32; ++i) {
            if (taken[i])
                continue;
            const uint32_t bit = 1u << (rest[i] & 31);
            if (banks & bit)
                continue;
            banks |= bit;
            taken[i] = 1;
            grp.push_back(rest[i]);
        }
        for (size_t i = first; i < rest.size() && grp.size() < 32; ++i) // fewer than 32 banks left
            if (!taken[i]) {
                taken[i] = 1;
                grp.push_back(rest[i]);
            }
        while (first < rest.size() && taken[first])
            ++first;
        place(grp, n);
        n += static_cast<int>(grp.size());
    }
}

int halo_order_size() { return kHaloCols; }

// Generation summary of every column, computed once per column instead of
// once per tile whose ext region holds it: x = terrain surface | final top
// << 16 (local y, int16), y = override list begin << 5 | min(count, 31),
// z = torch rows min | max << 16, w = rows of open cells under the final top
// min | max << 16 (empty ranges as 32767 | -32768 << 16).
__global__ void column_summary_kernel(const int16_t* terrain_top, const uint32_t* col_offset, const uint64_t* entries,
    int32_t H, uint64_t total, uint64_t columns, const uint8_t* env_mask, uint4* out)
{
    for (uint64_t col = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; col < total;
         col += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        if (env_mask && !env_mask[col / columns])
            continue;
        out[col] = summarize_column(terrain_top[col], col, col_offset, entries, H);
    }
}

int launch_column_summary(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask)
{
    const uint64_t total = static_cast<uint64_t>(ctx->cfg.num_envs) * ctx->columns_per_env;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 148ull * 32)
        blocks = 148ull * 32;
    column_summary_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(ctx->terrain_top, ctx->col_offset,
        ctx->entries, static_cast<int32_t>(ctx->cfg.height), total, ctx->columns_per_env, env_mask, ctx->col_summary);
    return cuda_fail(cudaGetLastError(), "column_summary_kernel launch");
}

int launch_terrain(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask)
{
    if (ctx->cfg.terrain_mode == BLK_TERRAIN_FBM) {
        const dim3 grid((ctx->cfg.width + kFbmBlock - 1) / kFbmBlock, (ctx->cfg.depth + kFbmBlock - 1) / kFbmBlock,
            std::min<uint32_t>(ctx->cfg.num_envs, 65535));
        terrain_fbm_kernel<<<grid, 256, 0, stream>>>(ctx->seeds, ctx->origins, terrain_params(ctx),
            static_cast<int32_t>(ctx->cfg.width), static_cast<int32_t>(ctx->cfg.depth), ctx->cfg.num_envs, env_mask,
            ctx->terrain_top, nullptr, nullptr, nullptr);
        return cuda_fail(cudaGetLastError(), "terrain_fbm_kernel launch");
    }
    const uint64_t total = static_cast<uint64_t>(ctx->cfg.num_envs) * ctx->columns_per_env;
    uint64_t blocks = (total + 255) / 256;
    if (blocks > 148ull * 32)
        blocks = 148ull * 32;
    terrain_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(ctx->seeds, ctx->origins, terrain_params(ctx),
        static_cast<int32_t>(ctx->cfg.width), static_cast<int32_t>(ctx->cfg.depth), total, env_mask, ctx->terrain_top);
    return cuda_fail(cudaGetLastError(), "terrain_kernel launch");
}

int launch_surface(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask)
{
    if (ctx->cfg.terrain_mode == BLK_TERRAIN_FBM) {
        // One pass: each column's fBm surface and, from it, its summary.
        const dim3 grid((ctx->cfg.width + kFbmBlock - 1) / kFbmBlock, (ctx->cfg.depth + kFbmBlock - 1) / kFbmBlock,
            std::min<uint32_t>(ctx->cfg.num_envs, 65535));
        terrain_fbm_kernel<<<grid, 256, 0, stream>>>(ctx->seeds, ctx->origins, terrain_params(ctx),
            static_cast<int32_t>(ctx->cfg.width), static_cast<int32_t>(ctx->cfg.depth), ctx->cfg.num_envs, env_mask,
            ctx->terrain_top, ctx->col_offset, ctx->entries, ctx->col_summary);
        return cuda_fail(cudaGetLastError(), "terrain_fbm_kernel launch");
    }
    const int rc = launch_terrain(ctx, stream, env_mask);
    return rc != BLK_OK ? rc : launch_column_summary(ctx, stream, env_mask);
}

namespace {

TileArgs tile_args(blk_ctx* ctx, int mode, uint32_t n_tiles, bool listed)
{
    TileArgs a {};
    a.ids = ctx->ids;
    a.light = ctx->light;
    a.hmap = ctx->hmap;
    a.terrain_top = ctx->terrain_top;
    a.halo_order = ctx->halo_order;
    a.col_offset = ctx->col_offset;
    a.entries = ctx->entries;
    a.col_summary = ctx->col_summary;
    a.dirty_list = ctx->dirty_list;
    a.dirty_window = ctx->dirty_window;
    a.dirty_count = ctx->dirty_count;
    a.flags = ctx->flags;
    a.park = ctx->park;
    a.n_tiles = n_tiles;
    a.origins = ctx->origins;
    a.W = static_cast<int32_t>(ctx->cfg.width);
    a.D = static_cast<int32_t>(ctx->cfg.depth);
    a.tiles_x = static_cast<int32_t>(ctx->tiles_x);
    a.tiles_z = static_cast<int32_t>(ctx->tiles_z);
    a.env_stride = ctx->env_stride;
    a.columns = ctx->columns_per_env;
    a.mode = mode;
    a.listed = listed ? 1 : 0;
    a.fallback_list = ctx->fallback_list;
    a.fallback_count = ctx->fallback_count;
    a.tile_cursor = ctx->fallback_count + 1;
    return a;
}

int launch_tile_args(blk_ctx* ctx, const TileArgs& a, uint32_t n_tiles, cudaStream_t stream)
{
    switch (ctx->cfg.height / 32) {
    case 1:
        return launch_nw<1>(ctx, a, n_tiles, stream);
    case 2:
        return launch_nw<2>(ctx, a, n_tiles, stream);
    case 3:
        return launch_nw<3>(ctx, a, n_tiles, stream);
    case 4:
        return launch_nw<4>(ctx, a, n_tiles, stream);
    case 5:
        return launch_nw<5>(ctx, a, n_tiles, stream);
    case 6:
        return launch_nw<6>(ctx, a, n_tiles, stream);
    case 7:
        return launch_nw<7>(ctx, a, n_tiles, stream);
    case 8:
        return launch_nw<8>(ctx, a, n_tiles, stream);
    default:
        set_error("unsupported height");
        return BLK_ERR_INVALID_ARGUMENT;
    }
}

int launch_surface_args(blk_ctx* ctx, const TileArgs& a, uint32_t n_tiles, cudaStream_t stream)
{
    switch (ctx->cfg.height / 32) {
    case 1:
        return launch_surface_nw<1>(ctx, a, n_tiles, stream);
    case 2:
        return launch_surface_nw<2>(ctx, a, n_tiles, stream);
    case 3:
        return launch_surface_nw<3>(ctx, a, n_tiles, stream);
    case 4:
        return launch_surface_nw<4>(ctx, a, n_tiles, stream);
    case 5:
        return launch_surface_nw<5>(ctx, a, n_tiles, stream);
    case 6:
        return launch_surface_nw<6>(ctx, a, n_tiles, stream);
    case 7:
        return launch_surface_nw<7>(ctx, a, n_tiles, stream);
    case 8:
        return launch_surface_nw<8>(ctx, a, n_tiles, stream);
    default:
        set_error("unsupported height");
        return BLK_ERR_INVALID_ARGUMENT;
    }
}

} // namespace

int launch_tiles(blk_ctx* ctx, int mode, uint32_t n_tiles, cudaStream_t stream, bool listed)
{
    return launch_tile_args(ctx, tile_args(ctx, mode, n_tiles, listed), n_tiles, stream);
}

int generation_path_of(const blk_ctx* ctx)
{
    if (ctx->generation_path != BLK_GENERATION_AUTO)
        return ctx->generation_path;
    // Measured on 128 envs of fBm terrain: amplitude 50 (256 x 128 x 256) 0.97 ms
    // on the surface path against 1.11 ms on the tile kernel; amplitude 120
    // (256 x 256 x 256) 3.18 ms against 2.79 ms, 88 % of its tiles handed over.
    const bool steep = ctx->cfg.terrain_mode == BLK_TERRAIN_FBM && ctx->cfg.fbm_amplitude > 80.0f;
    return steep ? BLK_GENERATION_TILES : BLK_GENERATION_SURFACE;
}

int launch_generation(blk_ctx* ctx, uint32_t n_tiles, cudaStream_t stream, bool listed)
{
    if (generation_path_of(ctx) == BLK_GENERATION_TILES)
        return launch_tiles(ctx, 0, n_tiles, stream, listed);
    // Fallback count and tile cursor.
    cudaError_t e = cudaMemsetAsync(ctx->fallback_count, 0, 2 * sizeof(uint32_t), stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "generation counters reset");
    int rc = launch_surface_args(ctx, tile_args(ctx, 0, n_tiles, listed), n_tiles, stream);
    if (rc != BLK_OK)
        return rc;
    // The tiles the surface kernel left (their number is on the device): the
    // tile kernel's CTAs read it and walk that many list entries.
    TileArgs g = tile_args(ctx, 0, n_tiles, true);
    g.dirty_list = ctx->fallback_list;
    g.list_count = ctx->fallback_count;
    return launch_tile_args(ctx, g, n_tiles, stream);
}

} // namespace blk
