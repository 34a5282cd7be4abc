// Fused world generation + exact sky/block light for one 32x32-column tile
// per CTA, and the same kernel in relight mode over dirty tiles.
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
// one bit per cell, 32 consecutive y cells of a column per 32-bit word. The
// y neighbours are in-register shifts, the x/z neighbours are the adjacent
// columns' words in shared memory. L(v) is accumulated into four bit planes
// (bit0 = xor of all S_k, bit1 = xor of even k, bit2 = xor of k % 4 == 0,
// bit3 = S_8), exact because the sets are nested.
//
// A tile is 32x32 output columns plus a 14-column halo (60x60 columns): light
// reaches 14 cells, so the halo holds every source and obstacle that can
// affect the tile. At level step s only columns within L1 distance 14 - s of
// the tile interior are updated (the "cone"), which is all the interior needs.
// In y only the band of rows that can hold non-trivial light is processed:
// torch rows +-14 for block light, dark open rows +-14 for sky light; every
// other row is 0 block light and trivial sky light (15 above the height map,
// 0 at or below it).
#include "blk_internal.h"

namespace blk {
namespace {

constexpr int kTile = 32;
constexpr int kExt = kTile + 2 * kHalo;             // 60
constexpr int kExtCols = kExt * kExt;               // 3600
constexpr int kHaloCols = kExtCols - kTile * kTile; // 2576
constexpr int kThreads = 1024;
constexpr int kMaxWords = 4;                        // H <= 128
constexpr int kSlots = 4;                           // interior + up to 3 halo columns per thread

struct TileArgs {
    uint8_t* ids;
    uint8_t* light;
    int16_t* hmap;
    const uint32_t* seeds;
    const uint32_t* col_offset;
    const uint64_t* entries;
    const uint32_t* dirty_list;
    const uint32_t* dirty_window;
    const uint32_t* dirty_count;
    uint32_t* flags;
    TerrainParams terrain;
    int32_t W, H, D;
    int32_t tiles_x, tiles_z;
    uint64_t env_stride;
    uint64_t columns;
    int32_t mode; // 0 = generate, 1 = relight dirty tiles from the resident ids
};

struct Smem {
    uint32_t O[kMaxWords * kExtCols];
    uint32_t B[kMaxWords * kExtCols];
    int16_t top_t[kExtCols];   // terrain surface (local, clamped to [-1, H+4]); unused in relight mode
    int16_t top_f[kExtCols];   // final highest opaque local y, -1 none, -2 outside the world
    uint32_t beg[kExtCols];
    uint16_t cnt[kExtCols];
    int32_t tmin, tmax, dmin, dmax;
    int32_t any_torch, any_dark;
};

__device__ inline uint32_t spread4(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }

__device__ inline uint32_t entry_y(uint64_t e) { return static_cast<uint32_t>(e >> 40); }
__device__ inline uint8_t entry_block(uint64_t e) { return static_cast<uint8_t>(e & 0xFF); }

// Bits j of the word starting at row ybase where ybase + j > top.
__device__ inline uint32_t above_mask(int32_t ybase, int32_t top)
{
    const int32_t k = top - ybase + 1; // first open bit
    if (k <= 0)
        return 0xFFFFFFFFu;
    if (k >= 32)
        return 0u;
    return 0xFFFFFFFFu << k;
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

__device__ inline void halo_coords(int h, int& ex, int& ez)
{
    if (h < kHalo * kExt) {
        ez = h / kExt;
        ex = h % kExt;
    } else if (h < 2 * kHalo * kExt) {
        const int h2 = h - kHalo * kExt;
        ez = kHalo + kTile + h2 / kExt;
        ex = h2 % kExt;
    } else {
        const int h3 = h - 2 * kHalo * kExt;
        const int r = h3 / (2 * kHalo), k = h3 % (2 * kHalo);
        ez = kHalo + r;
        ex = k < kHalo ? k : k + kTile;
    }
}

__device__ inline int cone_distance(int ex, int ez)
{
    const int dx = max(0, max(kHalo - ex, ex - (kHalo + kTile - 1)));
    const int dz = max(0, max(kHalo - ez, ez - (kHalo + kTile - 1)));
    return dx + dz;
}

// 14 dilation steps of S over the band words; accumulates the level bit
// planes of the thread's interior column into cnt[w][p].
__device__ void flood(Smem& s, int nwb, const int (&slot_col)[kSlots], const int (&slot_dist)[kSlots],
    uint32_t (&cnt)[kMaxWords][4])
{
    const int tid = threadIdx.x;
    // Level 15 = the sources themselves.
#pragma unroll
    for (int w = 0; w < kMaxWords; ++w) {
        const uint32_t v = w < nwb ? s.B[w * kExtCols + slot_col[0]] : 0u;
        cnt[w][0] = v;
        cnt[w][1] = 0;
        cnt[w][2] = 0;
        cnt[w][3] = 0;
    }
    (void)tid;
    for (int step = 1; step <= kMaxDistance; ++step) {
        const int level = 15 - step;
        uint32_t nxt[kSlots][kMaxWords];
#pragma unroll
        for (int k = 0; k < kSlots; ++k) {
            const int c = slot_col[k];
            const bool active = c >= 0 && slot_dist[k] <= kMaxDistance - step;
#pragma unroll
            for (int w = 0; w < kMaxWords; ++w) {
                nxt[k][w] = 0u;
                if (active && w < nwb) {
                    const uint32_t* Bw = s.B + w * kExtCols;
                    const uint32_t cur = Bw[c];
                    const uint32_t below = w > 0 ? s.B[(w - 1) * kExtCols + c] : 0u;
                    const uint32_t above = w + 1 < nwb ? s.B[(w + 1) * kExtCols + c] : 0u;
                    const uint32_t up = __funnelshift_l(below, cur, 1);   // cell y takes y-1
                    const uint32_t dn = __funnelshift_r(cur, above, 1);   // cell y takes y+1
                    const uint32_t n = up | dn | Bw[c - 1] | Bw[c + 1] | Bw[c - kExt] | Bw[c + kExt];
                    nxt[k][w] = cur | (s.O[w * kExtCols + c] & n);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kSlots; ++k) {
            const int c = slot_col[k];
            const bool active = c >= 0 && slot_dist[k] <= kMaxDistance - step;
#pragma unroll
            for (int w = 0; w < kMaxWords; ++w)
                if (active && w < nwb)
                    s.B[w * kExtCols + c] = nxt[k][w];
        }
#pragma unroll
        for (int w = 0; w < kMaxWords; ++w) {
            const uint32_t v = nxt[0][w];
            cnt[w][0] ^= v;
            if ((level & 1) == 0)
                cnt[w][1] ^= v;
            if ((level & 3) == 0)
                cnt[w][2] ^= v;
            if (level == 8)
                cnt[w][3] = v;
        }
        __syncthreads();
    }
}

__device__ inline bool in_world(const TileArgs& a, int gx, int gz) { return gx >= 0 && gz >= 0 && gx < a.W && gz < a.D; }

__global__ void __launch_bounds__(kThreads, 1) tile_kernel(TileArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x;

    // ---- which tile ----------------------------------------------------
    uint32_t tile_id;
    int32_t wlo_rows = 0, whi_rows = a.H - 1; // output rows
    if (a.mode == 0) {
        tile_id = blockIdx.x;
    } else {
        if (blockIdx.x >= *a.dirty_count)
            return;
        tile_id = a.dirty_list[blockIdx.x];
        const uint32_t win = a.dirty_window[tile_id];
        wlo_rows = static_cast<int32_t>(win & 0xFFFFu) & ~15;
        whi_rows = min(static_cast<int32_t>(win >> 16) | 15, a.H - 1);
    }
    const uint32_t tiles_per_env = static_cast<uint32_t>(a.tiles_x * a.tiles_z);
    const uint32_t env = tile_id / tiles_per_env;
    const uint32_t t_in_env = tile_id % tiles_per_env;
    const int x0 = static_cast<int>(t_in_env % a.tiles_x) * kTile;
    const int z0 = static_cast<int>(t_in_env / a.tiles_x) * kTile;
    const uint32_t seed = a.seeds[env];
    const uint64_t env_col0 = static_cast<uint64_t>(env) * a.columns;
    uint8_t* env_ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
    uint8_t* env_light = a.light + static_cast<uint64_t>(env) * a.env_stride;
    const int H = a.H;

    if (tid == 0) {
        s.tmin = 1 << 20;
        s.tmax = -(1 << 20);
        s.dmin = 1 << 20;
        s.dmax = -(1 << 20);
        s.any_torch = 0;
        s.any_dark = 0;
    }
    __syncthreads();

    // ---- phase A: per-column summary -----------------------------------
    for (int c = tid; c < kExtCols; c += kThreads) {
        const int ex = c % kExt, ez = c / kExt;
        const int gx = x0 - kHalo + ex, gz = z0 - kHalo + ez;
        const bool interior = ex >= kHalo && ex < kHalo + kTile && ez >= kHalo && ez < kHalo + kTile;
        if (!in_world(a, gx, gz)) {
            s.top_t[c] = -1;
            s.top_f[c] = -2;
            s.beg[c] = 0;
            s.cnt[c] = 0;
            continue;
        }
        const uint64_t col = env_col0 + static_cast<uint64_t>(gz) * a.W + gx;
        if (a.mode == 0) {
            int32_t top = terrain_top_local(a.terrain, seed, a.terrain.origin_x + gx, a.terrain.origin_z + gz);
            top = top < -1 ? -1 : (top > H + 4 ? H + 4 : top);
            const int32_t tc = min(top, H - 1);
            const uint32_t beg = a.col_offset[col], end = a.col_offset[col + 1];
            uint32_t n = end - beg;
            if (n > 0xFFFFu) {
                atomicOr(a.flags, kFlagOverrideList);
                n = 0xFFFFu;
            }
            int32_t hi_opaque = -1;
            int32_t dlo = 1 << 20, dhi = -(1 << 20);
            // Winners: the last entry of each y run (entries sorted by y, then input order).
            for (uint32_t i = 0; i < n; ++i) {
                const uint64_t e = a.entries[beg + i];
                const int32_t y = static_cast<int32_t>(entry_y(e));
                if (i + 1 < n && static_cast<int32_t>(entry_y(a.entries[beg + i + 1])) == y)
                    continue;
                const uint8_t b = entry_block(e);
                if (is_opaque(b))
                    hi_opaque = max(hi_opaque, y);
                if (b == Torch) {
                    atomicMin(&s.tmin, y);
                    atomicMax(&s.tmax, y);
                }
            }
            // Terrain part of the height map: walk down through cells whose
            // winning override is non-opaque.
            int32_t yt = tc;
            int32_t i = static_cast<int32_t>(n) - 1;
            while (yt >= 0) {
                while (i >= 0 && static_cast<int32_t>(entry_y(a.entries[beg + i])) > yt)
                    --i;
                if (i >= 0 && static_cast<int32_t>(entry_y(a.entries[beg + i])) == yt
                    && !is_opaque(entry_block(a.entries[beg + i]))) {
                    --yt;
                    continue;
                }
                break;
            }
            const int32_t topf = max(hi_opaque, yt);
            if (interior) {
                // Open cells below the final top: non-opaque overrides there, and
                // terrain air between the terrain surface and a higher opaque override.
                for (uint32_t k = 0; k < n; ++k) {
                    const uint64_t e = a.entries[beg + k];
                    const int32_t y = static_cast<int32_t>(entry_y(e));
                    if (k + 1 < n && static_cast<int32_t>(entry_y(a.entries[beg + k + 1])) == y)
                        continue;
                    if (!is_opaque(entry_block(e)) && y < topf) {
                        dlo = min(dlo, y);
                        dhi = max(dhi, y);
                    }
                }
                if (tc + 1 < topf) {
                    dlo = min(dlo, tc + 1);
                    dhi = max(dhi, topf - 1);
                }
                if (dlo <= dhi) {
                    atomicMin(&s.dmin, dlo);
                    atomicMax(&s.dmax, dhi);
                }
            }
            s.top_t[c] = static_cast<int16_t>(top);
            s.top_f[c] = static_cast<int16_t>(topf);
            s.beg[c] = beg;
            s.cnt[c] = static_cast<uint16_t>(n);
        } else {
            const int32_t topf = clamp_top(static_cast<int32_t>(a.hmap[col]) - a.terrain.origin_y, H);
            s.top_t[c] = -1;
            s.top_f[c] = static_cast<int16_t>(topf);
            s.beg[c] = 0;
            s.cnt[c] = 0;
        }
    }
    __syncthreads();

    // ---- slot ownership for the flood ------------------------------------
    int slot_col[kSlots], slot_dist[kSlots];
    slot_col[0] = (kHalo + tid / kTile) * kExt + kHalo + tid % kTile;
    slot_dist[0] = 0;
#pragma unroll
    for (int k = 1; k < kSlots; ++k) {
        const int h = tid + (k - 1) * kThreads;
        if (h < kHaloCols) {
            int ex, ez;
            halo_coords(h, ex, ez);
            slot_col[k] = ez * kExt + ex;
            slot_dist[k] = cone_distance(ex, ez);
        } else {
            slot_col[k] = -1;
            slot_dist[k] = 1 << 20;
        }
    }

    uint32_t cb[kMaxWords][4], cs[kMaxWords][4];
    int b_wlo = 0, b_nwb = 0, s_wlo = 0, s_nwb = 0;

    // ---- band planes -----------------------------------------------------
    // Builds s.O (open cells) and s.B (level-15 sources) over `nwb` words
    // starting at word `wlo`. source: 0 = torches, 1 = lit cells.
    auto build = [&](int wlo, int nwb, int source) {
        for (int idx = tid; idx < nwb * kExtCols; idx += kThreads) {
            const int w = idx / kExtCols, c = idx - w * kExtCols;
            const int ybase = (wlo + w) * 32;
            const int32_t topf = s.top_f[c];
            uint32_t o = 0u, src = 0u;
            if (topf >= -1) {
                if (a.mode == 0) {
                    o = above_mask(ybase, min(static_cast<int32_t>(s.top_t[c]), H - 1));
                    const uint32_t beg = s.beg[c], n = s.cnt[c];
                    for (uint32_t i = 0; i < n; ++i) {
                        const uint64_t e = a.entries[beg + i];
                        const int32_t y = static_cast<int32_t>(entry_y(e));
                        if (y < ybase || y >= ybase + 32)
                            continue;
                        if (i + 1 < n && static_cast<int32_t>(entry_y(a.entries[beg + i + 1])) == y)
                            continue;
                        const uint8_t b = entry_block(e);
                        const uint32_t bit = 1u << (y - ybase);
                        o = is_opaque(b) ? (o & ~bit) : (o | bit);
                        if (source == 0 && b == Torch)
                            src |= bit;
                    }
                } else {
                    const int ex = c % kExt, ez = c / kExt;
                    const int gx = x0 - kHalo + ex, gz = z0 - kHalo + ez;
                    const uint4* p = reinterpret_cast<const uint4*>(
                        env_ids + (static_cast<uint64_t>(gz) * a.W + gx) * H + ybase);
                    const uint4 q0 = p[0], q1 = p[1];
                    const uint32_t v[8] = { q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w };
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t t = bytes_eq(v[j], Torch);
                        const uint32_t op = bytes_eq(v[j], Air) | t;
                        o |= pack4(op) << (4 * j);
                        if (source == 0)
                            src |= pack4(t) << (4 * j);
                    }
                }
                if (source == 1)
                    src = above_mask(ybase, topf);
            }
            s.O[w * kExtCols + c] = o;
            s.B[w * kExtCols + c] = src & (source == 1 ? 0xFFFFFFFFu : o);
        }
    };

    auto band_words = [&](int32_t rlo, int32_t rhi, int& wlo, int& nwb) {
        rlo = max(rlo, 0);
        rhi = min(rhi, H - 1);
        if (rlo > rhi) {
            nwb = 0;
            return;
        }
        wlo = rlo >> 5;
        nwb = (rhi >> 5) - wlo + 1;
    };

    // ---- block light -------------------------------------------------------
    if (a.mode == 0) {
        if (s.tmin <= s.tmax)
            band_words(s.tmin - kMaxDistance, s.tmax + kMaxDistance, b_wlo, b_nwb);
    } else {
        band_words(wlo_rows - kMaxDistance, whi_rows + kMaxDistance, b_wlo, b_nwb);
    }
    if (b_nwb > kMaxWords) {
        if (tid == 0)
            atomicOr(a.flags, kFlagBandTooWide);
        b_nwb = kMaxWords;
    }
    if (b_nwb > 0) {
        build(b_wlo, b_nwb, 0);
        __syncthreads();
        if (a.mode == 1) {
            // Any torch in the band? (mode 0 knows from the override lists.)
            bool any = false;
            for (int idx = tid; idx < b_nwb * kExtCols; idx += kThreads)
                any |= s.B[idx] != 0u;
            if (__syncthreads_or(any) == 0)
                b_nwb = 0;
        }
    }
    if (b_nwb > 0)
        flood(s, b_nwb, slot_col, slot_dist, cb);

    // ---- sky light -----------------------------------------------------------
    if (a.mode == 0) {
        if (s.dmin <= s.dmax)
            band_words(s.dmin - kMaxDistance, s.dmax + kMaxDistance, s_wlo, s_nwb);
        if (s_nwb > kMaxWords) {
            if (tid == 0)
                atomicOr(a.flags, kFlagBandTooWide);
            s_nwb = kMaxWords;
        }
        if (s_nwb > 0) {
            __syncthreads();
            build(s_wlo, s_nwb, 1);
            __syncthreads();
        }
    } else {
        // Same band as block light; the open plane is still valid, only the
        // sources change. Sky BFS is needed if an interior column has an open
        // cell at or below its top inside the output rows.
        s_wlo = b_wlo;
        band_words(wlo_rows - kMaxDistance, whi_rows + kMaxDistance, s_wlo, s_nwb);
        if (s_nwb > kMaxWords)
            s_nwb = kMaxWords;
        if (b_nwb == 0 && s_nwb > 0) {
            // The block pass skipped its flood but built O already.
        }
        bool dark = false;
        {
            const int c = slot_col[0];
            const int32_t topf = s.top_f[c];
            if (topf >= 0) {
#pragma unroll
                for (int w = 0; w < kMaxWords; ++w)
                    if (w < s_nwb) {
                        const int ybase = (s_wlo + w) * 32;
                        const uint32_t below_top = ~above_mask(ybase, topf);
                        dark |= (s.O[w * kExtCols + c] & below_top & rows_mask(ybase, wlo_rows, whi_rows)) != 0u;
                    }
            }
        }
        __syncthreads();
        if (__syncthreads_or(dark) == 0)
            s_nwb = 0;
        if (s_nwb > 0) {
            for (int idx = tid; idx < s_nwb * kExtCols; idx += kThreads) {
                const int w = idx / kExtCols, c = idx - w * kExtCols;
                const int32_t topf = s.top_f[c];
                s.B[idx] = topf >= -1 ? above_mask((s_wlo + w) * 32, topf) : 0u;
            }
            __syncthreads();
        }
    }
    if (s_nwb > 0)
        flood(s, s_nwb, slot_col, slot_dist, cs);

    // ---- outputs for the interior column -------------------------------------
    const int lx = tid % kTile, lz = tid / kTile;
    const int gx = x0 + lx, gz = z0 + lz;
    if (!in_world(a, gx, gz))
        return;
    const int c0 = slot_col[0];
    const int32_t topf = s.top_f[c0];
    const uint64_t col_off = (static_cast<uint64_t>(gz) * a.W + gx) * H;
    uint4* light_col = reinterpret_cast<uint4*>(env_light + col_off);

    if (a.mode == 0) {
        a.hmap[env_col0 + static_cast<uint64_t>(gz) * a.W + gx] = static_cast<int16_t>(topf + a.terrain.origin_y);
        const int32_t top = s.top_t[c0];
        uint4* id_col = reinterpret_cast<uint4*>(env_ids + col_off);
        for (int r0 = 0; r0 < H; r0 += 16) {
            uint32_t wv[4];
            if (r0 > top) {
                wv[0] = wv[1] = wv[2] = wv[3] = 0u;
            } else if (r0 + 15 <= top - 4) {
                wv[0] = wv[1] = wv[2] = wv[3] = 0x03030303u;
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    uint32_t v = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b)
                        v |= static_cast<uint32_t>(layer_block(r0 + 4 * q + b, top)) << (8 * b);
                    wv[q] = v;
                }
            }
            id_col[r0 >> 4] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        // Overrides (same thread, program order: these bytes land last).
        const uint32_t beg = s.beg[c0], n = s.cnt[c0];
        for (uint32_t i = 0; i < n; ++i) {
            const uint64_t e = a.entries[beg + i];
            const int32_t y = static_cast<int32_t>(entry_y(e));
            if (i + 1 < n && static_cast<int32_t>(entry_y(a.entries[beg + i + 1])) == y)
                continue;
            env_ids[col_off + y] = entry_block(e);
        }
    }

    for (int r0 = wlo_rows; r0 <= whi_rows; r0 += 16) {
        const int word = r0 >> 5;
        const int j0 = r0 & 31;
        const int bw = word - b_wlo, sw = word - s_wlo;
        uint32_t bn[4] = { 0u, 0u, 0u, 0u }, sn[4] = { 0u, 0u, 0u, 0u };
        bool block_any = false;
        if (b_nwb > 0 && bw >= 0 && bw < b_nwb) {
#pragma unroll
            for (int w = 0; w < kMaxWords; ++w)
                if (w == bw) {
#pragma unroll
                    for (int p = 0; p < 4; ++p)
                        bn[p] = cb[w][p] >> j0;
                }
            block_any = ((bn[0] | bn[1] | bn[2] | bn[3]) & 0xFFFFu) != 0u;
        }
        const bool sky_bfs = s_nwb > 0 && sw >= 0 && sw < s_nwb;
        if (sky_bfs) {
#pragma unroll
            for (int w = 0; w < kMaxWords; ++w)
                if (w == sw) {
#pragma unroll
                    for (int p = 0; p < 4; ++p)
                        sn[p] = cs[w][p] >> j0;
                }
        }
        uint32_t wv[4];
        if (!block_any && !sky_bfs && (r0 > topf || r0 + 15 <= topf)) {
            const uint32_t v = r0 > topf ? 0xF0F0F0F0u : 0u;
            wv[0] = wv[1] = wv[2] = wv[3] = v;
        } else {
            const uint32_t lit = sky_bfs ? 0u : above_mask(r0, topf);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int j = 4 * q;
                uint32_t v = spread4((bn[0] >> j) & 0xFu) | (spread4((bn[1] >> j) & 0xFu) << 1)
                    | (spread4((bn[2] >> j) & 0xFu) << 2) | (spread4((bn[3] >> j) & 0xFu) << 3);
                if (sky_bfs)
                    v |= (spread4((sn[0] >> j) & 0xFu) << 4) | (spread4((sn[1] >> j) & 0xFu) << 5)
                        | (spread4((sn[2] >> j) & 0xFu) << 6) | (spread4((sn[3] >> j) & 0xFu) << 7);
                else
                    v |= spread4((lit >> j) & 0xFu) * 0xF0u;
                wv[q] = v;
            }
        }
        light_col[r0 >> 4] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
}

} // namespace

size_t tile_smem_bytes() { return sizeof(Smem); }

int launch_tiles(blk_ctx* ctx, int mode, uint32_t n_tiles, cudaStream_t stream)
{
    static bool attr_set[64] = {};
    int dev = ctx->device;
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
            static_cast<int>(sizeof(Smem)));
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaFuncSetAttribute(tile_kernel)");
        attr_set[dev] = true;
    }
    if (n_tiles == 0)
        return BLK_OK;
    TileArgs a {};
    a.ids = ctx->ids;
    a.light = ctx->light;
    a.hmap = ctx->hmap;
    a.seeds = ctx->seeds;
    a.col_offset = ctx->col_offset;
    a.entries = ctx->entries;
    a.dirty_list = ctx->dirty_list;
    a.dirty_window = ctx->dirty_window;
    a.dirty_count = ctx->dirty_count;
    a.flags = ctx->flags;
    a.terrain = terrain_params(ctx);
    a.W = static_cast<int32_t>(ctx->cfg.width);
    a.H = static_cast<int32_t>(ctx->cfg.height);
    a.D = static_cast<int32_t>(ctx->cfg.depth);
    a.tiles_x = static_cast<int32_t>(ctx->tiles_x);
    a.tiles_z = static_cast<int32_t>(ctx->tiles_z);
    a.env_stride = ctx->env_stride;
    a.columns = ctx->columns_per_env;
    a.mode = mode;
    tile_kernel<<<n_tiles, kThreads, sizeof(Smem), stream>>>(a);
    return cuda_fail(cudaGetLastError(), "tile_kernel launch");
}

} // namespace blk
