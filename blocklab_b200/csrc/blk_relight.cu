// Exact incremental relight after edits: the changed cells of an env are
// grouped into regions (boxes of columns x rows) whose one-cell boundary ring
// no edit of the step can have relit, and each region's light is recomputed
// from its resident boundary.
//
// Why a region with a clean ring is exact. Light is the unique solution of
//     L(v) = opaque(v) ? 0 : max(src(v), max_{n in N6(v)} L(n) - 1, 0)
// (src = 15 at torches for block light, at open cells above the column's top
// for sky light; cells outside the world are opaque). Restricted to a box R,
// the same equation with the values of the cells just outside R held fixed has
// exactly one solution: a positive level needs a neighbour one higher, so it is
// carried by a chain that ends at a source in R or at a fixed cell. The light
// of the whole world restricted to R is such a solution, so solving the box
// problem with the CORRECT boundary values gives the new light of R.
//
// A change can move light only within L-inf distance 14 of its cell or of the
// column span its top moved over (the dirty cube of the change). Outside the
// union of the step's dirty cubes the old light is the new light. So the
// resident light of a cell outside every cube is its correct new value: a box
// whose boundary ring avoids every cube can be solved from the resident ring.
// The regions are built per env by merging dirty cubes: two regions whose
// bounding boxes come within one cell of each other (one region's ring meets
// the other region) are replaced by their common bounding box, until no two
// regions touch. Every region's ring then lies outside every cube.
//
// Solving a region: with S_k = {v : L(v) >= k}, a fixed cell of level l joins
// the level sets at S_l and stays, a source joins at S_15, and
//     S_k = S_{k+1} | fixed_k | (open & dilate6(S_{k+1}))       k = 14 .. 1,
// one bit per cell, 32 rows of a column per word (as in the tile kernel).
// Fixed cells are the region's ring: the ring columns around it (every row of
// the region) and the rows just below and above the region in each of its
// columns. A region needs only its own columns and no halo: about 29 x 29
// columns and one word for a single change, instead of a 60 x 60-column tile
// with a 14-column halo.
//
// A region of more than 4096 columns or 64 a side is split into sub-boxes of
// 32 x 32 columns, each solved over itself and the region's columns within 14
// of it
// (light from farther away cannot reach it). Regions of more than 62 rows are
// relit by the tile kernel's halo path over the tiles they cover. Every path
// writes only correct new values, and a region's ring cells are never changed
// by any, so they may run side by side.
#include "blk_bits.cuh"
#include "blk_internal.h"

namespace blk {
namespace {

constexpr int kMaxRegionsPerEnv = 32; // more disjoint regions in one env: its bounding box goes to the tile path
constexpr int kRegionLists = 4;       // size classes, see launch_region_relight
constexpr int kMaxSide = 64;          // region columns along x or z in one item

// Low bit of each byte -> 4 packed bits.
__device__ inline uint32_t pack4_lo(uint32_t m) { return ((m & 0x01010101u) * 0x10204080u) >> 28; }

struct Box {
    int32_t x0, x1, z0, z1, y0, y1; // inclusive
};

__device__ inline bool touches(const Box& a, const Box& b)
{
    return a.x0 - 1 <= b.x1 && b.x0 <= a.x1 + 1 && a.z0 - 1 <= b.z1 && b.z0 <= a.z1 + 1 && a.y0 - 1 <= b.y1
        && b.y0 <= a.y1 + 1;
}

__device__ inline Box hull(const Box& a, const Box& b)
{
    return Box { min(a.x0, b.x0), max(a.x1, b.x1), min(a.z0, b.z0), max(a.z1, b.z1), min(a.y0, b.y0),
        max(a.y1, b.y1) };
}

// One thread per env: merges the env's dirty cubes (the change records that
// mark_changes_kernel marked) into regions and files each region by size
// (region lists), or, when it exceeds the region kernels' limits, widens the
// dirty row windows of the tiles it covers (tile path).
__global__ void region_build_kernel(RegionBuildArgs a)
{
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    if (env >= a.num_envs)
        return;
    Box reg[kMaxRegionsPerEnv];
    int n = 0;
    bool overflow = false;
    const uint64_t beg = 2ull * a.env_offset[env], end = 2ull * a.env_offset[env + 1];
    for (uint64_t i = beg; i < end; ++i) {
        const uint4 c = a.changes[i];
        if ((c.w & 3u) != 3u) // recorded and marked for relight
            continue;
        const int32_t x = static_cast<int32_t>(c.x & 0xFFFFu), z = static_cast<int32_t>(c.x >> 16);
        const int32_t ylo = static_cast<int32_t>(c.z & 0xFFFFu), yhi = static_cast<int32_t>(c.z >> 16);
        Box b { max(x - kMaxDistance, 0), min(x + kMaxDistance, a.W - 1), max(z - kMaxDistance, 0),
            min(z + kMaxDistance, a.D - 1), max(ylo - kMaxDistance, 0), min(yhi + kMaxDistance, a.H - 1) };
        if (overflow) {
            reg[0] = hull(reg[0], b);
            continue;
        }
        // Absorb every region the growing box touches; the others are
        // pairwise apart already.
        for (bool merged = true; merged;) {
            merged = false;
            for (int j = 0; j < n; ++j)
                if (touches(b, reg[j])) {
                    b = hull(b, reg[j]);
                    reg[j] = reg[--n];
                    merged = true;
                    break;
                }
        }
        if (n == kMaxRegionsPerEnv) {
            for (int j = 1; j < n; ++j)
                b = hull(b, reg[j]);
            reg[0] = hull(b, reg[0]);
            n = 1;
            overflow = true;
        } else {
            reg[n++] = b;
        }
    }
    // Files one item: solve the columns of box e (sides fixed by the resident
    // ring where `sides` says so), write those of box w; into the tile path
    // when the lists are full.
    auto emit = [&](int list, const Box& e, const Box& w, uint32_t sides) {
        const uint32_t k = atomicAdd(a.counts + list, 1u);
        if (k < a.capacity) {
            uint4* it = a.lists[list] + 2ull * k;
            it[0] = make_uint4(env, static_cast<uint32_t>(e.x0) | (static_cast<uint32_t>(e.z0) << 16),
                static_cast<uint32_t>(e.x1 - e.x0 + 1) | (static_cast<uint32_t>(e.z1 - e.z0 + 1) << 16),
                static_cast<uint32_t>(e.y0) | (static_cast<uint32_t>(e.y1 - e.y0 + 1) << 16));
            it[1] = make_uint4(static_cast<uint32_t>(w.x0) | (static_cast<uint32_t>(w.z0) << 16),
                static_cast<uint32_t>(w.x1 - w.x0 + 1) | (static_cast<uint32_t>(w.z1 - w.z0 + 1) << 16), sides, 0u);
            return;
        }
        for (int32_t tz = w.z0 / 32; tz <= w.z1 / 32; ++tz)
            for (int32_t tx = w.x0 / 32; tx <= w.x1 / 32; ++tx) {
                const uint64_t t = static_cast<uint64_t>(env) * a.tiles_x * a.tiles_z
                    + static_cast<uint64_t>(tz) * a.tiles_x + tx;
                atomicMin(a.win_lo + t, static_cast<uint32_t>(w.y0));
                atomicMax(a.win_hi + t, static_cast<uint32_t>(w.y1));
            }
    };
    for (int j = 0; j < n; ++j) {
        const Box& b = reg[j];
        const int32_t nx = b.x1 - b.x0 + 1, nz = b.z1 - b.z0 + 1, ny = b.y1 - b.y0 + 1;
        const int32_t span = ny + 2;                // the region's rows and its two ring rows
        const int nb = span <= 32 ? 1 : (span <= 64 ? 2 : 0);
        if (nb == 0) {                              // taller than the region kernels' words: tile path
            for (int32_t tz = b.z0 / 32; tz <= b.z1 / 32; ++tz)
                for (int32_t tx = b.x0 / 32; tx <= b.x1 / 32; ++tx) {
                    const uint64_t t = static_cast<uint64_t>(env) * a.tiles_x * a.tiles_z
                        + static_cast<uint64_t>(tz) * a.tiles_x + tx;
                    atomicMin(a.win_lo + t, static_cast<uint32_t>(b.y0));
                    atomicMax(a.win_hi + t, static_cast<uint32_t>(b.y1));
                }
            continue;
        }
        const int64_t cols = static_cast<int64_t>(nx) * nz;
        const int64_t big = 4096;                   // columns of the larger classes
        if (nx <= kMaxSide && nz <= kMaxSide && cols <= big) {
            emit((cols <= 1024 ? 0 : 2) + nb - 1, b, b, 0xFu);
            continue;
        }
        // Larger: sub-boxes of 32 x 32 columns, each solved over itself and the
        // region's columns within 14 of it. A side of that box inside the
        // region lies 15 columns from the sub-box, beyond the reach of light,
        // so it holds nothing; a side on the region's ring is held at the
        // resident light.
        const int32_t sub_x = 32;
        for (int32_t sz = b.z0; sz <= b.z1; sz += 32)
            for (int32_t sx = b.x0; sx <= b.x1; sx += sub_x) {
                const Box w { sx, min(sx + sub_x - 1, b.x1), sz, min(sz + 31, b.z1), b.y0, b.y1 };
                const Box e { max(w.x0 - kMaxDistance, b.x0), min(w.x1 + kMaxDistance, b.x1),
                    max(w.z0 - kMaxDistance, b.z0), min(w.z1 + kMaxDistance, b.z1), b.y0, b.y1 };
                const uint32_t sides = (e.x0 == b.x0 ? 1u : 0u) | (e.x1 == b.x1 ? 2u : 0u)
                    | (e.z0 == b.z0 ? 4u : 0u) | (e.z1 == b.z1 ? 8u : 0u);
                emit(2 + nb - 1, e, w, sides);
            }
    }
}

// 16 rows of a resident column from one aligned 16-byte chunk: open (Air or
// Torch) and torch bits.
__device__ inline void id_chunk_bits(const uint4 v, uint32_t& open, uint32_t& torch)
{
    const uint32_t w[4] = { v.x, v.y, v.z, v.w };
    open = 0u;
    torch = 0u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        open |= pack4_hi(zero_bytes(w[j] & 0xFBFBFBFBu)) << (4 * j);
        torch |= pack4_hi(zero_bytes(w[j] ^ 0x04040404u)) << (4 * j);
    }
}

// Bits [off, off + 32) of the concatenated 16-bit pieces m0, m1, m2 (off < 16).
__device__ inline uint32_t window32(uint32_t m0, uint32_t m1, uint32_t m2, int off)
{
    const uint64_t v = static_cast<uint64_t>(m0) | (static_cast<uint64_t>(m1) << 16) | (static_cast<uint64_t>(m2) << 32);
    return static_cast<uint32_t>(v >> off);
}

// Per-class limits of the region kernels. A CTA of THREADS threads owns CPT
// columns of the solved box per thread (column d = tid + k * THREADS); NB
// words of 32 rows per column.
template <int THREADS, int CPT, int NB>
struct RegionClass {
    static constexpr int kMaxCols = THREADS * CPT;           // columns of the solved box
    static constexpr int kRing = 4 * kMaxSide;               // ring columns (corners neighbour no solved cell)
    static constexpr int kMaxExt = kMaxCols + kRing + 4;     // with the ring
    static constexpr int kCtasPerSm = CPT == 1 ? 2048 / THREADS : (THREADS <= 256 ? 4 : (THREADS <= 512 ? 2 : 1));
    static constexpr int kParkWords = THREADS * CPT * NB * 4; // parked block counters per CTA
};

template <int THREADS, int CPT, int NB>
struct RegionSmem {
    using K = RegionClass<THREADS, CPT, NB>;
    uint32_t open[NB][K::kMaxExt];  // open cells of the solved rows (solved columns)
    uint32_t set[2][NB][K::kMaxExt];// level set S, ping-pong (set[1] holds torch bits before a block flood)
    uint32_t ring[8][NB][K::kRing]; // level planes of the ring columns: block 0..3, sky 4..7
    int16_t top[K::kMaxExt];        // local y of each solved column's highest opaque cell
};

// Cells of level >= L among 32 rows given as level bit planes p[0..3].
__device__ inline uint32_t at_least(int L, const uint32_t (&p)[4])
{
    uint32_t ge = 0u, eq = 0xFFFFFFFFu;
#pragma unroll
    for (int i = 3; i >= 0; --i) {
        const uint32_t m = ((L >> i) & 1) ? 0u : 0xFFFFFFFFu; // bit i of L clear: a set p[i] exceeds it
        ge |= eq & p[i] & m;
        eq &= m ? ~p[i] : p[i];
    }
    return ge | eq;
}

// The region kernels: a CTA solves one region at a time (persistent over its
// list). NB words of 32 rows from row wb = y0 - 1 hold the region's rows
// (bits 1 .. ny) and its two ring rows (bits 0 and ny + 1). Threads below the
// ring length also own one ring column. The ext column pitch is nx + 2.
template <int THREADS, int CPT, int NB>
__global__ void __launch_bounds__(THREADS, RegionClass<THREADS, CPT, NB>::kCtasPerSm)
    relight_region_kernel(RegionRelightArgs a)
{
    using K = RegionClass<THREADS, CPT, NB>;
    using Sm = RegionSmem<THREADS, CPT, NB>;
    static_assert(K::kRing <= THREADS, "one ring column per thread");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Sm& s = *reinterpret_cast<Sm*>(smem_raw);
    const int tid = threadIdx.x;
    const uint32_t count = min(*a.count, a.capacity);
    uint32_t* park = a.park + static_cast<uint64_t>(blockIdx.x) * K::kParkWords;

    for (uint32_t item = blockIdx.x; item < count; item += gridDim.x) {
        const uint4 rec = a.regions[2ull * item];
        const uint4 wrt = a.regions[2ull * item + 1];
        const uint32_t env = rec.x;
        // Columns written (a sub-box of the solved box for a split region),
        // and which sides of the solved box are held at the resident ring.
        const int32_t wx0 = static_cast<int32_t>(wrt.x & 0xFFFFu), wz0 = static_cast<int32_t>(wrt.x >> 16);
        const int32_t wnx = static_cast<int32_t>(wrt.y & 0xFFFFu), wnz = static_cast<int32_t>(wrt.y >> 16);
        const uint32_t sides = wrt.z;
        const int32_t x0 = static_cast<int32_t>(rec.y & 0xFFFFu), z0 = static_cast<int32_t>(rec.y >> 16);
        const int32_t nx = static_cast<int32_t>(rec.z & 0xFFFFu), nz = static_cast<int32_t>(rec.z >> 16);
        const int32_t y0 = static_cast<int32_t>(rec.w & 0xFFFFu), ny = static_cast<int32_t>(rec.w >> 16);
        const int32_t H = a.H;
        const int P = nx + 2;                 // ext pitch
        const int32_t wb = y0 - 1;            // row of bit 0 of word 0 (the lower ring row)
        const int32_t cs = wb & ~15;          // first 16-row chunk of the words' rows
        const int off = wb - cs;              // 0 .. 15
        const int w_hi = (ny + 1) >> 5;       // word and bit of the upper ring row
        const uint32_t b_hi = 1u << ((ny + 1) & 31);
        const uint8_t* ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
        uint8_t* light = a.light + static_cast<uint64_t>(env) * a.env_stride;
        const int16_t* hmap = a.hmap + static_cast<uint64_t>(env) * a.columns;
        const int32_t origin_y = __ldg(&a.origins[env].y);
        uint32_t dom[NB]; // the region's rows: bits 1 .. ny of the word stream
#pragma unroll
        for (int w = 0; w < NB; ++w) {
            const int lo = max(1 - 32 * w, 0), hi = min(ny - 32 * w, 31);
            dom[w] = lo > hi ? 0u : ((hi == 31 ? 0xFFFFFFFFu : ((1u << (hi + 1)) - 1u)) & ~((1u << lo) - 1u));
        }

        // ---- own region columns: open and torch bits, top, ring-row levels ----
        // Per own column: ext index (low 16 bits, 0xFFFF = none) and the levels
        // of its ring rows (high 16 bits: block lo | block hi << 4 | sky lo << 8
        // | sky hi << 12).
        uint32_t cl[CPT];
        bool any_torch = false, any_dark = false, any_ring_block = false;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int d = tid + k * THREADS;
            cl[k] = 0xFFFFu;
            if (d >= nx * nz)
                continue;
            const int dx = d % nx, dz = d / nx;
            const int c = (dz + 1) * P + dx + 1;
            const uint64_t gcol = static_cast<uint64_t>(z0 + dz) * a.W + (x0 + dx);
            const uint8_t* idc = ids + gcol * H;
            const uint8_t* lc = light + gcol * H;
            uint4 chunk[2 * NB + 1];
#pragma unroll
            for (int q = 0; q < 2 * NB + 1; ++q) {
                const int32_t r = cs + 16 * q;
                chunk[q] = r >= 0 && r < H ? __ldg(reinterpret_cast<const uint4*>(idc + r))
                                           : make_uint4(0x03030303u, 0x03030303u, 0x03030303u, 0x03030303u);
            }
            const int32_t t = static_cast<int32_t>(__ldg(hmap + gcol)) - origin_y;
            const uint32_t lo = wb >= 0 ? lc[wb] : 0u;
            const uint32_t hi = y0 + ny < H ? lc[y0 + ny] : 0u;
            uint32_t mo[2 * NB + 1], mt[2 * NB + 1];
#pragma unroll
            for (int q = 0; q < 2 * NB + 1; ++q)
                id_chunk_bits(chunk[q], mo[q], mt[q]); // rows outside the world read as stone
            s.top[c] = static_cast<int16_t>(t);
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                const uint32_t o = window32(mo[2 * w], mo[2 * w + 1], mo[2 * w + 2], off) & dom[w];
                const uint32_t tb = window32(mt[2 * w], mt[2 * w + 1], mt[2 * w + 2], off) & dom[w];
                s.open[w][c] = o;
                s.set[1][w][c] = tb;
                any_torch |= tb != 0u;
                any_dark |= (o & ~above_mask(wb + 32 * w, t)) != 0u;
            }
            cl[k] = static_cast<uint32_t>(c) | (((lo & 15u) | ((hi & 15u) << 4) | ((lo >> 4) << 8) | ((hi >> 4) << 12)) << 16);
            any_ring_block |= ((lo | hi) & 15u) != 0u;
        }

        // ---- own ring column: its level planes over the region's rows -------
        // Ring column r goes to thread (nx * nz + r) % THREADS: the slots past
        // the solved box's last column first, so that ring work falls on
        // threads with fewer own columns.
        const int n_ring = 2 * nx + 2 * nz;
        const int ri = (tid - (nx * nz) % THREADS + THREADS) % THREADS; // this thread's ring index
        int rc = -1;
        if (ri < n_ring) {
            int ex, ez;
            if (ri < nx) {
                ex = ri + 1;
                ez = 0;
            } else if (ri < 2 * nx) {
                ex = ri - nx + 1;
                ez = nz + 1;
            } else if (ri < 2 * nx + nz) {
                ex = 0;
                ez = ri - 2 * nx + 1;
            } else {
                ex = nx + 1;
                ez = ri - 2 * nx - nz + 1;
            }
            rc = ez * P + ex;
            const int32_t gx = x0 - 1 + ex, gz = z0 - 1 + ez;
            const uint32_t side = ex == 0 ? 1u : (ex == nx + 1 ? 2u : (ez == 0 ? 4u : 8u));
            const bool inside = (sides & side) != 0u && gx >= 0 && gz >= 0 && gx < a.W && gz < a.D;
            const uint8_t* lc = light + (static_cast<uint64_t>(inside ? gz : 0) * a.W + (inside ? gx : 0)) * H;
            uint4 v[2 * NB + 1];
#pragma unroll
            for (int q = 0; q < 2 * NB + 1; ++q) {
                const int32_t r = cs + 16 * q;
                v[q] = inside && r >= 0 && r < H ? __ldg(reinterpret_cast<const uint4*>(lc + r))
                                                 : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                // Plane i (block bits 0..3, sky bits 4..7) of the chunks, then
                // the words of the stream.
                uint32_t m[2 * NB + 1];
#pragma unroll
                for (int q = 0; q < 2 * NB + 1; ++q)
                    m[q] = pack4_lo(v[q].x >> i) | (pack4_lo(v[q].y >> i) << 4) | (pack4_lo(v[q].z >> i) << 8)
                        | (pack4_lo(v[q].w >> i) << 12);
#pragma unroll
                for (int w = 0; w < NB; ++w) {
                    const uint32_t pl = window32(m[2 * w], m[2 * w + 1], m[2 * w + 2], off) & dom[w];
                    s.ring[i][w][ri] = pl;
                    if (i < 4)
                        any_ring_block |= pl != 0u;
                }
            }
        }
        const bool need_block = __syncthreads_or(any_torch || any_ring_block) != 0;
        const bool need_sky = __syncthreads_or(any_dark) != 0;

        // ---- the floods: block (f = 0) and sky (f = 1) -------------------------
        // 14 level steps over the own columns; their level counters in cnt
        // (bit planes: parity of the level, bit 1, bit 2, bit 3). The block
        // counters wait in this CTA's scratch slice during a sky flood.
        uint32_t cnt[CPT][NB][4];
        const bool parked = need_block && need_sky;
        for (int f = need_block ? 0 : 1; f < (need_sky ? 2 : 1); ++f) {
            const bool sky = f == 1;
            const int lv_shift = sky ? 24 : 16;
            uint32_t own[CPT][NB];
            // Level-15 set: sources, and fixed cells of level 15.
#pragma unroll
            for (int k = 0; k < CPT; ++k) {
                const bool has = (cl[k] & 0xFFFFu) != 0xFFFFu;
                const int c = has ? static_cast<int>(cl[k] & 0xFFFFu) : 0;
                const uint32_t lv = cl[k] >> lv_shift;
                const int32_t t = s.top[c];
#pragma unroll
                for (int w = 0; w < NB; ++w) {
                    uint32_t v = 0u;
                    if (has) {
                        v = sky ? (s.open[w][c] & above_mask(wb + 32 * w, t)) : s.set[1][w][c];
                        if (w == 0 && (lv & 15u) == 15u)
                            v |= 1u;
                        if (w == w_hi && ((lv >> 4) & 15u) == 15u)
                            v |= b_hi;
                    }
                    own[k][w] = v;
                    cnt[k][w][0] = v;
                    cnt[k][w][1] = cnt[k][w][2] = cnt[k][w][3] = 0u;
                }
            }
            __syncthreads(); // the torch bits in set[1] are read
#pragma unroll
            for (int k = 0; k < CPT; ++k)
                if ((cl[k] & 0xFFFFu) != 0xFFFFu)
#pragma unroll
                    for (int w = 0; w < NB; ++w)
                        s.set[0][w][cl[k] & 0xFFFFu] = own[k][w];
            if (rc >= 0)
#pragma unroll
                for (int w = 0; w < NB; ++w) {
                    const uint32_t pl[4] = { s.ring[4 * f][w][ri], s.ring[4 * f + 1][w][ri],
                        s.ring[4 * f + 2][w][ri], s.ring[4 * f + 3][w][ri] };
                    s.set[0][w][rc] = at_least(15, pl);
                }
            __syncthreads();
            // Steps in groups of four (levels 14 - 4g .. 11 - 4g): the parity
            // tests of the counters are compile-time within a group.
            for (int g = 0; g < 4; ++g) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int step = 4 * g + u + 1;
                    if (step > kMaxDistance)
                        break;
                    const int level = 15 - step; // level & 3 == (2 - u) & 3
                    const uint32_t* cur = s.set[(step - 1) & 1][0];
                    uint32_t* nxt = s.set[step & 1][0];
#pragma unroll
                    for (int k = 0; k < CPT; ++k) {
                        if ((cl[k] & 0xFFFFu) == 0xFFFFu)
                            continue;
                        const int c = static_cast<int>(cl[k] & 0xFFFFu);
                        const uint32_t lv = cl[k] >> lv_shift;
                        const bool inj_lo = (lv & 15u) == static_cast<uint32_t>(level);
                        const bool inj_hi = ((lv >> 4) & 15u) == static_cast<uint32_t>(level);
                        // One word: the own word stays in a register; two: it is
                        // read back from the set (fewer registers per column).
                        uint32_t ow[NB];
#pragma unroll
                        for (int w = 0; w < NB; ++w)
                            ow[w] = NB == 1 ? own[k][w] : cur[w * K::kMaxExt + c];
                        uint32_t v[NB];
#pragma unroll
                        for (int w = 0; w < NB; ++w) {
                            const uint32_t* Bw = cur + w * K::kMaxExt + c;
                            const uint32_t below = w > 0 ? ow[w > 0 ? w - 1 : 0] : 0u;
                            const uint32_t above = w + 1 < NB ? ow[w + 1 < NB ? w + 1 : w] : 0u;
                            const uint32_t up = __funnelshift_l(below, ow[w], 1); // cell y takes y-1
                            const uint32_t dn = __funnelshift_r(ow[w], above, 1); // cell y takes y+1
                            const uint32_t nb = up | dn | Bw[-1] | Bw[1] | Bw[-P] | Bw[P];
                            uint32_t x = ow[w] | (s.open[w][c] & nb);
                            if (w == 0 && inj_lo)
                                x |= 1u;
                            if (w == w_hi && inj_hi)
                                x |= b_hi;
                            v[w] = x;
                        }
#pragma unroll
                        for (int w = 0; w < NB; ++w) {
                            if (NB == 1)
                                own[k][w] = v[w];
                            nxt[w * K::kMaxExt + c] = v[w];
                            cnt[k][w][0] ^= v[w];
                            if ((u & 1) == 0) // level even
                                cnt[k][w][1] ^= v[w];
                            if (u == 2) // level % 4 == 0
                                cnt[k][w][2] ^= v[w];
                            if (level == 8)
                                cnt[k][w][3] = v[w];
                        }
                    }
                    if (rc >= 0) {
#pragma unroll
                        for (int w = 0; w < NB; ++w) {
                            const uint32_t pl[4] = { s.ring[4 * f][w][ri], s.ring[4 * f + 1][w][ri],
                                s.ring[4 * f + 2][w][ri], s.ring[4 * f + 3][w][ri] };
                            nxt[w * K::kMaxExt + rc] = at_least(level, pl);
                        }
                    }
                    __syncthreads();
                }
            }
            if (!sky && parked)
#pragma unroll
                for (int k = 0; k < CPT; ++k)
#pragma unroll
                    for (int w = 0; w < NB; ++w)
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            park[((k * NB + w) * 4 + i) * THREADS + tid] = cnt[k][w][i];
        }

        // ---- new light of the region's rows -----------------------------------
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            if ((cl[k] & 0xFFFFu) == 0xFFFFu)
                continue;
            const int d = tid + k * THREADS;
            const int dx = d % nx, dz = d / nx;
            if (x0 + dx < wx0 || x0 + dx >= wx0 + wnx || z0 + dz < wz0 || z0 + dz >= wz0 + wnz)
                continue; // solved for the sub-box only
            uint8_t* lc = light + (static_cast<uint64_t>(z0 + dz) * a.W + (x0 + dx)) * H;
            const int32_t t = s.top[cl[k] & 0xFFFFu];
            // Light bytes of the word stream (rows wb ..), 4 rows per 32-bit
            // word, stored as aligned 4-row words of the column from row
            // A = wb & ~3: memory word j takes stream bytes 4j - e .. 4j - e + 3
            // (e = wb - A), i.e. the stream words j - 1 and j.
            const int32_t A = wb & ~3;
            const uint32_t sh = 8u * static_cast<uint32_t>(wb - A);
            uint32_t carry = 0u; // stream word 8w - 1
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                uint32_t bp[4], sp[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    bp[i] = parked ? park[((k * NB + w) * 4 + i) * THREADS + tid]
                                   : (need_block && !need_sky ? cnt[k][w][i] : 0u);
                    sp[i] = need_sky ? cnt[k][w][i] : above_mask(wb + 32 * w, t); // no dark cell: 15 above the top
                }
                uint32_t bn[4], sn[4];
                level_nibbles(bp[0], bp[1], bp[2], bp[3], bn[0], bn[1], bn[2], bn[3]);
                level_nibbles(sp[0], sp[1], sp[2], sp[3], sn[0], sn[1], sn[2], sn[3]);
                // nibble q of n_i = level of row 4q + i of the word.
                uint32_t out[9];
                out[0] = carry;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    uint32_t word = 0u;
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        word |= (((bn[i] >> (4 * q)) & 15u) | (((sn[i] >> (4 * q)) & 15u) << 4)) << (8 * i);
                    out[q + 1] = word;
                }
                carry = out[8];
#pragma unroll
                for (int q = 0; q <= 8; ++q) {
                    if (q == 8 && w + 1 < NB)
                        break; // memory word 8(w + 1) is stored with the next stream word
                    const int j = 8 * w + q;
                    const int32_t r = A + 4 * j; // rows r .. r + 3
                    const int32_t lo = max(r, y0), hi = min(r + 3, y0 + ny - 1);
                    if (lo > hi)
                        continue;
                    const uint32_t word = __funnelshift_l(out[q], q < 8 ? out[q + 1] : 0u, sh);
                    if (lo == r && hi == r + 3) {
                        *reinterpret_cast<uint32_t*>(lc + r) = word;
                    } else {
                        for (int32_t y = lo; y <= hi; ++y)
                            lc[y] = static_cast<uint8_t>(word >> (8 * (y - r)));
                    }
                }
            }
        }
        __syncthreads(); // shared planes are reused by the next region
    }
}

template <int THREADS, int CPT, int NB>
int launch_region_list(blk_ctx* ctx, const RegionRelightArgs& base, int list, cudaStream_t st)
{
    using K = RegionClass<THREADS, CPT, NB>;
    static bool attr_set[64] = {};
    const int dev = ctx->device;
    constexpr size_t kSmem = sizeof(RegionSmem<THREADS, CPT, NB>);
    if (dev < 0 || dev >= 64) {
        set_error("device index out of range");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(relight_region_kernel<THREADS, CPT, NB>,
            cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
        if (e != cudaSuccess)
            return cuda_fail(e, "cudaFuncSetAttribute(relight_region_kernel)");
        attr_set[dev] = true;
    }
    RegionRelightArgs a = base;
    a.regions = ctx->region_lists + 2ull * list * ctx->region_capacity;
    a.count = ctx->region_counts + list;
    a.park = ctx->region_park + static_cast<uint64_t>(list) * ctx->park_ctas * region_park_words_per_sm();
    const uint32_t grid = ctx->park_ctas * K::kCtasPerSm;
    static_assert(K::kCtasPerSm * K::kParkWords <= 32768, "park slice per SM");
    relight_region_kernel<THREADS, CPT, NB><<<grid, THREADS, kSmem, st>>>(a);
    return cuda_fail(cudaGetLastError(), "relight_region_kernel launch");
}

__global__ void dirty_compact_kernel(const uint32_t* win_lo, const uint32_t* win_hi, uint64_t n_tiles,
    uint32_t* window, uint32_t* list, uint32_t* count)
{
    for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < n_tiles;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t lo = win_lo[t], hi = win_hi[t];
        if (lo <= hi && hi != 0xFFFFFFFFu) {
            window[t] = lo | (hi << 16);
            list[atomicAdd(count, 1u)] = static_cast<uint32_t>(t);
        }
    }
}

} // namespace

// Scratch words one region kernel needs per SM (block counters parked during
// a sky flood); every size class fits in it, and each class has its own area.
uint64_t region_park_words_per_sm() { return 32768; }

// The relight of an edit step, after mark_changes_kernel: regions per env,
// the tile path's dirty tiles (regions beyond the region kernels' limits),
// then the tile kernel over those tiles and the region kernels over their
// lists. Everything stays on the device: no count comes back to the host.
int launch_relight(blk_ctx* ctx, cudaStream_t st)
{
    const uint64_t n_tiles = static_cast<uint64_t>(ctx->cfg.num_envs) * ctx->tiles_x * ctx->tiles_z;
    uint32_t* win_lo = ctx->dirty_window;
    uint32_t* win_hi = ctx->dirty_window + n_tiles;
    if (cudaMemsetAsync(win_lo, 0xFF, n_tiles * sizeof(uint32_t), st) != cudaSuccess
        || cudaMemsetAsync(win_hi, 0, n_tiles * sizeof(uint32_t), st) != cudaSuccess
        || cudaMemsetAsync(ctx->region_counts, 0, 4 * sizeof(uint32_t), st) != cudaSuccess
        || cudaMemsetAsync(ctx->dirty_count, 0, sizeof(uint32_t), st) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "relight memsets");
    RegionBuildArgs b {};
    b.changes = ctx->edit_changes;
    b.env_offset = ctx->edit_env_offset;
    b.num_envs = ctx->cfg.num_envs;
    b.W = static_cast<int32_t>(ctx->cfg.width);
    b.H = static_cast<int32_t>(ctx->cfg.height);
    b.D = static_cast<int32_t>(ctx->cfg.depth);
    for (int k = 0; k < kRegionLists; ++k)
        b.lists[k] = ctx->region_lists + 2ull * k * ctx->region_capacity;
    b.counts = ctx->region_counts;
    b.capacity = ctx->region_capacity;
    b.win_lo = win_lo;
    b.win_hi = win_hi;
    b.tiles_x = static_cast<int32_t>(ctx->tiles_x);
    b.tiles_z = static_cast<int32_t>(ctx->tiles_z);
    b.flags = ctx->flags;
    region_build_kernel<<<(b.num_envs + 127) / 128, 128, 0, st>>>(b);
    // Pack windows in place into win_lo's slots: window[t] = lo | hi << 16.
    uint64_t blocks = (n_tiles + 255) / 256;
    if (blocks > 148ull * 16)
        blocks = 148ull * 16;
    dirty_compact_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(win_lo, win_hi, n_tiles, win_lo,
        ctx->dirty_list, ctx->dirty_count);
    const int rc = cuda_fail(cudaGetLastError(), "relight region build launch");
    if (rc != BLK_OK)
        return rc;
    // The region kernels run on the context's side streams, forked from and
    // joined back into the caller's stream, beside the tile path on it (one
    // CTA per tile of the batch at most; CTAs past the device-side dirty count
    // exit at once).
    if (cudaEventRecord(ctx->relight_fork, st) != cudaSuccess)
        return cuda_fail(cudaGetLastError(), "relight fork");
    for (int k = 0; k < 4; ++k)
        if (cudaStreamWaitEvent(ctx->relight_streams[k], ctx->relight_fork, 0) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "relight fork wait");
    const int rr = launch_region_relight(ctx, ctx->relight_streams);
    if (rr != BLK_OK)
        return rr;
    const int rt = launch_tiles(ctx, 1, static_cast<uint32_t>(n_tiles), st);
    for (int k = 0; k < 4; ++k)
        if (cudaEventRecord(ctx->relight_join[k], ctx->relight_streams[k]) != cudaSuccess
            || cudaStreamWaitEvent(st, ctx->relight_join[k], 0) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "relight join");
    return rt;
}

int launch_region_relight(blk_ctx* ctx, const cudaStream_t (&side)[4])
{
    RegionRelightArgs a {};
    a.ids = ctx->ids;
    a.light = ctx->light;
    a.hmap = ctx->hmap;
    a.origins = ctx->origins;
    a.W = static_cast<int32_t>(ctx->cfg.width);
    a.H = static_cast<int32_t>(ctx->cfg.height);
    a.D = static_cast<int32_t>(ctx->cfg.depth);
    a.env_stride = ctx->env_stride;
    a.columns = ctx->columns_per_env;
    a.capacity = ctx->region_capacity;
    a.park = ctx->region_park;
    // Size classes (lists of region_build_kernel), each on its own stream so
    // that their tails overlap, all at most 64 columns a side: 0: <= 1024
    // columns, one word (1024 threads x 1 column, two CTAs per SM); 1: the
    // same, two words (512 x 2); 2: <= 4096 columns (a region, or a sub-box of
    // a larger one with its 14-column surround), one word (1024 x 4); 3: the
    // same, two words.
    int rc = launch_region_list<1024, 1, 1>(ctx, a, 0, side[0]);
    if (rc == BLK_OK)
        rc = launch_region_list<512, 2, 2>(ctx, a, 1, side[1]);
    if (rc == BLK_OK)
        rc = launch_region_list<1024, 4, 1>(ctx, a, 2, side[2]);
    if (rc == BLK_OK)
        rc = launch_region_list<1024, 4, 2>(ctx, a, 3, side[3]);
    return rc;
}

} // namespace blk
