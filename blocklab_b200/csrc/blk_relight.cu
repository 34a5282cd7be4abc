// Exact incremental relight after edits: the changed cells of an env are
// grouped into regions whose one-cell boundary ring no edit of the step can
// have relit, and each region's light is recomputed from its resident ring.
//
// Why a region with a clean ring is exact. Light is the unique solution of
//     L(v) = opaque(v) ? 0 : max(src(v), max_{n in N6(v)} L(n) - 1, 0)
// (src = 15 at torches for block light, at open cells above the column's top
// for sky light; cells outside the world are opaque). Restricted to a set R of
// cells, the same equation with the values of the cells just outside R held
// fixed has exactly one solution: a positive level needs a neighbour one
// higher, so it is carried by a chain that ends at a source in R or at a fixed
// cell. The light of the whole world restricted to R is such a solution, so
// solving the region problem with the CORRECT ring values gives the new light
// of R.
//
// The dirty prism of a change. Light falls by one per step along 6-connected
// paths, so a changed cell c (or a changed source: every cell of the span a
// column's top moved over) can move the light of v only if |v - c|_1 <= 14.
// That L1 ball lies inside the prism of the change: the columns within L1
// distance 14 of its column (a diamond of at most 421 columns) times the rows
// within 14 of its cell and moved span. Outside the union of the step's
// prisms the old light is the new light.
//
// Regions. Per env the prisms are grouped: two groups join while some pair of
// their columns lies within L1 distance 29 (their diamonds overlap or touch)
// and their row hulls overlap or touch. A region is the union of its group's
// diamonds times the group's row hull. Its ring: the columns at L1 distance
// exactly 15 from the nearest centre (over the hull's rows; each is a
// 4-neighbour of a diamond column), and the rows just below and above the
// hull in the region's columns. The ring avoids every prism: its columns lie
// beyond reach of the group's own centres; a prism of another group reaching a
// ring column would have a centre within 29 of this group's and rows inside
// this hull, and one reaching a ring row would have its rows touching this
// hull, and either would have joined the groups.
//
// Solving a region: with S_k = {v : L(v) >= k}, a fixed cell of level l joins
// the level sets at S_l and stays, a source joins at S_15, and
//     S_k = S_{k+1} | fixed_k | (open & dilate6(S_{k+1}))       k = 14 .. 1,
// one bit per cell, 32 rows of a column per word (as in the tile kernel). The
// region's columns and ring columns are compacted into slots (a column's four
// horizontal neighbours are slot indices), so a CTA works on the diamonds'
// columns only: 421 for a single change instead of a 29 x 29 box (841).
// Regions of more than 62 rows, or beyond the largest size class, are relit by
// the tile kernel's halo path over the tiles they cover (it reads no resident
// light). Every path writes only correct new values, and a region's ring cells
// are never changed by any, so they may run side by side.
#include "blk_bits.cuh"
#include "blk_internal.h"

#include <climits>

namespace blk {
namespace {

constexpr int kMaxPrisms = 64;                // separate prisms of one env; more: the env's hull goes to the tile path
constexpr int kMaxCentres = 32;               // diamond centres of one region; more: the tile path
constexpr int kBuildWarps = 4;                // envs per CTA of region_build_kernel (one warp each)
constexpr int kReach = 2 * kMaxDistance + 1;  // centres this close (L1) have overlapping or touching diamonds
constexpr int kBuildGuard = 4 * kMaxPrisms;   // grouping passes before an env falls back to the tile path

// Low bit of each byte -> 4 packed bits.
__device__ inline uint32_t pack4_lo(uint32_t m) { return ((m & 0x01010101u) * 0x10204080u) >> 28; }

struct Box {
    int32_t x0, x1, z0, z1, y0, y1; // inclusive
};

__device__ inline Box hull(const Box& a, const Box& b)
{
    return Box { min(a.x0, b.x0), max(a.x1, b.x1), min(a.z0, b.z0), max(a.z1, b.z1), min(a.y0, b.y0),
        max(a.y1, b.y1) };
}

// Per-class limits of the region kernels. A CTA of THREADS threads owns CPT
// solved columns per thread (slot d = tid + k * THREADS) and at most one ring
// column (slot kMaxCols + r); NB words of 32 rows per column. The block and
// sky floods run together, so both level counters of a column stay in
// registers.
template <int THREADS, int CPT, int NB>
struct RegionClass {
    static constexpr int kMaxCols = THREADS * CPT;         // solved columns
    static constexpr int kRing = THREADS / 2;              // ring columns
    static constexpr int kZero = kMaxCols + kRing;         // slot that stays empty: neighbours outside the world
    static constexpr int kExt = (kZero + 1 + 3) & ~3;      // slots per plane
    static constexpr int kMapCells = 10 * NB * kExt;       // grid cells the setup map can hold (16 bits each)
    static constexpr int kCtasPerSm = THREADS <= 512 ? 2 : 1;
};

template <int THREADS, int CPT, int NB>
struct RegionSmem {
    using K = RegionClass<THREADS, CPT, NB>;
    uint2 set[2][NB][K::kExt];        // level set S of the block (x) and sky (y) floods, ping-pong; during
                                      // setup (with open) the grid map: slot per grid cell
    uint32_t open[NB][K::kExt];       // open cells of the solved columns
    uint32_t ring[8][NB][K::kRing];   // level planes of the ring columns: block 0..3, sky 4..7
    uint2 nbr[K::kMaxCols];           // slots of each solved column's neighbours: x-1 | x+1 << 16, z-1 | z+1 << 16
    uint16_t pos[K::kMaxCols + K::kRing]; // grid cell of each solved and ring slot
    int16_t top[K::kMaxCols];         // local y of each solved column's highest opaque cell
    uint4 hdr[2][2];                  // item records: this region's and the next one's (prefetched)
    uint32_t cen[2][kMaxCentres];     // their diamond centres, x | z << 16
    uint32_t wcount[THREADS / 32];    // solved | ring << 16 grid cells per warp
};

template <int THREADS, int CPT, int NB>
__host__ __device__ constexpr bool class_fits(uint32_t cols, uint32_t ring, int64_t cells)
{
    using K = RegionClass<THREADS, CPT, NB>;
    return cols <= static_cast<uint32_t>(K::kMaxCols) && ring <= static_cast<uint32_t>(K::kRing)
        && cells <= K::kMapCells;
}

// Item list of a region with the given words, solved and ring columns and
// grid cells: 2 s + nb - 1 for size class s (512 x 1, 1024 x 1 and 1024 x 2
// columns); -1 when none fits (tile path).
__device__ inline int region_list_for(int nb, uint32_t cols, uint32_t ring, int64_t cells)
{
    if (nb == 1) {
        if (class_fits<512, 1, 1>(cols, ring, cells))
            return 0;
        if (class_fits<1024, 1, 1>(cols, ring, cells))
            return 2;
        if (class_fits<1024, 2, 1>(cols, ring, cells))
            return 4;
    } else {
        if (class_fits<512, 1, 2>(cols, ring, cells))
            return 1;
        if (class_fits<1024, 1, 2>(cols, ring, cells))
            return 3;
        if (class_fits<1024, 2, 2>(cols, ring, cells))
            return 5;
    }
    return -1;
}

// Columns q .. q + 31 of world row z that lie within L1 distance r of one of
// the centres, as bits.
__device__ inline uint32_t diamond_row_bits(const uint32_t* cen, int nc, int32_t r, int32_t z, int32_t q)
{
    uint32_t m = 0u;
    for (int i = 0; i < nc; ++i) {
        const int32_t cx = static_cast<int32_t>(cen[i] & 0xFFFFu), cz = static_cast<int32_t>(cen[i] >> 16);
        const int32_t h = r - abs(z - cz);
        if (h < 0)
            continue;
        const int32_t lo = max(cx - h, q) - q, hi = min(cx + h, q + 31) - q;
        if (lo > hi)
            continue;
        m |= (hi == 31 ? 0xFFFFFFFFu : ((2u << hi) - 1u)) & ~((1u << lo) - 1u);
    }
    return m;
}

// Tile path: widens the dirty row windows of the tiles box b covers.
__device__ inline void stamp_tiles(const RegionBuildArgs& a, uint32_t env, const Box& b)
{
    for (int32_t tz = b.z0 / 32; tz <= b.z1 / 32; ++tz)
        for (int32_t tx = b.x0 / 32; tx <= b.x1 / 32; ++tx) {
            const uint64_t t = static_cast<uint64_t>(env) * a.tiles_x * a.tiles_z
                + static_cast<uint64_t>(tz) * a.tiles_x + tx;
            atomicMin(a.win_lo + t, static_cast<uint32_t>(b.y0));
            atomicMax(a.win_hi + t, static_cast<uint32_t>(b.y1));
        }
}

struct BuildWarp {
    uint32_t xz[kMaxPrisms];          // prism column x | z << 16
    int32_t y0[kMaxPrisms], y1[kMaxPrisms]; // prism rows (inclusive)
    int32_t lab[kMaxPrisms];          // group label: the smallest prism index of the group
    int32_t hy0[kMaxPrisms], hy1[kMaxPrisms]; // row hull per label
    uint32_t cen[kMaxCentres];        // centres of the group being filed
};

// One warp per env: the env's marked change records become prisms, the
// prisms are grouped into regions (label propagation until no two groups
// touch), and each region is filed by size (region lists) with its diamond
// centres, or, beyond the region kernels' limits, widens the dirty row windows
// of the tiles it covers (tile path).
__global__ void __launch_bounds__(32 * kBuildWarps) region_build_kernel(RegionBuildArgs a)
{
    __shared__ BuildWarp sw[kBuildWarps];
    const int lane = threadIdx.x & 31;
    BuildWarp& w = sw[threadIdx.x >> 5];
    const uint32_t env = blockIdx.x * kBuildWarps + (threadIdx.x >> 5);
    if (env >= a.num_envs)
        return; // the whole warp
    constexpr unsigned kFull = 0xFFFFFFFFu;
    const unsigned lt = (1u << lane) - 1u;
    const uint64_t beg = 2ull * a.env_offset[env], end = 2ull * a.env_offset[env + 1];

    // ---- prisms: one per changed column and row span --------------------------
    int n = 0; // prisms filed (warp-uniform; may exceed kMaxPrisms)
    Box hb { INT_MAX, INT_MIN, INT_MAX, INT_MIN, INT_MAX, INT_MIN }; // this lane's prisms' cubes (tile path)
    for (uint64_t base = beg; base < end; base += 32) {
        const uint64_t i = base + lane;
        bool mk = false;
        uint32_t xz = 0u;
        int32_t y0 = 0, y1 = 0;
        if (i < end) {
            const uint4 c = a.changes[i];
            if ((c.w & 3u) == 3u) { // recorded and marked for relight
                mk = true;
                xz = c.x;
                const int32_t x = static_cast<int32_t>(xz & 0xFFFFu), z = static_cast<int32_t>(xz >> 16);
                y0 = max(static_cast<int32_t>(c.z & 0xFFFFu) - kMaxDistance, 0);
                y1 = min(static_cast<int32_t>(c.z >> 16) + kMaxDistance, a.H - 1);
                hb = hull(hb, Box { max(x - kMaxDistance, 0), min(x + kMaxDistance, a.W - 1),
                                   max(z - kMaxDistance, 0), min(z + kMaxDistance, a.D - 1), y0, y1 });
                // A filed prism of the same column whose rows touch: widen it.
                for (int j = 0; j < min(n, kMaxPrisms) && mk; ++j)
                    if (w.xz[j] == xz && w.y0[j] - 1 <= y1 && y0 <= w.y1[j] + 1) {
                        atomicMin(&w.y0[j], y0);
                        atomicMax(&w.y1[j], y1);
                        mk = false;
                    }
            }
        }
        const unsigned m = __ballot_sync(kFull, mk);
        if (mk) {
            const int k = n + __popc(m & lt);
            if (k < kMaxPrisms) {
                w.xz[k] = xz;
                w.y0[k] = y0;
                w.y1[k] = y1;
            }
        }
        n += __popc(m);
        __syncwarp();
    }
    bool overflow = n > kMaxPrisms;

    // ---- groups: label propagation over touching prisms ------------------------
    if (!overflow) {
        for (int i = lane; i < n; i += 32)
            w.lab[i] = i;
        __syncwarp();
        bool converged = n == 0;
        for (int it = 0; it < kBuildGuard && !converged; ++it) {
            for (int i = lane; i < n; i += 32) {
                w.hy0[i] = INT_MAX;
                w.hy1[i] = INT_MIN;
            }
            __syncwarp();
            for (int i = lane; i < n; i += 32) {
                atomicMin(&w.hy0[w.lab[i]], w.y0[i]);
                atomicMax(&w.hy1[w.lab[i]], w.y1[i]);
            }
            __syncwarp();
            int nl[2];
            bool changed = false;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const int i = lane + 32 * t;
                nl[t] = -1;
                if (i >= n)
                    continue;
                const int li = w.lab[i];
                int best = li;
                const int32_t xi = static_cast<int32_t>(w.xz[i] & 0xFFFFu), zi = static_cast<int32_t>(w.xz[i] >> 16);
                const int32_t g0 = w.hy0[li], g1 = w.hy1[li];
                for (int j = 0; j < n; ++j) {
                    const int lj = w.lab[j];
                    if (lj >= best)
                        continue;
                    const int32_t d = abs(static_cast<int32_t>(w.xz[j] & 0xFFFFu) - xi)
                        + abs(static_cast<int32_t>(w.xz[j] >> 16) - zi);
                    if (d <= kReach && g0 - 1 <= w.hy1[lj] && w.hy0[lj] <= g1 + 1)
                        best = lj;
                }
                nl[t] = best;
                changed |= best != li;
            }
            __syncwarp();
#pragma unroll
            for (int t = 0; t < 2; ++t)
                if (nl[t] >= 0)
                    w.lab[lane + 32 * t] = nl[t];
            __syncwarp();
            converged = !__any_sync(kFull, changed);
        }
        overflow = !converged;
    }
    if (overflow) {
        // The env's hull goes to the tile path.
        const Box b { __reduce_min_sync(kFull, hb.x0), __reduce_max_sync(kFull, hb.x1),
            __reduce_min_sync(kFull, hb.z0), __reduce_max_sync(kFull, hb.z1), __reduce_min_sync(kFull, hb.y0),
            __reduce_max_sync(kFull, hb.y1) };
        if (lane == 0 && b.x0 <= b.x1)
            stamp_tiles(a, env, b);
        return;
    }

    // ---- file each group: the warp together, one group at a time -------------
    for (int r = 0; r < n; ++r) {
        if (w.lab[r] != r) // warp-uniform
            continue;
        // Distinct centres (in prism order) and the footprint's bounding box.
        int nc = 0;
        int32_t cx0 = INT_MAX, cx1 = INT_MIN, cz0 = INT_MAX, cz1 = INT_MIN;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + lane;
            bool keep = false;
            if (j < n && w.lab[j] == r) {
                const uint32_t xz = w.xz[j];
                const int32_t x = static_cast<int32_t>(xz & 0xFFFFu), z = static_cast<int32_t>(xz >> 16);
                cx0 = min(cx0, x);
                cx1 = max(cx1, x);
                cz0 = min(cz0, z);
                cz1 = max(cz1, z);
                keep = true;
                for (int q = 0; q < j && keep; ++q)
                    keep = !(w.lab[q] == r && w.xz[q] == xz);
            }
            const unsigned m = __ballot_sync(kFull, keep);
            if (keep) {
                const int k = nc + __popc(m & lt);
                if (k < kMaxCentres)
                    w.cen[k] = w.xz[j];
            }
            nc += __popc(m);
        }
        const bool many = nc > kMaxCentres;
        nc = min(nc, kMaxCentres);
        cx0 = __reduce_min_sync(kFull, cx0);
        cx1 = __reduce_max_sync(kFull, cx1);
        cz0 = __reduce_min_sync(kFull, cz0);
        cz1 = __reduce_max_sync(kFull, cz1);
        __syncwarp();
        const Box b { max(cx0 - kMaxDistance, 0), min(cx1 + kMaxDistance, a.W - 1), max(cz0 - kMaxDistance, 0),
            min(cz1 + kMaxDistance, a.D - 1), w.hy0[r], w.hy1[r] };
        const int32_t span = b.y1 - b.y0 + 3; // the region's rows and its two ring rows
        const int nb = span <= 32 ? 1 : (span <= 64 ? 2 : 0);
        int list = -1;
        if (nb != 0 && !many) {
            // Solved and ring columns over the box and its one-column margin,
            // exactly as the region kernel classifies them; a lane per row.
            const int32_t gx0 = max(b.x0 - 1, 0), gx1 = min(b.x1 + 1, a.W - 1);
            uint32_t n_act = 0u, n_ring = 0u;
            for (int32_t z = max(b.z0 - 1, 0) + lane; z <= min(b.z1 + 1, a.D - 1); z += 32)
                for (int32_t q = gx0; q <= gx1; q += 32) {
                    const int32_t qe = min(q + 31, gx1);
                    const uint32_t valid = qe - q == 31 ? 0xFFFFFFFFu : ((2u << (qe - q)) - 1u);
                    const uint32_t m14 = diamond_row_bits(w.cen, nc, kMaxDistance, z, q) & valid;
                    const uint32_t m15 = diamond_row_bits(w.cen, nc, kMaxDistance + 1, z, q) & valid;
                    n_act += __popc(m14);
                    n_ring += __popc(m15 & ~m14);
                }
            n_act = __reduce_add_sync(kFull, n_act);
            n_ring = __reduce_add_sync(kFull, n_ring);
            const int64_t cells = static_cast<int64_t>(b.x1 - b.x0 + 3) * (b.z1 - b.z0 + 3);
            list = region_list_for(nb, n_act, n_ring, cells);
            if (list >= 0) {
                uint32_t k = 0u, co = 0u;
                if (lane == 0) {
                    k = atomicAdd(a.counts + list, 1u);
                    co = atomicAdd(a.counts + kRegionLists, static_cast<uint32_t>(nc));
                }
                k = __shfl_sync(kFull, k, 0);
                co = __shfl_sync(kFull, co, 0);
                if (k < a.capacity && co <= a.capacity && static_cast<uint32_t>(nc) <= a.capacity - co) {
                    if (lane < nc)
                        a.centres[co + lane] = w.cen[lane];
                    if (lane == 0) {
                        uint4* it = a.lists[list] + 2ull * k;
                        it[0] = make_uint4(env, static_cast<uint32_t>(b.x0) | (static_cast<uint32_t>(b.z0) << 16),
                            static_cast<uint32_t>(b.x1 - b.x0 + 1) | (static_cast<uint32_t>(b.z1 - b.z0 + 1) << 16),
                            static_cast<uint32_t>(b.y0) | (static_cast<uint32_t>(b.y1 - b.y0 + 1) << 16));
                        it[1] = make_uint4(co, static_cast<uint32_t>(nc), n_act | (n_ring << 16), 0u);
                    }
                } else {
                    list = -1;
                }
            }
        }
        if (list < 0 && lane == 0)
            stamp_tiles(a, env, b);
        __syncwarp(); // the centre array is reused by the next group
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

// The region kernels: a CTA solves one region at a time, persistent over its
// list. NB words of 32 rows from row wb = y0 - 1 hold the region's rows (bits
// 1 .. ny) and its two ring rows (bits 0 and ny + 1). Setup classifies the
// cells of the region's bounding box and its one-column margin (the grid,
// pitch nx + 2) by L1 distance to the nearest centre, compacts the solved
// (<= 14) and ring (== 15) columns into slots and records each solved column's
// neighbour slots. The block and sky floods then run together: 14 steps over
// (block, sky) word pairs, one barrier per step.
template <int THREADS, int CPT, int NB>
__global__ void __launch_bounds__(THREADS, RegionClass<THREADS, CPT, NB>::kCtasPerSm)
    relight_region_kernel(RegionRelightArgs a)
{
    using K = RegionClass<THREADS, CPT, NB>;
    using Sm = RegionSmem<THREADS, CPT, NB>;
    static_assert(K::kRing <= THREADS, "one ring column per thread");
    static_assert(K::kZero < 0xFFFF, "slots fit 16 bits");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Sm& s = *reinterpret_cast<Sm*>(smem_raw);
    uint16_t* map = reinterpret_cast<uint16_t*>(&s.set[0][0][0]);
    const int tid = threadIdx.x, lane = tid & 31;
    const uint32_t count = min(*a.count, a.capacity);

    // The item record and centres of the next region are copied into shared
    // memory (cp.async) while this one is solved: the header at the start,
    // the centres once the header is in.
    uint32_t item = blockIdx.x;
    int hb = 0; // buffer of this region's record and centres
    if (item < count) {
        if (tid < 2)
            s.hdr[0][tid] = a.regions[2ull * item + tid];
        __syncthreads();
        const uint4 inf0 = s.hdr[0][1];
        if (tid < min(static_cast<int>(inf0.y), kMaxCentres))
            s.cen[0][tid] = __ldg(a.centres + inf0.x + tid);
        __syncthreads();
    }
    for (; item < count; item += gridDim.x, hb ^= 1) {
        const uint4 rec = s.hdr[hb][0];
        const uint4 inf = s.hdr[hb][1];
        const uint32_t next = item + gridDim.x;
        if (tid < 2 && next < count)
            cp_async16(&s.hdr[hb ^ 1][tid], a.regions + 2ull * next + tid);
        const uint32_t env = rec.x;
        const int32_t x0 = static_cast<int32_t>(rec.y & 0xFFFFu), z0 = static_cast<int32_t>(rec.y >> 16);
        const int32_t nx = static_cast<int32_t>(rec.z & 0xFFFFu), nz = static_cast<int32_t>(rec.z >> 16);
        const int32_t y0 = static_cast<int32_t>(rec.w & 0xFFFFu), ny = static_cast<int32_t>(rec.w >> 16);
        const int32_t H = a.H;
        const int P = nx + 2;                 // grid pitch
        // The build files no region past the map; one that were would be
        // flagged and left unsolved (no centres, no grid).
        const bool bad = P * (nz + 2) > K::kMapCells || nx < 1 || nz < 1;
        if (bad && tid == 0)
            atomicOr(a.flags, kFlagRelightRegion);
        const int G = bad ? 0 : P * (nz + 2); // grid cells
        const int nc = bad ? 0 : min(static_cast<int>(inf.y), kMaxCentres);
        const uint32_t* cen = s.cen[hb];
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

        // ---- grid: solved and ring columns, compacted into slots ---------------
        // Kind of grid cell g: 1 solved (L1 distance to the nearest centre <=
        // 14), 2 ring (== 15), 0 neither or outside the world. Two passes:
        // the warps' ballots and counts (cell g = g0 + tid, its coordinates
        // stepped without division), then slots from the prefix of the warp
        // counts (warp w's cells g = 32 w + lane + i THREADS, in that order).
        // The ballots wait in the ring planes, which setup fills later.
        const int warp = tid >> 5;
        const unsigned lt = (1u << lane) - 1u;
        uint2* masks = reinterpret_cast<uint2*>(&s.ring[0][0][0]); // [iteration][warp]: solved, ring
        static_assert((K::kMapCells / THREADS + 1) * (THREADS / 32) * sizeof(uint2) <= sizeof(s.ring),
            "grid ballots fit the ring planes");
        {
            const int step_z = THREADS / P, step_x = THREADS - step_z * P;
            int gx = tid % P, gz = tid / P;
            uint32_t ca = 0u, cr = 0u;
            for (int g0 = 0, it = 0; g0 < G; g0 += THREADS, ++it) { // warp-uniform trip count (ballots)
                int kind = 0;
                const int32_t x = x0 - 1 + gx, z = z0 - 1 + gz;
                if (g0 + tid < G && x >= 0 && z >= 0 && x < a.W && z < a.D) {
                    int32_t m = INT_MAX;
                    for (int i = 0; i < nc; ++i) {
                        const uint32_t c = cen[i];
                        m = min(m, abs(x - static_cast<int32_t>(c & 0xFFFFu)) + abs(z - static_cast<int32_t>(c >> 16)));
                    }
                    kind = m <= kMaxDistance ? 1 : (m == kMaxDistance + 1 ? 2 : 0);
                }
                const unsigned ma = __ballot_sync(0xFFFFFFFFu, kind == 1), mr = __ballot_sync(0xFFFFFFFFu, kind == 2);
                if (lane == 0)
                    masks[it * (THREADS / 32) + warp] = make_uint2(ma, mr);
                ca += __popc(ma);
                cr += __popc(mr);
                gx += step_x;
                gz += step_z;
                if (gx >= P) {
                    gx -= P;
                    ++gz;
                }
            }
            if (lane == 0)
                s.wcount[warp] = ca | (cr << 16);
        }
        __syncthreads();
        uint32_t tot_a = 0u, tot_r = 0u;
        {
            uint32_t base_a = 0u, base_r = 0u;
            for (int w = 0; w < THREADS / 32; ++w) {
                const uint32_t v = s.wcount[w];
                if (w < warp) {
                    base_a += v & 0xFFFFu;
                    base_r += v >> 16;
                }
                tot_a += v & 0xFFFFu;
                tot_r += v >> 16;
            }
            for (int g0 = 0, it = 0; g0 < G; g0 += THREADS, ++it) {
                const int g = g0 + tid;
                const uint2 mk = masks[it * (THREADS / 32) + warp];
                if (g < G) {
                    uint16_t v = static_cast<uint16_t>(K::kZero);
                    if ((mk.x >> lane) & 1u) {
                        const uint32_t d = base_a + __popc(mk.x & lt);
                        if (d < static_cast<uint32_t>(K::kMaxCols)) {
                            v = static_cast<uint16_t>(d);
                            s.pos[d] = static_cast<uint16_t>(g);
                        }
                    } else if ((mk.y >> lane) & 1u) {
                        const uint32_t d = base_r + __popc(mk.y & lt);
                        if (d < static_cast<uint32_t>(K::kRing)) {
                            v = static_cast<uint16_t>(K::kMaxCols + d);
                            s.pos[K::kMaxCols + d] = static_cast<uint16_t>(g);
                        }
                    }
                    map[g] = v;
                }
                base_a += __popc(mk.x);
                base_r += __popc(mk.y);
            }
        }
        __syncthreads();
        const int n_act = min(static_cast<int>(tot_a), K::kMaxCols);
        const int n_ring = min(static_cast<int>(tot_r), K::kRing);
        if (tid == 0 && (tot_a > static_cast<uint32_t>(K::kMaxCols) || tot_r > static_cast<uint32_t>(K::kRing)))
            atomicOr(a.flags, kFlagRelightRegion); // columns past the class stay unsolved
        // Neighbour slots (solved columns lie inside the grid's margin).
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int d = tid + k * THREADS;
            if (d < n_act) {
                const int g = s.pos[d];
                s.nbr[d] = make_uint2(static_cast<uint32_t>(map[g - 1]) | (static_cast<uint32_t>(map[g + 1]) << 16),
                    static_cast<uint32_t>(map[g - P]) | (static_cast<uint32_t>(map[g + P]) << 16));
            }
        }
        __syncthreads(); // the map is read: the planes take the columns
        if (tid < 2 * NB)
            s.set[tid / NB][tid % NB][K::kZero] = make_uint2(0u, 0u);

        // ---- own columns: open bits, top, ring-row levels, level-15 sets -------
        // Per own column: slot (low 16 bits, 0xFFFF = none) and the levels of
        // its ring rows (high 16 bits: block lo | block hi << 4 | sky lo << 8 |
        // sky hi << 12). The level-15 sets: torches and sky sources (open cells
        // above the top), and ring rows of level 15.
        uint32_t cl[CPT];
        uint2 own[CPT][NB];
        bool any_block = false, any_dark = false;
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            const int d = tid + k * THREADS;
            cl[k] = 0xFFFFu;
#pragma unroll
            for (int w = 0; w < NB; ++w)
                own[k][w] = make_uint2(0u, 0u);
            if (d >= n_act)
                continue;
            const int g = s.pos[d];
            const uint64_t gcol = static_cast<uint64_t>(z0 - 1 + g / P) * a.W + (x0 - 1 + g % P);
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
            s.top[d] = static_cast<int16_t>(t);
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                const uint32_t o = window32(mo[2 * w], mo[2 * w + 1], mo[2 * w + 2], off) & dom[w];
                const uint32_t tb = window32(mt[2 * w], mt[2 * w + 1], mt[2 * w + 2], off) & dom[w];
                const uint32_t above = above_mask(wb + 32 * w, t);
                s.open[w][d] = o;
                any_block |= tb != 0u;
                any_dark |= (o & ~above) != 0u;
                uint32_t vb = tb, vs = o & above;
                if (w == 0) {
                    vb |= (lo & 15u) == 15u ? 1u : 0u;
                    vs |= (lo >> 4) == 15u ? 1u : 0u;
                }
                if (w == w_hi) {
                    vb |= (hi & 15u) == 15u ? b_hi : 0u;
                    vs |= (hi >> 4) == 15u ? b_hi : 0u;
                }
                own[k][w] = make_uint2(vb, vs);
                s.set[0][w][d] = own[k][w];
            }
            cl[k] = static_cast<uint32_t>(d) | (((lo & 15u) | ((hi & 15u) << 4) | ((lo >> 4) << 8) | ((hi >> 4) << 12)) << 16);
            any_block |= ((lo | hi) & 15u) != 0u;
        }

        // ---- own ring column: its level planes over the region's rows ---------
        // Ring column r goes to thread (base + r) % THREADS, base = the first
        // warp past the last solved column when the ring fits there (no warp
        // then runs both a solved and a ring column per step, the step's
        // longest path), else the last n_ring threads.
        const int last = (n_act - 1) % THREADS + 1;                 // threads with the most solved columns
        const int ring_base = min((last + 31) & ~31, THREADS - n_ring);
        const int ri = (tid - ring_base + THREADS) % THREADS;       // this thread's ring index
        const int rc = ri < n_ring ? K::kMaxCols + ri : -1;
        if (rc >= 0) {
            const int g = s.pos[rc];
            const uint8_t* lc = light + (static_cast<uint64_t>(z0 - 1 + g / P) * a.W + (x0 - 1 + g % P)) * H;
            uint4 v[2 * NB + 1];
#pragma unroll
            for (int q = 0; q < 2 * NB + 1; ++q) {
                const int32_t r = cs + 16 * q;
                v[q] = r >= 0 && r < H ? __ldg(reinterpret_cast<const uint4*>(lc + r)) : make_uint4(0u, 0u, 0u, 0u);
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
                        any_block |= pl != 0u;
                }
            }
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                const uint32_t pb[4] = { s.ring[0][w][ri], s.ring[1][w][ri], s.ring[2][w][ri], s.ring[3][w][ri] };
                const uint32_t ps[4] = { s.ring[4][w][ri], s.ring[5][w][ri], s.ring[6][w][ri], s.ring[7][w][ri] };
                s.set[0][w][rc] = make_uint2(at_least(15, pb), at_least(15, ps));
            }
        }
        // Floods only where they can give more than the level-15 sets: block
        // light needs a torch or block light on the ring, sky light a dark open
        // cell (else sky = 15 above the top, 0 below).
        if (tid < 2)
            cp_async_wait_all(); // the next record is in (visible after the barrier)
        const bool need_block = __syncthreads_or(any_block) != 0;
        const bool floods = __syncthreads_or(any_dark) != 0 || need_block;
        if (next < count) {
            const uint4 ninf = s.hdr[hb ^ 1][1];
            if (tid < min(static_cast<int>(ninf.y), kMaxCentres))
                cp_async4(&s.cen[hb ^ 1][tid], a.centres + ninf.x + tid);
        }

        // ---- the floods: 14 level steps of both sets ---------------------------
        // Level counters of the own words, block (b = 0) and sky (b = 1), as bit
        // planes: parity of the level, bit 1, bit 2, bit 3.
        uint32_t cnt[CPT][NB][2][4];
#pragma unroll
        for (int k = 0; k < CPT; ++k)
#pragma unroll
            for (int w = 0; w < NB; ++w) {
                cnt[k][w][0][0] = own[k][w].x;
                cnt[k][w][1][0] = own[k][w].y;
#pragma unroll
                for (int i = 1; i < 4; ++i)
                    cnt[k][w][0][i] = cnt[k][w][1][i] = 0u;
            }
        if (floods) {
#pragma unroll 1
            for (int step = 1; step <= kMaxDistance; ++step) {
                const int level = 15 - step;
                const bool even = (level & 1) == 0, four = (level & 3) == 0, eight = level == 8;
                const uint2* cur = s.set[(step - 1) & 1][0];
                uint2* nxt = s.set[step & 1][0];
#pragma unroll
                for (int k = 0; k < CPT; ++k) {
                    if ((cl[k] & 0xFFFFu) == 0xFFFFu)
                        continue;
                    const int c = static_cast<int>(cl[k] & 0xFFFFu);
                    const uint32_t lv = cl[k] >> 16;
                    const uint32_t L = static_cast<uint32_t>(level);
                    const bool ib_lo = (lv & 15u) == L, ib_hi = ((lv >> 4) & 15u) == L;
                    const bool is_lo = ((lv >> 8) & 15u) == L, is_hi = (lv >> 12) == L;
                    const uint2 nbr = s.nbr[c];
                    const int n0 = static_cast<int>(nbr.x & 0xFFFFu), n1 = static_cast<int>(nbr.x >> 16);
                    const int n2 = static_cast<int>(nbr.y & 0xFFFFu), n3 = static_cast<int>(nbr.y >> 16);
                    // One word: the own pair stays in registers; two: it is read
                    // back from the set (fewer registers per column).
                    uint2 ow[NB];
#pragma unroll
                    for (int w = 0; w < NB; ++w)
                        ow[w] = NB == 1 ? own[k][w] : cur[w * K::kExt + c];
                    uint2 v[NB];
#pragma unroll
                    for (int w = 0; w < NB; ++w) {
                        const uint2* Cw = cur + w * K::kExt;
                        const uint2 a0 = Cw[n0], a1 = Cw[n1], a2 = Cw[n2], a3 = Cw[n3];
                        const uint2 below = w > 0 ? ow[w > 0 ? w - 1 : 0] : make_uint2(0u, 0u);
                        const uint2 above = w + 1 < NB ? ow[w + 1 < NB ? w + 1 : w] : make_uint2(0u, 0u);
                        const uint32_t o = s.open[w][c];
                        // cell y takes y-1 (funnel left) and y+1 (funnel right)
                        const uint32_t nbx = __funnelshift_l(below.x, ow[w].x, 1) | __funnelshift_r(ow[w].x, above.x, 1)
                            | a0.x | a1.x | a2.x | a3.x;
                        const uint32_t nby = __funnelshift_l(below.y, ow[w].y, 1) | __funnelshift_r(ow[w].y, above.y, 1)
                            | a0.y | a1.y | a2.y | a3.y;
                        uint32_t xb = ow[w].x | (o & nbx), xs = ow[w].y | (o & nby);
                        if (w == 0) {
                            xb |= ib_lo ? 1u : 0u;
                            xs |= is_lo ? 1u : 0u;
                        }
                        if (w == w_hi) {
                            xb |= ib_hi ? b_hi : 0u;
                            xs |= is_hi ? b_hi : 0u;
                        }
                        v[w] = make_uint2(xb, xs);
                    }
#pragma unroll
                    for (int w = 0; w < NB; ++w) {
                        if (NB == 1)
                            own[k][w] = v[w];
                        nxt[w * K::kExt + c] = v[w];
                        cnt[k][w][0][0] ^= v[w].x;
                        cnt[k][w][1][0] ^= v[w].y;
                        if (even) {
                            cnt[k][w][0][1] ^= v[w].x;
                            cnt[k][w][1][1] ^= v[w].y;
                        }
                        if (four) {
                            cnt[k][w][0][2] ^= v[w].x;
                            cnt[k][w][1][2] ^= v[w].y;
                        }
                        if (eight) {
                            cnt[k][w][0][3] = v[w].x;
                            cnt[k][w][1][3] = v[w].y;
                        }
                    }
                }
                if (rc >= 0) {
#pragma unroll
                    for (int w = 0; w < NB; ++w) {
                        const uint32_t pb[4] = { s.ring[0][w][ri], s.ring[1][w][ri], s.ring[2][w][ri], s.ring[3][w][ri] };
                        const uint32_t ps[4] = { s.ring[4][w][ri], s.ring[5][w][ri], s.ring[6][w][ri], s.ring[7][w][ri] };
                        nxt[w * K::kExt + rc] = make_uint2(at_least(level, pb), at_least(level, ps));
                    }
                }
                __syncthreads();
            }
        }

        // ---- new light of the region's rows ------------------------------------
        // Light bytes of the word stream (rows wb ..), 4 rows per 32-bit word,
        // go out as aligned 4-row memory words of each column from row
        // A = wb & ~3: memory word j takes stream bytes 4j - e .. 4j - e + 3
        // (e = wb - A), i.e. the stream words j - 1 and j. Each thread builds
        // its column's memory words in its warp's staging area (the dead set,
        // open and ring planes; odd pitch kW); the warp then stores them with
        // consecutive lanes on consecutive words of a column (a few lines per
        // store instead of one per lane). Words jlo .. jlo + nw - 1 hold the
        // region's rows (the first and last may be partial: byte stores).
        constexpr int kW = 8 * NB + 1;
        static_assert(THREADS * kW * sizeof(uint32_t) <= sizeof(s.set) + sizeof(s.open) + sizeof(s.ring),
            "output staging fits the dead planes");
        const int32_t A = wb & ~3;
        const uint32_t sh = 8u * static_cast<uint32_t>(wb - A);
        const int jlo = (y0 - A) >> 2;
        const int nw = max(((y0 + ny - 1 - A) >> 2) - jlo + 1, 1);
        const int rq = 32 / nw, rr = 32 - rq * nw; // a lane's step of 32 (column, word) pairs
        uint32_t* stage = reinterpret_cast<uint32_t*>(&s.set[0][0][0]) + (tid & ~31) * kW;
        uint32_t* colbase = reinterpret_cast<uint32_t*>(&s.nbr[0]) + (tid & ~31); // the warp's column offsets (nbr is dead)
#pragma unroll
        for (int k = 0; k < CPT; ++k) {
            if ((cl[k] & 0xFFFFu) != 0xFFFFu) {
                const int g = s.pos[cl[k] & 0xFFFFu];
                colbase[lane] = static_cast<uint32_t>((z0 - 1 + g / P) * a.W + (x0 - 1 + g % P)) * static_cast<uint32_t>(H);
                const int32_t t = s.top[cl[k] & 0xFFFFu];
                uint32_t carry = 0u; // stream word 8w - 1
#pragma unroll
                for (int w = 0; w < NB; ++w) {
                    uint32_t bp[4], sp[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        bp[i] = floods ? cnt[k][w][0][i] : 0u;
                        sp[i] = floods ? cnt[k][w][1][i] : above_mask(wb + 32 * w, t); // no dark cell: 15 above the top
                    }
                    uint32_t bytes[8];
                    planes_to_bytes(bp, sp, bytes);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        stage[lane * kW + 8 * w + q] = __funnelshift_l(q == 0 ? carry : bytes[q > 0 ? q - 1 : 0], bytes[q], sh);
                    carry = bytes[7];
                }
                stage[lane * kW + 8 * NB] = __funnelshift_l(carry, 0u, sh);
            }
            __syncwarp();
            const int dbase = (tid & ~31) + k * THREADS; // slot of lane 0's column
            int c = lane / nw, jj = lane - c * nw;
            for (int p = lane; p < 32 * nw; p += 32) {
                const int d = dbase + c;
                if (d < n_act) {
                    const int j = jlo + jj;
                    const uint32_t word = stage[c * kW + j];
                    uint8_t* lc = light + colbase[c];
                    const int32_t r = A + 4 * j; // rows r .. r + 3
                    const int32_t lo = max(r, y0), hi = min(r + 3, y0 + ny - 1);
                    if (lo == r && hi == r + 3) {
                        *reinterpret_cast<uint32_t*>(lc + r) = word;
                    } else {
                        for (int32_t y = lo; y <= hi; ++y)
                            lc[y] = static_cast<uint8_t>(word >> (8 * (y - r)));
                    }
                }
                c += rq;
                jj += rr;
                if (jj >= nw) {
                    jj -= nw;
                    ++c;
                }
            }
            __syncwarp(); // the staging area is refilled for the next column
        }
        cp_async_wait_all(); // the next region's centres
        __syncthreads();     // shared planes and counters are reused by the next region
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
    const unsigned grid = ctx->park_ctas * K::kCtasPerSm;
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
        || cudaMemsetAsync(ctx->region_counts, 0, (kRegionLists + 1) * sizeof(uint32_t), st) != cudaSuccess
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
    b.centres = ctx->region_centres;
    b.win_lo = win_lo;
    b.win_hi = win_hi;
    b.tiles_x = static_cast<int32_t>(ctx->tiles_x);
    b.tiles_z = static_cast<int32_t>(ctx->tiles_z);
    b.flags = ctx->flags;
    region_build_kernel<<<(b.num_envs + kBuildWarps - 1) / kBuildWarps, 32 * kBuildWarps, 0, st>>>(b);
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
    for (int k = 0; k < kRegionLists; ++k)
        if (cudaStreamWaitEvent(ctx->relight_streams[k], ctx->relight_fork, 0) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "relight fork wait");
    const int rr = launch_region_relight(ctx, ctx->relight_streams);
    if (rr != BLK_OK)
        return rr;
    const int rt = launch_tiles(ctx, 1, static_cast<uint32_t>(n_tiles), st);
    for (int k = 0; k < kRegionLists; ++k)
        if (cudaEventRecord(ctx->relight_join[k], ctx->relight_streams[k]) != cudaSuccess
            || cudaStreamWaitEvent(st, ctx->relight_join[k], 0) != cudaSuccess)
            return cuda_fail(cudaGetLastError(), "relight join");
    return rt;
}

int launch_region_relight(blk_ctx* ctx, const cudaStream_t (&side)[kRegionLists])
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
    a.centres = ctx->region_centres;
    a.flags = ctx->flags;
    // Size classes (lists of region_build_kernel), each on its own stream so
    // that their tails overlap: list 2 s + nb - 1 holds regions of nb words
    // solved by CTAs of 512 x 1, 1024 x 1 and 1024 x 2 columns (threads x
    // columns per thread); the largest first.
    int rc = launch_region_list<1024, 2, 2>(ctx, a, 5, side[5]);
    if (rc == BLK_OK)
        rc = launch_region_list<1024, 2, 1>(ctx, a, 4, side[4]);
    if (rc == BLK_OK)
        rc = launch_region_list<1024, 1, 2>(ctx, a, 3, side[3]);
    if (rc == BLK_OK)
        rc = launch_region_list<1024, 1, 1>(ctx, a, 2, side[2]);
    if (rc == BLK_OK)
        rc = launch_region_list<512, 1, 2>(ctx, a, 1, side[1]);
    if (rc == BLK_OK)
        rc = launch_region_list<512, 1, 1>(ctx, a, 0, side[0]);
    return rc;
}

} // namespace blk
