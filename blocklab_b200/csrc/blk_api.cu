// C ABI of libblk_world.so and the small kernels around the tile kernel:
// override column-CSR build, torch placement, edit application with
// World::setBlock semantics + dirty-window marking, render voxel list,
// day/night effective light, RGBA8 -> float NCHW.
#include "blk_internal.h"

#include <cstdio>
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

namespace blk {


namespace {
thread_local std::string g_last_error;
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 8; // per thread: two 16-byte loads / stores
constexpr uint32_t kScanTile = kScanThreads * kScanItems;

inline cudaStream_t as_stream(uintptr_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------- scans --
__device__ inline uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_sums, uint32_t& total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o)
            x += y;
    }
    if (lane == 31)
        warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o)
                w += y;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    const uint32_t warp_prefix = warp > 0 ? warp_sums[warp - 1] : 0u;
    total = warp_sums[(blockDim.x >> 5) - 1];
    __syncthreads();
    return warp_prefix + x - v;
}

// A thread's kScanItems consecutive items from `base`: two 16-byte loads when
// the array is 16-byte aligned and the items are all in range, else one by one.
__device__ inline void scan_load(const uint32_t* in, uint64_t n, uint64_t base, uint32_t (&v)[kScanItems])
{
    if ((reinterpret_cast<uintptr_t>(in) & 15u) == 0u && base + kScanItems <= n) {
        const uint4 a = *reinterpret_cast<const uint4*>(in + base);
        const uint4 b = *reinterpret_cast<const uint4*>(in + base + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
            v[k] = base + k < n ? in[base + k] : 0u;
    }
}

__global__ void scan_reduce_kernel(const uint32_t* in, uint64_t n, uint32_t* partials)
{
    __shared__ uint32_t ws[32];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kScanTile + threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    scan_load(in, n, base, v);
    uint32_t sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
        sum += v[k];
    uint32_t total;
    block_exclusive_scan(sum, ws, total);
    if (threadIdx.x == 0)
        partials[blockIdx.x] = total;
}

__global__ void scan_partials_kernel(uint32_t* partials, uint64_t n)
{
    __shared__ uint32_t ws[32];
    uint32_t carry = 0;
    for (uint64_t base = 0; base < n; base += blockDim.x) {
        const uint64_t i = base + threadIdx.x;
        const uint32_t v = i < n ? partials[i] : 0u;
        uint32_t total;
        const uint32_t ex = block_exclusive_scan(v, ws, total);
        if (i < n)
            partials[i] = carry + ex;
        carry += total;
    }
}

__global__ void scan_final_kernel(const uint32_t* in, uint64_t n, const uint32_t* partials, uint32_t* out)
{
    __shared__ uint32_t ws[32];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kScanTile + threadIdx.x * kScanItems;
    uint32_t v[kScanItems];
    scan_load(in, n, base, v);
    uint32_t sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k)
        sum += v[k];
    uint32_t total;
    uint32_t run = partials[blockIdx.x] + block_exclusive_scan(sum, ws, total);
    uint32_t o[kScanItems];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        o[k] = run;
        run += v[k];
    }
    if ((reinterpret_cast<uintptr_t>(out) & 15u) == 0u && base + kScanItems <= n) {
        *reinterpret_cast<uint4*>(out + base) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(out + base + 4) = make_uint4(o[4], o[5], o[6], o[7]);
    } else {
#pragma unroll
        for (int k = 0; k < kScanItems; ++k)
            if (base + k < n)
                out[base + k] = o[k];
    }
}

// Exclusive scan of n uint32 (n <= scan capacity of the context).
int exclusive_scan(blk_ctx* ctx, const uint32_t* in, uint32_t* out, uint64_t n, cudaStream_t st)
{
    const uint64_t blocks = (n + kScanTile - 1) / kScanTile;
    if (blocks > ctx->scan_blocks) {
        set_error("internal: scan larger than its scratch");
        return BLK_ERR_CAPACITY;
    }
    scan_reduce_kernel<<<static_cast<unsigned>(blocks), kScanThreads, 0, st>>>(in, n, ctx->scan_partials);
    scan_partials_kernel<<<1, kScanThreads, 0, st>>>(ctx->scan_partials, blocks);
    scan_final_kernel<<<static_cast<unsigned>(blocks), kScanThreads, 0, st>>>(in, n, ctx->scan_partials, out);
    return cuda_fail(cudaGetLastError(), "scan launch");
}

// ------------------------------------------------------------ overrides --
struct RegionDims {
    const int4* origin;      // [env] world coordinates of each env's local (0, 0, 0)
    int32_t W, H, D;
    uint32_t num_envs;
    const uint8_t* env_mask; // override kernels: only envs set here (nullptr = all)
};

__device__ inline bool local_cell(const RegionDims& r, const blk_override& o, int32_t& x, int32_t& y, int32_t& z)
{
    if (o.env >= r.num_envs || (r.env_mask && !r.env_mask[o.env]) || o.block > Torch)
        return false;
    const int4 org = r.origin[o.env];
    x = o.x - org.x;
    y = o.y - org.y;
    z = o.z - org.z;
    return x >= 0 && y >= 0 && z >= 0 && x < r.W && y < r.H && z < r.D;
}

__global__ void ovr_count_kernel(const blk_override* ovr, uint32_t n, RegionDims r, uint32_t* col_count)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const blk_override o = ovr[i];
        int32_t x, y, z;
        if (!local_cell(r, o, x, y, z))
            continue;
        const uint64_t col = static_cast<uint64_t>(o.env) * r.W * r.D + static_cast<uint64_t>(z) * r.W + x;
        atomicAdd(col_count + col, 1u);
    }
}

// Scatters each override into its column segment, taking the segment's slots
// from its count down (the counts the scan read; left at zero). The override
// that takes slot 0 is recorded as the segment's owner (owner[i] = 1), so
// exactly one thread sorts each segment afterwards.
__global__ void ovr_scatter_kernel(const blk_override* ovr, uint32_t n, RegionDims r, const uint32_t* col_offset,
    uint32_t* count, uint64_t* entries, uint8_t* owner)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const blk_override o = ovr[i];
        int32_t x, y, z;
        if (!local_cell(r, o, x, y, z)) {
            owner[i] = 0;
            continue;
        }
        const uint64_t col = static_cast<uint64_t>(o.env) * r.W * r.D + static_cast<uint64_t>(z) * r.W + x;
        const uint32_t slot = atomicSub(count + col, 1u) - 1u;
        entries[col_offset[col] + slot] = (static_cast<uint64_t>(y) << 40) | (static_cast<uint64_t>(i) << 8) | o.block;
        owner[i] = slot == 0 ? 1 : 0;
    }
}

// Sorts each column segment by (y, input order); only the segment's owner
// touches it.
__global__ void ovr_sort_kernel(const blk_override* ovr, uint32_t n, RegionDims r, const uint32_t* col_offset,
    uint64_t* entries, const uint8_t* owner)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        if (!owner[i])
            continue;
        const blk_override o = ovr[i];
        int32_t x, y, z;
        local_cell(r, o, x, y, z);
        const uint64_t col = static_cast<uint64_t>(o.env) * r.W * r.D + static_cast<uint64_t>(z) * r.W + x;
        const uint32_t beg = col_offset[col], end = col_offset[col + 1];
        for (uint32_t k = beg + 1; k < end; ++k) {
            const uint64_t v = entries[k];
            uint32_t m = k;
            while (m > beg && entries[m - 1] > v) {
                entries[m] = entries[m - 1];
                --m;
            }
            entries[m] = v;
        }
    }
}

// --------------------------------------------------------------- torches --
__global__ void place_torches_kernel(const uint32_t* seeds, uint32_t num_envs, uint32_t per_env, RegionDims r,
    TerrainParams t, blk_override* out, uint32_t* out_count, uint32_t* flags)
{
    const uint64_t total = static_cast<uint64_t>(num_envs) * per_env;
    if (blockIdx.x == 0 && threadIdx.x == 0)
        *out_count = static_cast<uint32_t>(total);
    const uint32_t columns = static_cast<uint32_t>(r.W) * static_cast<uint32_t>(r.D);
    for (uint64_t g = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; g < total;
         g += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t env = static_cast<uint32_t>(g / per_env);
        const uint32_t i = static_cast<uint32_t>(g % per_env);
        blk_override o {};
        o.env = static_cast<uint16_t>(env);
        o.block = Torch;
        o.kind = 0;
        o.x = 0;
        o.y = INT32_MIN; // "not placed": outside every region
        o.z = 0;
        if (i < columns) {
            const uint32_t seed = seeds[env];
            const uint32_t key = hash_combine2(seed, 0x7f4a7c15u);
            uint32_t c;
            if (!permute(i, columns, key, c))
                atomicOr(flags, kFlagPermuteGuard);
            const int32_t x = static_cast<int32_t>(c % static_cast<uint32_t>(r.W));
            const int32_t z = static_cast<int32_t>(c / static_cast<uint32_t>(r.W));
            const int4 org = r.origin[env];
            const int32_t top = clamp_top(terrain_top_local(t, seed, org.x + x, org.z + z, org.y), r.H);
            if (top + 1 < r.H) {
                o.x = org.x + x;
                o.y = org.y + top + 1;
                o.z = org.z + z;
            }
        }
        out[g] = o;
    }
}

// ----------------------------------------------------------- conversion --
__global__ void rgba_to_nchw_vec_kernel(const uint4* __restrict__ in, float4* __restrict__ out, uint32_t quads_per_image,
    uint64_t total_quads)
{
    const float inv255 = 1.0f / 255.0f;
    for (uint64_t q = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; q < total_quads;
         q += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t img = q / quads_per_image;
        const uint64_t p = q - img * quads_per_image;
        const uint4 v = __ldcs(in + q);
        const uint32_t px[4] = { v.x, v.y, v.z, v.w };
        float4 c[3];
        float* cr = reinterpret_cast<float*>(&c[0]);
        float* cg = reinterpret_cast<float*>(&c[1]);
        float* cbl = reinterpret_cast<float*>(&c[2]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            cr[k] = __fmul_rn(static_cast<float>(px[k] & 0xFFu), inv255);
            cg[k] = __fmul_rn(static_cast<float>((px[k] >> 8) & 0xFFu), inv255);
            cbl[k] = __fmul_rn(static_cast<float>((px[k] >> 16) & 0xFFu), inv255);
        }
        float4* base = out + img * 3 * quads_per_image + p;
        base[0] = c[0];
        base[quads_per_image] = c[1];
        base[2 * static_cast<uint64_t>(quads_per_image)] = c[2];
    }
}

__global__ void rgba_to_nchw_scalar_kernel(const uchar4* in, float* out, uint32_t pixels_per_image, uint64_t total)
{
    const float inv255 = 1.0f / 255.0f;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t img = i / pixels_per_image;
        const uint64_t p = i - img * pixels_per_image;
        const uchar4 s = in[i];
        float* base = out + img * 3 * pixels_per_image + p;
        base[0] = __fmul_rn(static_cast<float>(s.x), inv255);
        base[pixels_per_image] = __fmul_rn(static_cast<float>(s.y), inv255);
        base[2 * static_cast<uint64_t>(pixels_per_image)] = __fmul_rn(static_cast<float>(s.z), inv255);
    }
}

// ---------------------------------------------------------------- edits --
__global__ void edit_count_kernel(const blk_override* e, uint32_t n, uint32_t num_envs, uint32_t* env_count)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (e[i].env < num_envs)
            atomicAdd(env_count + e[i].env, 1u);
}

__global__ void edit_scatter_kernel(const blk_override* e, uint32_t n, uint32_t num_envs, const uint32_t* env_offset,
    uint32_t* cursor, uint32_t* order)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        if (e[i].env < num_envs)
            order[env_offset[e[i].env] + atomicAdd(cursor + e[i].env, 1u)] = i;
}

struct EditArgs {
    const blk_override* edits;
    const uint32_t* env_offset;
    uint32_t* order;
    uint4* changes;    // 2 per edit: the cells it changed (x | z << 16, y | old << 16 | new << 24, rows ylo | yhi << 16, flags)
    uint8_t* ids;
    int16_t* hmap;
    RegionDims r;
    uint64_t env_stride;
};

constexpr int kEditWarps = 4; // envs per CTA of apply_edits_kernel (one warp each)

// One warp per env: put the env's edit indices back in input order (the
// scatter filed them in any order), then apply them with World::setBlock
// semantics (src/world/World.cpp:239-287). An edit changes its own column
// only (the cell, the torch it may knock off above it, the column's top), so
// edits of different columns run side by side, 32 at a time; an edit waits
// for the earlier edits of its column.
__global__ void __launch_bounds__(32 * kEditWarps) apply_edits_kernel(EditArgs a)
{
    constexpr unsigned kFull = 0xFFFFFFFFu;
    const int lane = threadIdx.x & 31;
    const unsigned lt = (1u << lane) - 1u;
    const uint32_t env = blockIdx.x * kEditWarps + (threadIdx.x >> 5);
    if (env >= a.r.num_envs)
        return; // the whole warp
    const uint32_t beg = a.env_offset[env], end = a.env_offset[env + 1];
    if (end - beg <= 32) {
        // Rank of each index among the env's (all distinct).
        const uint32_t v = beg + lane < end ? a.order[beg + lane] : 0xFFFFFFFFu;
        uint32_t rank = 0u;
        for (uint32_t j = 0; j < end - beg; ++j)
            rank += __shfl_sync(kFull, v, static_cast<int>(j)) < v ? 1u : 0u;
        __syncwarp();
        if (beg + lane < end)
            a.order[beg + rank] = v;
    } else if (lane == 0) {
        for (uint32_t k = beg + 1; k < end; ++k) { // insertion sort (the scatter keeps most of the order)
            const uint32_t v = a.order[k];
            uint32_t m = k;
            while (m > beg && a.order[m - 1] > v) {
                a.order[m] = a.order[m - 1];
                --m;
            }
            a.order[m] = v;
        }
    }
    __syncwarp();
    uint8_t* ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
    int16_t* hm = a.hmap + static_cast<uint64_t>(env) * a.r.W * a.r.D;
    const int32_t H = a.r.H;
    const int4 org = a.r.origin[env];
    for (uint32_t k0 = beg; k0 < end; k0 += 32) {
        const uint32_t k = k0 + lane;
        bool valid = false;
        blk_override e {};
        int32_t x = 0, y = 0, z = 0;
        uint8_t block = Air;
        uint64_t col = 0;
        if (k < end) {
            a.changes[2 * static_cast<uint64_t>(k)].w = 0u;
            a.changes[2 * static_cast<uint64_t>(k) + 1].w = 0u;
            e = a.edits[a.order[k]];
            x = e.x - org.x;
            y = e.y - org.y;
            z = e.z - org.z;
            block = e.kind == 1 ? Air : e.block;
            valid = !(x < 0 || z < 0 || y < 0 || x >= a.r.W || z >= a.r.D || y >= H || block > Torch);
            col = valid ? static_cast<uint64_t>(z) * a.r.W + x : 0;
        }
        // Lanes of one column go in lane order (= input order); distinct
        // keys for lanes without an edit.
        const uint64_t key = valid ? col : (0xFFFFFFFF00000000ull | static_cast<uint32_t>(lane));
        const unsigned same = __match_any_sync(kFull, key);
        unsigned pending = __ballot_sync(kFull, valid);
        while (pending) { // warp-uniform
            const bool ready = ((pending >> lane) & 1u) != 0u && (same & pending & lt) == 0u;
            if (ready && !(e.kind == 1 && ids[col * H + y] != Torch)) {
                // setBlock, with the torch-support rule unrolled (the torch
                // removal cannot cascade: Air is not solid).
                int32_t yc = y;
                uint8_t bc = block;
                for (int pass = 0; pass < 2; ++pass) {
                    uint8_t& cell = ids[col * H + yc];
                    const uint8_t old = cell;
                    if (old == bc)
                        break;
                    cell = bc;
                    const int32_t old_top = hm[col] - org.y;
                    int32_t top = old_top;
                    if (is_opaque(bc) && yc > top)
                        top = yc;
                    else if (!is_opaque(bc) && is_opaque(old) && yc == top) {
                        top = -1;
                        for (int32_t yy = yc - 1; yy >= 0; --yy)
                            if (is_opaque(ids[col * H + yy])) {
                                top = yy;
                                break;
                            }
                    }
                    hm[col] = static_cast<int16_t>(top + org.y);
                    int32_t ylo = yc, yhi = yc;
                    if (top != old_top) {
                        ylo = min(ylo, min(top, old_top) + 1);
                        yhi = max(yhi, max(top, old_top));
                    }
                    // Light depends on which cells are opaque and which are
                    // torches only (the height map follows the opaque cells):
                    // an opaque cell replaced by another opaque block changes no
                    // light anywhere. Other changes are recorded, with the
                    // column's top just before the change (w = 1 | (old_top + 2)
                    // << 8), and marked for relight by mark_changes_kernel once
                    // every env's last edit is in.
                    if (!(is_opaque(old) && is_opaque(bc)))
                        a.changes[2 * static_cast<uint64_t>(k) + pass] = make_uint4(
                            static_cast<uint32_t>(x) | (static_cast<uint32_t>(z) << 16),
                            static_cast<uint32_t>(yc) | (static_cast<uint32_t>(old) << 16) | (static_cast<uint32_t>(bc) << 24),
                            static_cast<uint32_t>(max(ylo, 0)) | (static_cast<uint32_t>(min(yhi, H - 1)) << 16),
                            1u | (static_cast<uint32_t>(old_top + 2) << 8));
                    if (!(is_opaque(old) && !is_opaque(bc) && yc + 1 < H && ids[col * H + yc + 1] == Torch))
                        break;
                    yc = yc + 1;
                    bc = Air;
                }
            }
            __syncwarp(); // this round's column writes are seen by the next round
            pending &= ~__ballot_sync(kFull, ready);
        }
    }
}

// Marks the changes apply_edits_kernel recorded, except an air <-> opaque
// change of a cell that lay below its column's top when it changed and ends
// the step enclosed: below its column's final top and with all six neighbours
// opaque (or outside the region) once every edit of its env is in, no torch
// before or after. Every change that moves a column's top is then marked with
// the span it moved, so a skipped cell was no sky source before the step
// unless a marked span covers it. A light path of the old world into a skipped
// cell enters it from a neighbour that is opaque at the end of the step, i.e.
// from a changed cell: marked (its window covers the path's end) or skipped
// (then the path came through an earlier skipped cell, back to a source, which
// no skipped cell is). So outside the marked windows no light path and no
// source differs between the two worlds, and their light agrees there. One
// thread per record (two per edit position of the env-grouped list).
__global__ void mark_changes_kernel(EditArgs a)
{
    const uint64_t n_rec = 2ull * a.env_offset[a.r.num_envs]; // edits grouped to an env
    const int32_t H = a.r.H;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n_rec;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint4 c = a.changes[i];
        if (!c.w)
            continue;
        const uint32_t env = a.edits[a.order[i / 2]].env;
        const uint8_t* ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
        const int16_t* hm = a.hmap + static_cast<uint64_t>(env) * a.r.W * a.r.D;
        auto opaque_at = [&](int32_t x, int32_t y, int32_t z) {
            if (x < 0 || z < 0 || y < 0 || x >= a.r.W || z >= a.r.D || y >= H)
                return true;
            return is_opaque(ids[(static_cast<uint64_t>(z) * a.r.W + x) * H + y]);
        };
        const int32_t x = static_cast<int32_t>(c.x & 0xFFFFu), z = static_cast<int32_t>(c.x >> 16);
        const int32_t y = static_cast<int32_t>(c.y & 0xFFFFu);
        const uint8_t old = static_cast<uint8_t>((c.y >> 16) & 0xFFu), now = static_cast<uint8_t>(c.y >> 24);
        const int32_t top = hm[static_cast<uint64_t>(z) * a.r.W + x] - a.r.origin[env].y;
        const int32_t top_then = static_cast<int32_t>(c.w >> 8) - 2; // the column's top just before the change
        const bool enclosed = old != Torch && now != Torch && y < top && y < top_then && opaque_at(x - 1, y, z)
            && opaque_at(x + 1, y, z) && opaque_at(x, y - 1, z) && opaque_at(x, y + 1, z) && opaque_at(x, y, z - 1)
            && opaque_at(x, y, z + 1);
        if (!enclosed)
            a.changes[i].w = c.w | 2u; // marked: its dirty cube joins the env's relight regions
    }
}

// --------------------------------------------------------- render voxels --
struct VoxelArgs {
    const uint8_t* ids;
    const uint8_t* light;
    int32_t W, H, D;
    uint32_t* row_count;  // [D*H]
};

__device__ inline bool voxel_at(const VoxelArgs& a, int x, int y, int z, uint32_t out[3])
{
    const uint64_t idx = (static_cast<uint64_t>(z) * a.W + x) * a.H + y;
    const uint8_t b = a.ids[idx];
    if (b == Air)
        return false;
    // left, right, top, bottom, front, back (src/world/Voxel.h:10-17)
    const int nx[6] = { x - 1, x + 1, x, x, x, x };
    const int ny[6] = { y, y, y + 1, y - 1, y, y };
    const int nz[6] = { z, z, z, z, z + 1, z - 1 };
    uint8_t nb[6], nl[6];
#pragma unroll
    for (int f = 0; f < 6; ++f) {
        if (nx[f] < 0 || ny[f] < 0 || nz[f] < 0 || nx[f] >= a.W || ny[f] >= a.H || nz[f] >= a.D) {
            nb[f] = Air;
            nl[f] = 0;
        } else {
            const uint64_t j = (static_cast<uint64_t>(nz[f]) * a.W + nx[f]) * a.H + ny[f];
            nb[f] = a.ids[j];
            nl[f] = a.light[j];
        }
    }
    uint32_t faces = 0, bl = 0, sl = 0;
    if (b == Torch) {
        faces = 0x1 | 0x2 | 0x4 | 0x10 | 0x20;
        bl = 0xFFFFFFu;
    } else {
        bool all = true;
#pragma unroll
        for (int f = 0; f < 6; ++f)
            all = all && is_opaque(nb[f]);
        if (all)
            return false;
#pragma unroll
        for (int f = 0; f < 6; ++f) {
            faces |= is_opaque(nb[f]) ? 0u : (1u << f);
            bl |= static_cast<uint32_t>(nl[f] & 0xF) << (4 * f);
        }
    }
#pragma unroll
    for (int f = 0; f < 6; ++f)
        sl |= static_cast<uint32_t>(nl[f] >> 4) << (4 * f);
    out[0] = static_cast<uint32_t>(b) | (faces << 5) | (static_cast<uint32_t>(z) << 11) | (static_cast<uint32_t>(y) << 17)
        | (static_cast<uint32_t>(x) << 26);
    out[1] = bl;
    out[2] = sl;
    return true;
}

__global__ void voxel_count_kernel(VoxelArgs a)
{
    const int row = blockIdx.x * blockDim.x + threadIdx.x; // row = z*H + y
    if (row >= a.D * a.H)
        return;
    const int z = row / a.H, y = row % a.H;
    uint32_t n = 0, tmp[3];
    for (int x = 0; x < a.W; ++x)
        n += voxel_at(a, x, y, z, tmp) ? 1u : 0u;
    a.row_count[row] = n;
}

// The header's origin comes from `origin_dev` (device, one record) when it
// is given, else from `origin`.
__global__ void voxel_write_kernel(VoxelArgs a, const uint32_t* row_offset, uint32_t* voxels, uint32_t max_voxels,
    uint32_t* count, int32_t* header, const int4* origin_dev, int3 origin)
{
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    const int rows = a.D * a.H;
    if (row == 0) {
        if (origin_dev)
            origin = make_int3(origin_dev->x, origin_dev->y, origin_dev->z);
        header[0] = origin.x;
        header[1] = origin.y;
        header[2] = origin.z;
    }
    if (row >= rows)
        return;
    if (row == rows - 1)
        *count = row_offset[row] + a.row_count[row];
    const int z = row / a.H, y = row % a.H;
    uint32_t pos = row_offset[row], v[3];
    for (int x = 0; x < a.W; ++x)
        if (voxel_at(a, x, y, z, v)) {
            if (pos < max_voxels) {
                voxels[3 * static_cast<uint64_t>(pos)] = v[0];
                voxels[3 * static_cast<uint64_t>(pos) + 1] = v[1];
                voxels[3 * static_cast<uint64_t>(pos) + 2] = v[2];
            }
            ++pos;
        }
}

// Render voxels without allocation: the per-row counts and offsets live in a
// fixed device array. depth * height rows at most; the reference's packing
// (z < 64, y < 512) never needs more.
constexpr uint32_t kStaticVoxelRows = 64u * 512u;
static __device__ __align__(256) uint32_t g_voxel_rows[2 * kStaticVoxelRows]; // counts | offsets

// Exclusive scan of n <= 32768 row counts by one block of 1024 threads, each
// owning a run of consecutive rows.
__global__ void __launch_bounds__(1024) row_scan_one_block(const uint32_t* in, uint32_t* out, uint32_t n)
{
    __shared__ uint32_t warp_sums[32];
    const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
    const uint32_t per = (n + 1023u) / 1024u;
    const uint32_t b = t * per;
    uint32_t sum = 0;
    for (uint32_t i = 0; i < per; ++i)
        if (b + i < n)
            sum += in[b + i];
    uint32_t v = sum; // inclusive scan over the warp
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t u = __shfl_up_sync(0xFFFFFFFFu, v, d);
        if (lane >= static_cast<uint32_t>(d))
            v += u;
    }
    if (lane == 31u)
        warp_sums[warp] = v;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = warp_sums[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t u = __shfl_up_sync(0xFFFFFFFFu, w, d);
            if (lane >= static_cast<uint32_t>(d))
                w += u;
        }
        warp_sums[lane] = w;
    }
    __syncthreads();
    uint32_t run = v - sum + (warp ? warp_sums[warp - 1] : 0u);
    for (uint32_t i = 0; i < per; ++i)
        if (b + i < n) {
            out[b + i] = run;
            run += in[b + i];
        }
}

// ---------------------------------------------------------- region origins --
// origins[i] = (xyz[3i], xyz[3i + 1], xyz[3i + 2]) for the n envs.
__global__ void set_origins_kernel(const int32_t* xyz, uint32_t n, int4* origins)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        origins[i] = make_int4(xyz[3 * static_cast<uint64_t>(i)], xyz[3 * static_cast<uint64_t>(i) + 1],
            xyz[3 * static_cast<uint64_t>(i) + 2], 0);
}

// ---------------------------------------------------------- partial reset --
// Marks the listed envs, installs their seeds (and origins, when given) and
// lists their tiles (0xFFFFFFFF for an out-of-range env id, which also raises
// a flag).
__global__ void env_select_kernel(const uint32_t* env_ids, const uint32_t* seeds, const int32_t* origin_xyz,
    uint32_t n, uint32_t num_envs, uint32_t tiles_per_env, uint8_t* mask, uint32_t* env_seeds, int4* origins,
    uint32_t* tile_list, uint32_t* flags)
{
    const uint64_t total = static_cast<uint64_t>(n) * tiles_per_env;
    for (uint64_t k = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; k < total;
         k += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t i = static_cast<uint32_t>(k / tiles_per_env), t = static_cast<uint32_t>(k % tiles_per_env);
        const uint32_t e = env_ids[i];
        if (e >= num_envs) {
            tile_list[k] = 0xFFFFFFFFu;
            if (t == 0)
                atomicOr(flags, kFlagEnvIndex);
            continue;
        }
        tile_list[k] = e * tiles_per_env + t;
        if (t == 0) {
            mask[e] = 1;
            env_seeds[e] = seeds[i];
            if (origin_xyz)
                origins[e] = make_int4(origin_xyz[3 * static_cast<uint64_t>(i)],
                    origin_xyz[3 * static_cast<uint64_t>(i) + 1], origin_xyz[3 * static_cast<uint64_t>(i) + 2], 0);
        }
    }
}

// ---------------------------------------------------------- sparse queries --
__global__ void query_cells_kernel(const blk_cell_query* q, uint32_t n, const uint8_t* ids, const uint8_t* light,
    const int16_t* hmap, RegionDims r, uint64_t env_stride, uint8_t* out_block, uint8_t* out_light,
    int32_t* out_height)
{
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const blk_cell_query c = q[i];
        const int4 org = c.env < r.num_envs ? r.origin[c.env] : make_int4(0, 0, 0, 0);
        const int32_t x = c.x - org.x, y = c.y - org.y, z = c.z - org.z;
        const bool column = c.env < r.num_envs && x >= 0 && x < r.W && z >= 0 && z < r.D;
        const bool inside = column && y >= 0 && y < r.H;
        const uint64_t col = static_cast<uint64_t>(z) * r.W + x;
        uint8_t b = 255, l = 0;
        if (inside) {
            const uint64_t idx = static_cast<uint64_t>(c.env) * env_stride + col * r.H + y;
            b = ids[idx];
            l = light[idx];
        }
        if (out_block)
            out_block[i] = b;
        if (out_light)
            out_light[i] = l;
        if (out_height)
            out_height[i] = column ? static_cast<int32_t>(hmap[static_cast<uint64_t>(c.env) * r.W * r.D + col])
                                   : INT32_MIN;
    }
}

// One warp per box; the warp stops at the first solid cell it meets.
__global__ void query_solid_kernel(const blk_box_query* q, uint32_t n, const uint8_t* ids, RegionDims r,
    uint64_t env_stride, uint8_t* out)
{
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    for (uint32_t i = (blockIdx.x * blockDim.x + threadIdx.x) / 32; i < n; i += warps) {
        const blk_box_query b = q[i];
        const int4 org = b.env < r.num_envs ? r.origin[b.env] : make_int4(0, 0, 0, 0);
        const int32_t x0 = max(b.min_x - org.x, 0), x1 = min(b.max_x - org.x, r.W - 1);
        const int32_t y0 = max(b.min_y - org.y, 0), y1 = min(b.max_y - org.y, r.H - 1);
        const int32_t z0 = max(b.min_z - org.z, 0), z1 = min(b.max_z - org.z, r.D - 1);
        bool found = false;
        if (b.env < r.num_envs && x0 <= x1 && y0 <= y1 && z0 <= z1) {
            const uint64_t ny = y1 - y0 + 1, nx = x1 - x0 + 1;
            const uint64_t total = ny * nx * static_cast<uint64_t>(z1 - z0 + 1);
            const uint8_t* env_ids = ids + static_cast<uint64_t>(b.env) * env_stride;
            for (uint64_t base = 0; base < total; base += 32) {
                const uint64_t k = base + lane;
                bool solid = false;
                if (k < total) {
                    const int32_t y = y0 + static_cast<int32_t>(k % ny);
                    const int32_t x = x0 + static_cast<int32_t>((k / ny) % nx);
                    const int32_t z = z0 + static_cast<int32_t>(k / (ny * nx));
                    solid = is_opaque(env_ids[(static_cast<uint64_t>(z) * r.W + x) * r.H + y]);
                }
                if (__any_sync(0xFFFFFFFFu, solid)) {
                    found = true;
                    break;
                }
            }
        }
        if (lane == 0)
            out[i] = found ? 1 : 0;
    }
}

// ------------------------------------------------------------- snapshots --
// Cells of one env whose block differs from its terrain (layer rule of the
// column's surface): count per column, then write in (z, x, y) order.
__global__ void snapshot_count_kernel(const uint8_t* ids, const int16_t* terrain_top, RegionDims r, uint32_t* count)
{
    const uint64_t columns = static_cast<uint64_t>(r.W) * r.D;
    for (uint64_t col = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; col < columns;
         col += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const int32_t top = terrain_top[col];
        uint32_t n = 0;
        for (int32_t y = 0; y < r.H; ++y)
            n += ids[col * r.H + y] != layer_block(y, top) ? 1u : 0u;
        count[col] = n;
    }
}

__global__ void snapshot_write_kernel(const uint8_t* ids, const int16_t* terrain_top, RegionDims r, uint32_t env,
    const uint32_t* count, const uint32_t* offset, blk_override* out, uint32_t capacity, uint32_t* total)
{
    const uint64_t columns = static_cast<uint64_t>(r.W) * r.D;
    for (uint64_t col = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; col < columns;
         col += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        if (col == columns - 1)
            *total = offset[col] + count[col];
        uint32_t pos = offset[col];
        if (count[col] == 0 || pos >= capacity)
            continue;
        const int32_t top = terrain_top[col];
        const int32_t x = static_cast<int32_t>(col % r.W), z = static_cast<int32_t>(col / r.W);
        const int4 org = r.origin[env];
        for (int32_t y = 0; y < r.H && pos < capacity; ++y) {
            const uint8_t b = ids[col * r.H + y];
            if (b == layer_block(y, top))
                continue;
            blk_override o;
            o.x = x + org.x;
            o.y = y + org.y;
            o.z = z + org.z;
            o.env = static_cast<uint16_t>(env);
            o.block = b;
            o.kind = 0;
            out[pos++] = o;
        }
    }
}

// ------------------------------------------------------- effective light --
__global__ void effective_light_kernel(const uint4* light, uint4* out, const uint8_t* dimming, uint64_t quads_per_env,
    uint64_t total)
{
    for (uint64_t q = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; q < total;
         q += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t d = dimming[q / quads_per_env] * 0x01010101u;
        const uint4 v = light[q];
        uint32_t w[4] = { v.x, v.y, v.z, v.w };
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t sky = (w[k] >> 4) & 0x0F0F0F0Fu;
            w[k] = (__vsubus4(sky, d) << 4) | (w[k] & 0x0F0F0F0Fu);
        }
        out[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

int grid_for(uint64_t work, int threads)
{
    uint64_t blocks = (work + threads - 1) / threads;
    if (blocks > 148ull * 16)
        blocks = 148ull * 16;
    return static_cast<int>(blocks < 1 ? 1 : blocks);
}

RegionDims region(const blk_ctx* ctx)
{
    RegionDims r;
    r.origin = ctx->origins;
    r.W = static_cast<int32_t>(ctx->cfg.width);
    r.H = static_cast<int32_t>(ctx->cfg.height);
    r.D = static_cast<int32_t>(ctx->cfg.depth);
    r.num_envs = ctx->cfg.num_envs;
    r.env_mask = nullptr;
    return r;
}

template <typename T>
int dalloc(T** p, size_t count, const char* what)
{
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16);
    if (e != cudaSuccess) {
        *p = nullptr;
        cudaGetLastError();
        set_error(std::string("cudaMalloc ") + what + ": " + cudaGetErrorString(e));
        return e == cudaErrorMemoryAllocation ? BLK_ERR_OUT_OF_MEMORY : BLK_ERR_CUDA;
    }
    return BLK_OK;
}

} // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int cuda_fail(cudaError_t e, const char* what)
{
    if (e == cudaSuccess)
        return BLK_OK;
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return BLK_ERR_CUDA;
}

bool device_memory(const void* p)
{
    cudaPointerAttributes attr {};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

int stage_input(const void* src, size_t bytes, void* staging, cudaStream_t stream, const void** out)
{
    if (bytes == 0) {
        *out = src;
        return BLK_OK;
    }
    cudaPointerAttributes attr {};
    cudaError_t e = cudaPointerGetAttributes(&attr, src);
    if (e != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        *out = src;
        return BLK_OK;
    }
    e = cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaMemcpyAsync (input staging)");
    *out = staging;
    return BLK_OK;
}

TerrainParams terrain_params(const blk_ctx* ctx)
{
    TerrainParams t;
    t.mode = ctx->cfg.terrain_mode;
    t.base = ctx->cfg.fbm_base;
    t.amplitude = ctx->cfg.fbm_amplitude;
    t.height = static_cast<int32_t>(ctx->cfg.height);
    return t;
}

} // namespace blk

using namespace blk;

#define BLK_CHECK(expr)                                                                                                \
    do {                                                                                                               \
        const int rc_ = (expr);                                                                                        \
        if (rc_ != BLK_OK)                                                                                             \
            return rc_;                                                                                                \
    } while (0)

#define BLK_CUDA(expr, what) BLK_CHECK(cuda_fail((expr), what))

extern "C" {

const char* blk_last_error(void) { return g_last_error.c_str(); }

int blk_ctx_create(int device, const blk_world_config* config, blk_ctx** out)
{
    if (!config || !out) {
        set_error("blk_ctx_create: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    const blk_world_config& c = *config;
    if (c.num_envs == 0 || c.num_envs > 65536 || c.max_overrides > (1u << 26) || c.width == 0 || c.depth == 0 || c.width > 4096 || c.depth > 4096
        || c.height == 0 || c.height % 32 != 0 || c.height > 256 || c.terrain_mode < 0 || c.terrain_mode > 2) {
        set_error("blk_ctx_create: unsupported configuration (num_envs 1..65536, W/D 1..4096, H a multiple of 32 up "
                  "to 256, terrain_mode 0..2)");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    BLK_CUDA(cudaSetDevice(device), "cudaSetDevice");
    auto* ctx = new blk_ctx();
    ctx->device = device;
    ctx->cfg = c;
    if (ctx->cfg.max_overrides == 0)
        ctx->cfg.max_overrides = 1;
    if (ctx->cfg.max_edits == 0)
        ctx->cfg.max_edits = 1;
    ctx->tiles_x = (c.width + 31) / 32;
    ctx->tiles_z = (c.depth + 31) / 32;
    ctx->columns_per_env = static_cast<uint64_t>(c.width) * c.depth;
    ctx->env_stride = ctx->columns_per_env * c.height;
    const uint64_t envs = c.num_envs;
    const uint64_t n_cols = envs * ctx->columns_per_env + 1;
    const uint64_t n_tiles = envs * ctx->tiles_x * ctx->tiles_z;
    const uint64_t scan_n = (n_cols > n_tiles ? n_cols : n_tiles) + envs + 1;
    ctx->scan_blocks = (scan_n + kScanTile - 1) / kScanTile;
    int rc = BLK_OK;
    auto A = [&](int r) {
        if (rc == BLK_OK)
            rc = r;
    };
    A(dalloc(&ctx->ids, envs * ctx->env_stride, "ids"));
    A(dalloc(&ctx->light, envs * ctx->env_stride, "light"));
    A(dalloc(&ctx->hmap, envs * ctx->columns_per_env, "height map"));
    A(dalloc(&ctx->seeds, envs, "seeds"));
    A(dalloc(&ctx->origins, envs, "region origins"));
    A(dalloc(&ctx->origin_stage, 3 * envs, "region origin staging"));
    A(dalloc(&ctx->terrain_top, envs * ctx->columns_per_env, "terrain heights"));
    A(dalloc(&ctx->halo_order, static_cast<size_t>(halo_order_size()), "halo order"));
    A(dalloc(&ctx->ovr, ctx->cfg.max_overrides, "override staging"));
    A(dalloc(&ctx->col_count, n_cols, "column counts"));
    A(dalloc(&ctx->col_offset, n_cols, "column offsets"));
    A(dalloc(&ctx->entries, ctx->cfg.max_overrides, "override entries"));
    A(dalloc(&ctx->ovr_owner, ctx->cfg.max_overrides, "override segment owners"));
    A(dalloc(&ctx->scan_partials, ctx->scan_blocks, "scan partials"));
    A(dalloc(&ctx->edits, ctx->cfg.max_edits, "edit staging"));
    A(dalloc(&ctx->edit_env_count, envs + 1, "edit counts"));
    A(dalloc(&ctx->edit_env_offset, envs + 1, "edit offsets"));
    A(dalloc(&ctx->edit_order, ctx->cfg.max_edits, "edit order"));
    A(dalloc(&ctx->edit_changes, 2ull * ctx->cfg.max_edits, "edit changes"));
    A(dalloc(&ctx->dirty_window, 2 * n_tiles, "dirty windows"));
    A(dalloc(&ctx->dirty_list, n_tiles, "dirty list"));
    A(dalloc(&ctx->dirty_count, 1, "dirty count"));
    A(dalloc(&ctx->fallback_list, n_tiles, "generation fallback tiles"));
    A(dalloc(&ctx->fallback_count, 2, "generation fallback count and tile cursor"));
    ctx->box_capacity = 2 * std::max<uint32_t>(c.max_edits, 1);
    ctx->region_capacity = ctx->box_capacity; // every item holds a marked change
    A(dalloc(&ctx->region_lists, 2ull * kRegionLists * ctx->region_capacity, "relight region lists"));
    A(dalloc(&ctx->region_centres, ctx->region_capacity, "relight region centres"));
    A(dalloc(&ctx->region_counts, kRegionLists + 1, "relight region counts"));
    A(dalloc(&ctx->render_params, envs, "render parameters"));
    A(dalloc(&ctx->col_summary, envs * ctx->columns_per_env, "column summaries"));
    A(dalloc(&ctx->env_mask, envs, "partial reset env mask"));
    A(dalloc(&ctx->env_list, envs, "partial reset env ids"));
    A(dalloc(&ctx->seed_list, envs, "partial reset seeds"));
    A(dalloc(&ctx->flags, 1, "flags"));
    {
        int sms = 148;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) {
            cudaGetLastError();
            sms = 148;
        }
        ctx->park_ctas = static_cast<uint32_t>(sms);
        A(dalloc(&ctx->park, static_cast<size_t>(sms) * 16 * 1024, "tile scratch"));
    }
    if (rc == BLK_OK) {
        bool ok = cudaEventCreateWithFlags(&ctx->relight_fork, cudaEventDisableTiming) == cudaSuccess;
        for (int k = 0; k < kRegionLists && ok; ++k)
            ok = cudaStreamCreateWithFlags(&ctx->relight_streams[k], cudaStreamNonBlocking) == cudaSuccess
                && cudaEventCreateWithFlags(&ctx->relight_join[k], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) {
            rc = cuda_fail(cudaGetLastError(), "relight streams");
            if (rc == BLK_OK)
                rc = BLK_ERR_CUDA;
        }
    }
    if (rc == BLK_OK) {
        if (cudaMallocHost(reinterpret_cast<void**>(&ctx->h_flags), sizeof(uint32_t)) != cudaSuccess
            || cudaMallocHost(reinterpret_cast<void**>(&ctx->h_dirty_count), sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            set_error("cudaMallocHost failed");
            rc = BLK_ERR_OUT_OF_MEMORY;
        }
    }
    if (rc == BLK_OK) {
        std::vector<uint16_t> order(static_cast<size_t>(halo_order_size()));
        halo_order_table(order.data());
        rc = cuda_fail(cudaMemcpy(ctx->halo_order, order.data(), order.size() * sizeof(uint16_t),
                           cudaMemcpyHostToDevice),
            "halo order upload");
    }
    if (rc == BLK_OK) {
        // Every env starts at the configuration's origin.
        const std::vector<int4> org(envs, make_int4(c.origin_x, c.origin_y, c.origin_z, 0));
        rc = cuda_fail(cudaMemcpy(ctx->origins, org.data(), envs * sizeof(int4), cudaMemcpyHostToDevice),
            "origin upload");
    }
    if (rc == BLK_OK)
        rc = cuda_fail(cudaMemset(ctx->flags, 0, sizeof(uint32_t)), "cudaMemset flags");
    if (rc == BLK_OK) {
        rc = cuda_fail(cudaMemset(ctx->col_count, 0, (n_cols) * sizeof(uint32_t)), "cudaMemset column counts");
        ctx->counts_zero = rc == BLK_OK;
    }
    if (rc == BLK_OK)
        rc = cuda_fail(cudaMemset(ctx->hmap, 0, envs * ctx->columns_per_env * sizeof(int16_t)), "cudaMemset hmap");
    if (rc == BLK_OK)
        rc = launch_tiles(ctx, 0, 0, 0); // sets the kernels' shared-memory attributes
    if (rc == BLK_OK)
        rc = launch_generation(ctx, 0, 0);
    if (rc == BLK_OK)
        rc = cuda_fail(cudaDeviceSynchronize(), "context setup");
    if (rc != BLK_OK) {
        blk_ctx_destroy(ctx);
        return rc;
    }
    *out = ctx;
    return BLK_OK;
}

int blk_ctx_destroy(blk_ctx* ctx)
{
    if (!ctx)
        return BLK_OK;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    for (auto& m : ctx->marks)
        for (cudaEvent_t ev : m.e)
            cudaEventDestroy(ev);
    for (int k = 0; k < kRegionLists; ++k) {
        if (ctx->relight_streams[k])
            cudaStreamDestroy(ctx->relight_streams[k]);
        if (ctx->relight_join[k])
            cudaEventDestroy(ctx->relight_join[k]);
    }
    if (ctx->relight_fork)
        cudaEventDestroy(ctx->relight_fork);
    void* bufs[] = { ctx->ids, ctx->light, ctx->hmap, ctx->seeds, ctx->origins, ctx->origin_stage, ctx->terrain_top, ctx->halo_order, ctx->ovr, ctx->col_count, ctx->col_offset,
        ctx->entries, ctx->ovr_owner, ctx->scan_partials, ctx->edits, ctx->edit_env_count, ctx->edit_env_offset, ctx->edit_order, ctx->edit_changes,
        ctx->dirty_window, ctx->dirty_list, ctx->dirty_count, ctx->fallback_list, ctx->fallback_count, ctx->region_lists, ctx->region_centres, ctx->region_counts, ctx->render_params, ctx->col_summary, ctx->env_mask, ctx->env_list, ctx->seed_list, ctx->flags, ctx->park };
    for (void* b : bufs)
        if (b)
            cudaFree(b);
    if (ctx->h_flags)
        cudaFreeHost(ctx->h_flags);
    if (ctx->h_dirty_count)
        cudaFreeHost(ctx->h_dirty_count);
    delete ctx;
    cudaGetLastError();
    return BLK_OK;
}

int blk_views(blk_ctx* ctx, blk_world_views* out)
{
    if (!ctx || !out) {
        set_error("blk_views: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    out->ids = ctx->ids;
    out->light = ctx->light;
    out->height_map = ctx->hmap;
    out->env_origins = reinterpret_cast<const int32_t*>(ctx->origins);
    out->env_stride = ctx->env_stride;
    out->num_envs = ctx->cfg.num_envs;
    out->width = ctx->cfg.width;
    out->height = ctx->cfg.height;
    out->depth = ctx->cfg.depth;
    return BLK_OK;
}

int blk_generate(blk_ctx* ctx, const uint32_t* env_seeds, const int32_t* env_origins, const blk_override* overrides,
    uint32_t n_overrides, uintptr_t stream_handle)
{
    if (!ctx || !env_seeds || (n_overrides && !overrides)) {
        set_error("blk_generate: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (n_overrides > ctx->cfg.max_overrides) {
        set_error("blk_generate: " + std::to_string(n_overrides) + " overrides exceed max_overrides "
            + std::to_string(ctx->cfg.max_overrides));
        return BLK_ERR_CAPACITY;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t envs = ctx->cfg.num_envs;
    const void* seeds_dev = nullptr;
    BLK_CHECK(stage_input(env_seeds, envs * sizeof(uint32_t), ctx->seeds, st, &seeds_dev));
    if (seeds_dev != ctx->seeds)
        BLK_CUDA(cudaMemcpyAsync(ctx->seeds, seeds_dev, envs * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st),
            "seed copy");
    if (env_origins) {
        const void* org_dev = nullptr;
        BLK_CHECK(stage_input(env_origins, envs * 3 * sizeof(int32_t), ctx->origin_stage, st, &org_dev));
        set_origins_kernel<<<grid_for(envs, 256), 256, 0, st>>>(static_cast<const int32_t*>(org_dev),
            static_cast<uint32_t>(envs), ctx->origins);
        BLK_CUDA(cudaGetLastError(), "origin install launch");
    }
    const void* ovr_dev = nullptr;
    BLK_CHECK(stage_input(overrides, static_cast<size_t>(n_overrides) * sizeof(blk_override), ctx->ovr, st, &ovr_dev));
    const auto* ovr = static_cast<const blk_override*>(ovr_dev);
    const uint64_t n_cols = envs * ctx->columns_per_env;
    const RegionDims r = region(ctx);
    const int mark = prof_begin(ctx, 0, st);
    // The counts start at zero: left so by the previous generation's scatter
    // unless another call used them as scratch since.
    if (!ctx->counts_zero)
        BLK_CUDA(cudaMemsetAsync(ctx->col_count, 0, (n_cols + 1) * sizeof(uint32_t), st), "memset column counts");
    ctx->counts_zero = false;
    if (n_overrides)
        ovr_count_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_count);
    BLK_CHECK(exclusive_scan(ctx, ctx->col_count, ctx->col_offset, n_cols + 1, st));
    if (n_overrides) {
        ovr_scatter_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_offset,
            ctx->col_count, ctx->entries, ctx->ovr_owner);
        ovr_sort_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_offset, ctx->entries,
            ctx->ovr_owner);
        BLK_CUDA(cudaGetLastError(), "override kernels");
    }
    ctx->counts_zero = true; // the scatter counted every column back down
    const uint64_t n_tiles = envs * ctx->tiles_x * ctx->tiles_z;
    BLK_CHECK(launch_surface(ctx, st));
    prof_mark(ctx, mark, 1, st);
    BLK_CHECK(launch_generation(ctx, static_cast<uint32_t>(n_tiles), st));
    prof_mark(ctx, mark, 2, st);
    ctx->generated = true;
    return BLK_OK;
}

int blk_generate_envs(blk_ctx* ctx, const uint32_t* env_ids, uint32_t n_envs, const uint32_t* env_seeds,
    const int32_t* env_origins, const blk_override* overrides, uint32_t n_overrides, uintptr_t stream_handle)
{
    if (!ctx || (n_envs && (!env_ids || !env_seeds)) || (n_overrides && !overrides)) {
        set_error("blk_generate_envs: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_generate_envs: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    if (n_envs > ctx->cfg.num_envs || n_overrides > ctx->cfg.max_overrides) {
        set_error("blk_generate_envs: more envs or overrides than the context holds");
        return BLK_ERR_CAPACITY;
    }
    if (n_envs == 0)
        return BLK_OK;
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t envs = ctx->cfg.num_envs;
    const void *ids_dev = nullptr, *seeds_dev = nullptr, *ovr_dev = nullptr, *org_dev = nullptr;
    BLK_CHECK(stage_input(env_ids, n_envs * sizeof(uint32_t), ctx->env_list, st, &ids_dev));
    BLK_CHECK(stage_input(env_seeds, n_envs * sizeof(uint32_t), ctx->seed_list, st, &seeds_dev));
    if (env_origins)
        BLK_CHECK(stage_input(env_origins, n_envs * 3 * sizeof(int32_t), ctx->origin_stage, st, &org_dev));
    BLK_CHECK(stage_input(overrides, static_cast<size_t>(n_overrides) * sizeof(blk_override), ctx->ovr, st, &ovr_dev));
    const auto* ovr = static_cast<const blk_override*>(ovr_dev);
    const uint32_t tiles_per_env = ctx->tiles_x * ctx->tiles_z;
    const uint64_t n_items = static_cast<uint64_t>(n_envs) * tiles_per_env;
    BLK_CUDA(cudaMemsetAsync(ctx->env_mask, 0, envs, st), "memset env mask");
    env_select_kernel<<<grid_for(n_items, 256), 256, 0, st>>>(static_cast<const uint32_t*>(ids_dev),
        static_cast<const uint32_t*>(seeds_dev), static_cast<const int32_t*>(org_dev), n_envs, ctx->cfg.num_envs,
        tiles_per_env, ctx->env_mask, ctx->seeds, ctx->origins, ctx->dirty_list, ctx->flags);
    BLK_CUDA(cudaGetLastError(), "env select launch");
    RegionDims r = region(ctx);
    r.env_mask = ctx->env_mask;
    const uint64_t n_cols = envs * ctx->columns_per_env;
    const int mark = prof_begin(ctx, 0, st);
    // The counts start at zero: left so by the previous generation's scatter
    // unless another call used them as scratch since.
    if (!ctx->counts_zero)
        BLK_CUDA(cudaMemsetAsync(ctx->col_count, 0, (n_cols + 1) * sizeof(uint32_t), st), "memset column counts");
    ctx->counts_zero = false;
    if (n_overrides)
        ovr_count_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_count);
    BLK_CHECK(exclusive_scan(ctx, ctx->col_count, ctx->col_offset, n_cols + 1, st));
    if (n_overrides) {
        ovr_scatter_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_offset,
            ctx->col_count, ctx->entries, ctx->ovr_owner);
        ovr_sort_kernel<<<grid_for(n_overrides, 256), 256, 0, st>>>(ovr, n_overrides, r, ctx->col_offset, ctx->entries,
            ctx->ovr_owner);
        BLK_CUDA(cudaGetLastError(), "override kernels");
    }
    ctx->counts_zero = true; // the scatter counted every column back down
    BLK_CHECK(launch_surface(ctx, st, ctx->env_mask));
    prof_mark(ctx, mark, 1, st);
    BLK_CHECK(launch_generation(ctx, static_cast<uint32_t>(n_items), st, true));
    prof_mark(ctx, mark, 2, st);
    return BLK_OK;
}

int blk_place_torches(blk_ctx* ctx, const uint32_t* env_seeds, uint32_t per_env, blk_override* out,
    uint32_t* out_count, uintptr_t stream_handle)
{
    if (!ctx || !env_seeds || !out || !out_count) {
        set_error("blk_place_torches: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t envs = ctx->cfg.num_envs;
    const void* seeds_dev = nullptr;
    BLK_CHECK(stage_input(env_seeds, envs * sizeof(uint32_t), ctx->seeds, st, &seeds_dev));
    const uint64_t total = envs * per_env;
    if (total > 0xFFFFFFFFull) {
        set_error("blk_place_torches: too many torches");
        return BLK_ERR_CAPACITY;
    }
    // Entry g = env * per_env + i; entries that found no free surface cell
    // carry y = INT32_MIN and are ignored by blk_generate.
    place_torches_kernel<<<grid_for(total ? total : 1, 256), 256, 0, st>>>(static_cast<const uint32_t*>(seeds_dev),
        ctx->cfg.num_envs, per_env, region(ctx), terrain_params(ctx), out, out_count, ctx->flags);
    return cuda_fail(cudaGetLastError(), "place_torches launch");
}

int blk_apply_edits(blk_ctx* ctx, const blk_override* edits, uint32_t n_edits, uintptr_t stream_handle)
{
    if (!ctx || (n_edits && !edits)) {
        set_error("blk_apply_edits: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_apply_edits: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    if (n_edits > ctx->cfg.max_edits) {
        set_error("blk_apply_edits: " + std::to_string(n_edits) + " edits exceed max_edits "
            + std::to_string(ctx->cfg.max_edits));
        return BLK_ERR_CAPACITY;
    }
    if (n_edits == 0)
        return BLK_OK;
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const void* e_dev = nullptr;
    BLK_CHECK(stage_input(edits, static_cast<size_t>(n_edits) * sizeof(blk_override), ctx->edits, st, &e_dev));
    const auto* e = static_cast<const blk_override*>(e_dev);
    const uint32_t envs = ctx->cfg.num_envs;
    const int mark = prof_begin(ctx, 1, st);
    BLK_CUDA(cudaMemsetAsync(ctx->edit_env_count, 0, (envs + 1) * sizeof(uint32_t), st), "memset edit counts");
    edit_count_kernel<<<grid_for(n_edits, 256), 256, 0, st>>>(e, n_edits, envs, ctx->edit_env_count);
    BLK_CHECK(exclusive_scan(ctx, ctx->edit_env_count, ctx->edit_env_offset, envs + 1, st));
    BLK_CUDA(cudaMemsetAsync(ctx->edit_env_count, 0, (envs + 1) * sizeof(uint32_t), st), "memset edit cursors");
    edit_scatter_kernel<<<grid_for(n_edits, 256), 256, 0, st>>>(e, n_edits, envs, ctx->edit_env_offset,
        ctx->edit_env_count, ctx->edit_order);
    EditArgs a;
    a.edits = e;
    a.env_offset = ctx->edit_env_offset;
    a.order = ctx->edit_order;
    a.changes = ctx->edit_changes;
    a.ids = ctx->ids;
    a.hmap = ctx->hmap;
    a.r = region(ctx);
    a.env_stride = ctx->env_stride;
    apply_edits_kernel<<<(envs + kEditWarps - 1) / kEditWarps, 32 * kEditWarps, 0, st>>>(a);
    mark_changes_kernel<<<grid_for(2ull * n_edits, 256), 256, 0, st>>>(a);
    BLK_CUDA(cudaGetLastError(), "apply edits launch");
    prof_mark(ctx, mark, 1, st);
    BLK_CHECK(launch_relight(ctx, st));
    prof_mark(ctx, mark, 2, st);
    return BLK_OK;
}

int blk_build_render_voxels(blk_ctx* ctx, uint32_t env, void* voxels, uint32_t max_voxels, uint32_t* count,
    int32_t* header, uintptr_t stream_handle)
{
    if (!ctx || !count || !header || (max_voxels && !voxels) || env >= ctx->cfg.num_envs) {
        set_error("blk_build_render_voxels: invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_build_render_voxels: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    VoxelArgs a;
    a.ids = ctx->ids + static_cast<uint64_t>(env) * ctx->env_stride;
    a.light = ctx->light + static_cast<uint64_t>(env) * ctx->env_stride;
    a.W = static_cast<int32_t>(ctx->cfg.width);
    a.H = static_cast<int32_t>(ctx->cfg.height);
    a.D = static_cast<int32_t>(ctx->cfg.depth);
    const uint64_t rows = static_cast<uint64_t>(a.D) * a.H;
    if (rows + 1 > static_cast<uint64_t>(ctx->cfg.num_envs) * ctx->columns_per_env + 1) {
        set_error("blk_build_render_voxels: region too small for the row scratch");
        return BLK_ERR_CAPACITY;
    }
    a.row_count = ctx->col_count; // scratch: the override counts are not live between calls
    ctx->counts_zero = false;
    uint32_t* row_offset = ctx->col_offset;
    voxel_count_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, st>>>(a);
    BLK_CHECK(exclusive_scan(ctx, a.row_count, row_offset, rows, st));
    voxel_write_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, st>>>(a, row_offset,
        static_cast<uint32_t*>(voxels), max_voxels, count, header, ctx->origins + env, make_int3(0, 0, 0));
    return cuda_fail(cudaGetLastError(), "render voxel launch");
}

int blk_effective_light(blk_ctx* ctx, const uint8_t* dimming, uint8_t* out, uintptr_t stream_handle)
{
    if (!ctx || !dimming || !out) {
        set_error("blk_effective_light: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const void* d_dev = nullptr;
    // dimming is staged through the edit-count scratch (num_envs + 1 words >= num_envs bytes).
    BLK_CHECK(stage_input(dimming, ctx->cfg.num_envs, ctx->edit_env_count, st, &d_dev));
    if (ctx->env_stride % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0) {
        set_error("blk_effective_light: output must be 16-byte aligned");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    const uint64_t quads_per_env = ctx->env_stride / 16;
    const uint64_t total = quads_per_env * ctx->cfg.num_envs;
    effective_light_kernel<<<grid_for(total, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(ctx->light),
        reinterpret_cast<uint4*>(out), static_cast<const uint8_t*>(d_dev), quads_per_env, total);
    return cuda_fail(cudaGetLastError(), "effective light launch");
}

uint8_t blk_sky_light_at_time(uint32_t t)
{
    // src/world/Lighting.cpp:21-49 with src/world/WorldTime.h:10-18.
    const int sunsetStart = 12000, sunsetEnd = 13702, sunriseStart = 22300, sunriseEnd = 23961;
    const int tt = static_cast<int>(t % 24000u);
    if (tt < sunsetStart)
        return 15;
    if (tt <= sunsetEnd)
        return static_cast<uint8_t>(15 - 11 * (tt - sunsetStart) / (sunsetEnd - sunsetStart));
    if (tt <= sunriseStart)
        return 4;
    if (tt <= sunriseEnd)
        return static_cast<uint8_t>(4 + 11 * (tt - sunriseStart) / (sunriseEnd - sunriseStart));
    return 15;
}

void blk_render_params_at(float x, float y, float z, float yaw, float pitch, uint32_t tick, blk_render_params* out)
{
    if (!out)
        return;
    const float pi = 3.14159265358979323846f;
    const int t = static_cast<int>(tick % 24000u);
    auto normalize3 = [](float v[3]) {
        const float inv = 1.0f / std::sqrt(v[0] * v[0] + v[1] * v[1] + v[2] * v[2]);
        v[0] *= inv;
        v[1] *= inv;
        v[2] *= inv;
    };
    // Camera (src/graphics/Renderer.cpp:76-80, 773-778): eye 1.62 above the feet.
    blk_render_params p {};
    p.origin[0] = x;
    p.origin[1] = y + 1.62f;
    p.origin[2] = z;
    const float pc = std::cos(pitch);
    p.forward[0] = std::sin(yaw) * pc;
    p.forward[1] = std::sin(pitch);
    p.forward[2] = std::cos(yaw) * pc;
    normalize3(p.forward);
    p.right[0] = std::cos(yaw);
    p.right[1] = 0.0f;
    p.right[2] = -std::sin(yaw);
    normalize3(p.right);
    p.up[0] = p.forward[1] * p.right[2] - p.forward[2] * p.right[1];
    p.up[1] = p.forward[2] * p.right[0] - p.forward[0] * p.right[2];
    p.up[2] = p.forward[0] * p.right[1] - p.forward[1] * p.right[0];
    normalize3(p.up);
    // Projection and fog (src/graphics/Renderer.cpp:795-800).
    p.far_plane = 48.0f;
    p.fov_radians = pi / 2.25f;
    p.fog_start = 10.0f;
    p.fog_end = 28.0f;
    // Sky light factor (src/world/Lighting.cpp:21-51, float trait 4/15 .. 1).
    const float fmin = 4.0f / 15.0f, fmax = 1.0f;
    float factor = fmax;
    if (t >= 12000 && t <= 13702)
        factor = fmax - (fmax - fmin) * static_cast<float>(t - 12000) / static_cast<float>(13702 - 12000);
    else if (t > 13702 && t <= 22300)
        factor = fmin;
    else if (t > 22300 && t <= 23961)
        factor = fmin + (fmax - fmin) * static_cast<float>(t - 22300) / static_cast<float>(23961 - 22300);
    // Sky colour (src/world/Lighting.cpp:53-80): night-day mix by brightness,
    // then sunset / sunrise tints over their ramps.
    const float day[3] = { 0.42f, 0.64f, 0.86f }, night[3] = { 0.015f, 0.025f, 0.070f };
    const float sunrise[3] = { 0.72f, 0.42f, 0.24f }, sunset[3] = { 0.75f, 0.34f, 0.20f };
    const float brightness = (factor - fmin) / (fmax - fmin);
    for (int k = 0; k < 3; ++k)
        p.sky_color[k] = night[k] * (1.0f - brightness) + day[k] * brightness;
    auto tint = [&](int start, int end, const float* target) {
        if (t >= start && t <= end) {
            const float progress = static_cast<float>(t - start) / static_cast<float>(end - start);
            const float tri = 1.0f - std::fabs(2.0f * progress - 1.0f);
            const float c = std::fmin(std::fmax(tri, 0.0f), 1.0f);
            const float w = c * c * (3.0f - 2.0f * c);
            for (int k = 0; k < 3; ++k)
                p.sky_color[k] = p.sky_color[k] * (1.0f - w) + target[k] * w;
        }
    };
    tint(12000, 13702, sunset);
    tint(22300, 23961, sunrise);
    p.sky_light_dimming = 15u - blk_sky_light_at_time(static_cast<uint32_t>(t));
    // Light direction (src/world/Lighting.cpp:88-112): the sun (or moon) on a
    // circle around noon, tilted 0.3 along z, always above the horizon.
    int offset = t - 6000;
    if (offset < -12000)
        offset += 24000;
    else if (offset >= 12000)
        offset -= 24000;
    const float angle = 2.0f * pi * static_cast<float>(offset) / 24000.0f;
    float sun[3] = { -std::sin(angle), std::cos(angle), 0.3f };
    if (sun[1] < 0.0f)
        for (float& v : sun)
            v = -v;
    normalize3(sun);
    for (int k = 0; k < 3; ++k)
        p.sky_light_direction[k] = sun[k];
    *out = p;
}

static int render_common(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height,
    uint8_t* out_rgba, float* out_nchw, uintptr_t stream_handle, const char* name)
{
    if (!ctx || !params || (!out_rgba && !out_nchw) || width == 0 || height == 0 || width > 8192 || height > 8192) {
        set_error(std::string(name) + ": invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error(std::string(name) + ": call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if ((out_rgba && !device_memory(out_rgba)) || (out_nchw && !device_memory(out_nchw))) {
        set_error(std::string(name) + ": outputs must be device memory");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    const void* p = nullptr;
    BLK_CHECK(stage_input(params, sizeof(blk_render_params) * ctx->cfg.num_envs, ctx->render_params, st, &p));
    return launch_render(ctx, static_cast<const blk_render_params*>(p), width, height, out_rgba, out_nchw, st);
}

int blk_render_frames(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height,
    uint8_t* out_rgba, uintptr_t stream_handle)
{
    return render_common(ctx, params, width, height, out_rgba, nullptr, stream_handle, "blk_render_frames");
}

int blk_render_observations(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height,
    float* out_nchw, uint8_t* out_rgba, uintptr_t stream_handle)
{
    if (!out_nchw) {
        set_error("blk_render_observations: null observation tensor");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    return render_common(ctx, params, width, height, out_rgba, out_nchw, stream_handle, "blk_render_observations");
}

int blk_readback(blk_ctx* ctx, uint32_t env_begin, uint32_t n_envs, uint8_t* ids, uint8_t* light, int16_t* height_map,
    uintptr_t stream_handle)
{
    if (!ctx || static_cast<uint64_t>(env_begin) + n_envs > ctx->cfg.num_envs) {
        set_error("blk_readback: invalid env range");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    const uint64_t vb = ctx->env_stride * n_envs, off = ctx->env_stride * env_begin;
    if (ids)
        BLK_CUDA(cudaMemcpyAsync(ids, ctx->ids + off, vb, cudaMemcpyDefault, st), "readback ids");
    if (light)
        BLK_CUDA(cudaMemcpyAsync(light, ctx->light + off, vb, cudaMemcpyDefault, st), "readback light");
    if (height_map)
        BLK_CUDA(cudaMemcpyAsync(height_map, ctx->hmap + ctx->columns_per_env * env_begin,
                     ctx->columns_per_env * n_envs * sizeof(int16_t), cudaMemcpyDefault, st),
            "readback height map");
    return BLK_OK;
}

int blk_query_cells(blk_ctx* ctx, const blk_cell_query* queries, uint32_t n, uint8_t* out_block, uint8_t* out_light,
    int32_t* out_height, uintptr_t stream_handle)
{
    if (!ctx || (n && !queries)) {
        set_error("blk_query_cells: invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_query_cells: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    if (n == 0)
        return BLK_OK;
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!device_memory(queries) || (out_block && !device_memory(out_block)) || (out_light && !device_memory(out_light))
        || (out_height && !device_memory(out_height))) {
        set_error("blk_query_cells: queries and outputs must be device memory");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    query_cells_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream_handle)>>>(queries, n, ctx->ids, ctx->light,
        ctx->hmap, region(ctx), ctx->env_stride, out_block, out_light, out_height);
    return cuda_fail(cudaGetLastError(), "query_cells_kernel launch");
}

int blk_query_solid(blk_ctx* ctx, const blk_box_query* queries, uint32_t n, uint8_t* out_solid,
    uintptr_t stream_handle)
{
    if (!ctx || (n && (!queries || !out_solid))) {
        set_error("blk_query_solid: invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_query_solid: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    if (n == 0)
        return BLK_OK;
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!device_memory(queries) || !device_memory(out_solid)) {
        set_error("blk_query_solid: queries and outputs must be device memory");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    query_solid_kernel<<<grid_for(static_cast<uint64_t>(n) * 32, 256), 256, 0, as_stream(stream_handle)>>>(queries,
        n, ctx->ids, region(ctx), ctx->env_stride, out_solid);
    return cuda_fail(cudaGetLastError(), "query_solid_kernel launch");
}

int blk_snapshot_overrides(blk_ctx* ctx, uint32_t env, blk_override* out, uint32_t capacity, uint32_t* count,
    uintptr_t stream_handle)
{
    if (!ctx || !count || (capacity && !out) || env >= ctx->cfg.num_envs) {
        set_error("blk_snapshot_overrides: invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (!ctx->generated) {
        set_error("blk_snapshot_overrides: call blk_generate first");
        return BLK_ERR_NOT_READY;
    }
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!device_memory(count) || (capacity && !device_memory(out))) {
        set_error("blk_snapshot_overrides: outputs must be device memory");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    const uint64_t columns = ctx->columns_per_env;
    const uint8_t* ids = ctx->ids + static_cast<uint64_t>(env) * ctx->env_stride;
    const int16_t* top = ctx->terrain_top + static_cast<uint64_t>(env) * columns;
    // Scratch: the override CSR counts / offsets are not live between calls.
    ctx->counts_zero = false; // the counts serve as scratch here
    snapshot_count_kernel<<<grid_for(columns, 256), 256, 0, st>>>(ids, top, region(ctx), ctx->col_count);
    BLK_CUDA(cudaGetLastError(), "snapshot count launch");
    BLK_CHECK(exclusive_scan(ctx, ctx->col_count, ctx->col_offset, columns, st));
    snapshot_write_kernel<<<grid_for(columns, 256), 256, 0, st>>>(ids, top, region(ctx), env, ctx->col_count,
        ctx->col_offset, out, capacity, count);
    return cuda_fail(cudaGetLastError(), "snapshot write launch");
}

int blk_sync(blk_ctx* ctx, uintptr_t stream_handle)
{
    if (!ctx) {
        set_error("blk_sync: null context");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    BLK_CUDA(cudaMemcpyAsync(ctx->h_flags, ctx->flags, sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "flag copy");
    BLK_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    const uint32_t f = *ctx->h_flags;
    if (f) {
        BLK_CUDA(cudaMemsetAsync(ctx->flags, 0, sizeof(uint32_t), st), "flag reset");
        BLK_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
        std::string msg = "device flags:";
        if (f & kFlagOverrideList)
            msg += " override list of a column longer than 65535";
        if (f & kFlagBandTooWide)
            msg += " light band wider than supported";
        if (f & kFlagEditOverflow)
            msg += " edit bookkeeping overflow";
        if (f & kFlagPermuteGuard)
            msg += " permutation guard hit";
        if (f & kFlagEnvIndex)
            msg += " partial reset env index out of range";
        if (f & kFlagRelightRegion)
            msg += " relight region larger than its size class";
        set_error(msg);
        return BLK_ERR_DEVICE_FLAG;
    }
    return BLK_OK;
}

int blk_set_generation_path(blk_ctx* ctx, int path)
{
    if (!ctx || (path != BLK_GENERATION_SURFACE && path != BLK_GENERATION_TILES && path != BLK_GENERATION_AUTO)) {
        set_error("blk_set_generation_path: null context or unknown path");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    ctx->generation_path = path;
    return BLK_OK;
}

int blk_generation_fallback_tiles(blk_ctx* ctx, uint32_t* count)
{
    if (!ctx || !count) {
        set_error("blk_generation_fallback_tiles: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (generation_path_of(ctx) != BLK_GENERATION_SURFACE) {
        *count = 0;
        return BLK_OK;
    }
    BLK_CUDA(cudaDeviceSynchronize(), "device synchronize");
    BLK_CUDA(cudaMemcpy(count, ctx->fallback_count, sizeof(uint32_t), cudaMemcpyDeviceToHost), "fallback count read");
    return BLK_OK;
}

int blk_profile_enable(blk_ctx* ctx, int enable)
{
    if (!ctx) {
        set_error("blk_profile_enable: null context");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    ctx->profiling = enable != 0;
    return BLK_OK;
}

int blk_profile_read(blk_ctx* ctx, blk_profile* out, int reset)
{
    if (!ctx || !out) {
        set_error("blk_profile_read: null argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    BLK_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    for (auto& m : ctx->marks) {
        BLK_CUDA(cudaEventSynchronize(m.e[2]), "cudaEventSynchronize");
        float a = 0.f, b = 0.f;
        BLK_CUDA(cudaEventElapsedTime(&a, m.e[0], m.e[1]), "cudaEventElapsedTime");
        BLK_CUDA(cudaEventElapsedTime(&b, m.e[1], m.e[2]), "cudaEventElapsedTime");
        if (m.kind == 0) {
            ctx->prof.generate_prep_ms += a;
            ctx->prof.generate_tiles_ms += b;
            ctx->prof.generate_calls += 1;
        } else {
            ctx->prof.edits_prep_ms += a;
            ctx->prof.relight_ms += b;
            ctx->prof.edit_calls += 1;
        }
        for (cudaEvent_t ev : m.e)
            cudaEventDestroy(ev);
    }
    ctx->marks.clear();
    *out = ctx->prof;
    if (reset)
        ctx->prof = blk_profile {};
    return BLK_OK;
}

int blk_convert_rgba8_to_float_nchw(const void* rgba8, float* nchw, uint32_t batch, uint32_t width, uint32_t height,
    uintptr_t stream_handle)
{
    if ((!rgba8 || !nchw) && batch && width && height) {
        set_error("blk_convert_rgba8_to_float_nchw: null pointer");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    const uint64_t ppi = static_cast<uint64_t>(width) * height;
    const uint64_t total = ppi * batch;
    if (total == 0)
        return BLK_OK;
    if (ppi > 0xFFFFFFFFull) {
        set_error("blk_convert_rgba8_to_float_nchw: image too large");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t st = as_stream(stream_handle);
    const bool vec = ppi % 4 == 0 && reinterpret_cast<uintptr_t>(rgba8) % 16 == 0 && reinterpret_cast<uintptr_t>(nchw) % 16 == 0;
    if (vec) {
        const uint64_t quads = total / 4;
        int blocks = static_cast<int>((quads + 255) / 256);
        if (blocks > 148 * 32)
            blocks = 148 * 32;
        rgba_to_nchw_vec_kernel<<<blocks, 256, 0, st>>>(static_cast<const uint4*>(rgba8), reinterpret_cast<float4*>(nchw),
            static_cast<uint32_t>(ppi / 4), quads);
    } else {
        int blocks = static_cast<int>((total + 255) / 256);
        if (blocks > 148 * 32)
            blocks = 148 * 32;
        rgba_to_nchw_scalar_kernel<<<blocks, 256, 0, st>>>(static_cast<const uchar4*>(rgba8), nchw,
            static_cast<uint32_t>(ppi), total);
    }
    return cuda_fail(cudaGetLastError(), "rgba8 conversion launch");
}

int blk_build_render_voxels_static(const uint8_t* ids, const uint8_t* light, uint32_t width, uint32_t height,
    uint32_t depth, int32_t origin_x, int32_t origin_y, int32_t origin_z, void* voxels, uint32_t max_voxels,
    uint32_t* count, int32_t* header, uintptr_t stream_handle)
{
    if (!ids || !light || !count || !header || (max_voxels && !voxels) || width == 0 || height == 0 || depth == 0) {
        set_error("blk_build_render_voxels_static: invalid argument");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    if (width > 64 || depth > 64 || height > 512
        || static_cast<uint64_t>(depth) * height > static_cast<uint64_t>(kStaticVoxelRows)) {
        set_error("blk_build_render_voxels_static: region exceeds the static scratch (width, depth <= 64, "
                  "height <= 512, depth * height <= 32768 rows)");
        return BLK_ERR_CAPACITY;
    }
    // The scratch array's device address on the current device. Outside a
    // stream capture it is looked up on every call (a cheap query that
    // allocates nothing), so a cudaDeviceReset or a reloaded module never
    // leaves a stale address behind; inside a capture the address of the
    // device's last uncaptured call is used, so the first call on a device
    // must come before any capture.
    constexpr int kMaxDevices = 64;
    static std::mutex setup_mutex;
    static uint32_t* scratch_of[kMaxDevices] = {};
    int dev = 0;
    BLK_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("blk_build_render_voxels_static: device ordinal out of range");
        return BLK_ERR_INVALID_ARGUMENT;
    }
    {
        // The world must live on the current device: the scratch is per device.
        cudaPointerAttributes attr {};
        if (cudaPointerGetAttributes(&attr, ids) != cudaSuccess) {
            cudaGetLastError();
            attr.type = cudaMemoryTypeUnregistered;
        }
        if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
            set_error("blk_build_render_voxels_static: ids must be device memory");
            return BLK_ERR_INVALID_ARGUMENT;
        }
        if (attr.type == cudaMemoryTypeDevice && attr.device != dev) {
            set_error("blk_build_render_voxels_static: ids live on device " + std::to_string(attr.device)
                + ", not on the current device " + std::to_string(dev));
            return BLK_ERR_INVALID_ARGUMENT;
        }
    }
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    BLK_CUDA(cudaStreamIsCapturing(as_stream(stream_handle), &capture), "cudaStreamIsCapturing");
    uint32_t* scratch;
    {
        std::lock_guard<std::mutex> lock(setup_mutex);
        if (capture == cudaStreamCaptureStatusNone) {
            void* addr = nullptr;
            BLK_CUDA(cudaGetSymbolAddress(&addr, g_voxel_rows), "cudaGetSymbolAddress (render voxel scratch)");
            scratch_of[dev] = static_cast<uint32_t*>(addr);
        } else if (!scratch_of[dev]) {
            set_error("blk_build_render_voxels_static: the first call on a device must come before any stream "
                      "capture");
            return BLK_ERR_INVALID_ARGUMENT;
        }
        scratch = scratch_of[dev];
    }
    cudaStream_t st = as_stream(stream_handle);
    VoxelArgs a;
    a.ids = ids;
    a.light = light;
    a.W = static_cast<int32_t>(width);
    a.H = static_cast<int32_t>(height);
    a.D = static_cast<int32_t>(depth);
    a.row_count = scratch; // every entry is written before it is read: nothing has to start at zero
    uint32_t* row_offset = scratch + kStaticVoxelRows;
    const uint32_t rows = depth * height;
    voxel_count_kernel<<<(rows + 127) / 128, 128, 0, st>>>(a);
    BLK_CUDA(cudaGetLastError(), "render voxel count launch");
    row_scan_one_block<<<1, 1024, 0, st>>>(a.row_count, row_offset, rows);
    BLK_CUDA(cudaGetLastError(), "render voxel scan launch");
    voxel_write_kernel<<<(rows + 127) / 128, 128, 0, st>>>(a, row_offset, static_cast<uint32_t*>(voxels), max_voxels,
        count, header, nullptr, make_int3(origin_x, origin_y, origin_z));
    return cuda_fail(cudaGetLastError(), "render voxel launch");
}

} // extern "C"

namespace blk {

int prof_begin(blk_ctx* ctx, int kind, cudaStream_t stream)
{
    if (!ctx->profiling)
        return -1;
    blk_ctx::Mark m {};
    m.kind = kind;
    for (cudaEvent_t& ev : m.e)
        if (cudaEventCreate(&ev) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
    cudaEventRecord(m.e[0], stream);
    ctx->marks.push_back(m);
    return static_cast<int>(ctx->marks.size()) - 1;
}

void prof_mark(blk_ctx* ctx, int mark, int which, cudaStream_t stream)
{
    if (mark >= 0 && mark < static_cast<int>(ctx->marks.size()))
        cudaEventRecord(ctx->marks[mark].e[which], stream);
}

} // namespace blk
