// ORACLE — TEST INFRASTRUCTURE ONLY.
// A plain sequential C++ restatement of the reference world-state path. Only
// tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it,
// and only as the checker or the timed CPU baseline. The product library never
// links or calls it.
//
// Pinning: tests compare this restatement cell-for-cell with the reference's
// own code compiled from its sources (oracle/_ref/libref_cpu.so, see
// oracle/Makefile) and with the golden light masks of the reference's
// tests/WorldLighting.cpp. Compiled with -ffp-contract=off so float terrain
// arithmetic is one IEEE operation per source operation.

#include "blk_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <unordered_map>
#include <vector>

namespace {

enum : uint8_t { Air = 0, Grass = 1, Dirt = 2, Stone = 3, Torch = 4 };

// src/world/Block.h:30-34: solid and opaque are the same predicate.
inline bool opaque(uint8_t b) { return b != Air && b != Torch; }

constexpr int kMaxDistance = 14;               // src/world/WorldGenerator.cu:22
constexpr int kCube = 2 * kMaxDistance + 1;    // 29, src/world/WorldGenerator.cu:376

inline std::size_t vidx(uint32_t W, uint32_t H, int x, int y, int z)
{
    return static_cast<std::size_t>(x) + static_cast<std::size_t>(W) * (static_cast<std::size_t>(y) + static_cast<std::size_t>(H) * z);
}

// src/world/WorldGenerator.cu:112-116
float value_noise(uint32_t seed, int32_t x, int32_t z)
{
    const uint32_t h = orc_hash_combine3(seed, static_cast<uint32_t>(x), static_cast<uint32_t>(z));
    return static_cast<float>(h & 0x00ffffffU) / static_cast<float>(0x00ffffffU) * 2.0f - 1.0f;
}

// src/world/WorldGenerator.cu:118-127 (CPU-fallback flavour: libm sinf/cosf,
// include/blocklab/gpu/cuda/CudaHelpers.h:146-148).
float terrain_height_reference(uint32_t seed, int32_t x, int32_t z)
{
    const int32_t sx = x + orc_seed_offset(seed, 0x4f1bbc21U);
    const int32_t sz = z + orc_seed_offset(seed, 0x9a7c15d3U);
    const float low = std::sin(static_cast<float>(sx) * 0.17f) * 2.2f;
    const float high = std::cos(static_cast<float>(sz) * 0.13f) * 1.8f;
    const float diagonal = std::sin(static_cast<float>(sx + sz) * 0.08f) * 2.0f;
    const float rough = value_noise(seed, sx / 3, sz / 3) * 0.55f;
    return 9.0f + low + high + diagonal + rough;
}

// Lattice value of the fBm terrain in [-1, 1]: the reference's hash finalizer
// (src/utility/Hash.h:26-34) over hash_combine(octave seed, x, z). Without the
// finalizer hash_combine of small lattice coordinates changes only low bits
// and the terrain comes out flat.
float fbm_lattice(uint32_t seed, int32_t x, int32_t z)
{
    const uint32_t h = orc_hash(orc_hash_combine3(seed, static_cast<uint32_t>(x), static_cast<uint32_t>(z)));
    return static_cast<float>(h & 0x00ffffffU) / static_cast<float>(0x00ffffffU) * 2.0f - 1.0f;
}

// fBm terrain of the benchmark worlds (this project's spec; the reference has
// none). Four octaves of bilinear value noise with smoothstep weights on a
// lattice of spacing 64 >> o, lacunarity 2, gain 0.5, normalised by 1.875.
// Octave o uses the seed hash(hash_combine(seed, o)).
float fbm(uint32_t seed, int32_t x, int32_t z)
{
    float acc = 0.0f;
    float amp = 1.0f;
    for (int o = 0; o < 4; ++o) {
        const uint32_t s = orc_hash(orc_hash_combine2(seed, static_cast<uint32_t>(o)));
        const float scale = 1.0f / static_cast<float>(64 >> o); // exact power of two
        const float fx = static_cast<float>(x) * scale;
        const float fz = static_cast<float>(z) * scale;
        const float flx = std::floor(fx);
        const float flz = std::floor(fz);
        const int32_t ix = static_cast<int32_t>(flx);
        const int32_t iz = static_cast<int32_t>(flz);
        const float tx = fx - flx;
        const float tz = fz - flz;
        const float wx = (tx * tx) * (3.0f - 2.0f * tx);
        const float wz = (tz * tz) * (3.0f - 2.0f * tz);
        const float v00 = fbm_lattice(s, ix, iz);
        const float v10 = fbm_lattice(s, ix + 1, iz);
        const float v01 = fbm_lattice(s, ix, iz + 1);
        const float v11 = fbm_lattice(s, ix + 1, iz + 1);
        const float a = v00 + (v10 - v00) * wx;
        const float b = v01 + (v11 - v01) * wx;
        const float n = a + (b - a) * wz;
        acc = acc + amp * n;
        amp = amp * 0.5f;
    }
    return acc / 1.875f;
}

// src/world/WorldGenerator.cu:129-140 layer rule.
inline uint8_t layer_block(int32_t y, int32_t h)
{
    if (y > h)
        return Air;
    if (y == h)
        return Grass;
    if (y > h - 4)
        return Dirt;
    return Stone;
}

// One light type of the reference: breadth-first propagation of level 15 from
// each source over a 29^3 cube, out-of-region cells counting as solid, then a
// max-merge into the volume (src/world/WorldGenerator.cu:364-488).
void propagate_from_sources(uint32_t W, uint32_t H, uint32_t D, const uint8_t* blocks,
    const std::vector<int32_t>& sources, uint8_t* light)
{
    std::vector<uint8_t> solid(kCube * kCube * kCube);
    std::vector<uint8_t> cache(kCube * kCube * kCube);
    std::vector<int32_t> cur, next;
    auto cidx = [](int x, int y, int z) { return x + kCube * (y + kCube * z); };
    for (std::size_t s = 0; s < sources.size(); s += 3) {
        const int sx = sources[s], sy = sources[s + 1], sz = sources[s + 2];
        for (int z = 0; z < kCube; ++z)
            for (int y = 0; y < kCube; ++y)
                for (int x = 0; x < kCube; ++x) {
                    const int wx = sx + x - kMaxDistance, wy = sy + y - kMaxDistance, wz = sz + z - kMaxDistance;
                    const bool out = wx < 0 || wy < 0 || wz < 0 || wx >= static_cast<int>(W)
                        || wy >= static_cast<int>(H) || wz >= static_cast<int>(D);
                    solid[cidx(x, y, z)] = out || opaque(blocks[vidx(W, H, wx, wy, wz)]);
                    cache[cidx(x, y, z)] = 0;
                }
        cache[cidx(kMaxDistance, kMaxDistance, kMaxDistance)] = 15;
        cur.assign({ kMaxDistance, kMaxDistance, kMaxDistance });
        static const int dirs[6][3] = { { -1, 0, 0 }, { 1, 0, 0 }, { 0, -1, 0 }, { 0, 1, 0 }, { 0, 0, -1 }, { 0, 0, 1 } };
        for (int iter = 0; iter < kMaxDistance && !cur.empty(); ++iter) {
            next.clear();
            for (std::size_t q = 0; q < cur.size(); q += 3) {
                const int x = cur[q], y = cur[q + 1], z = cur[q + 2];
                const int l = cache[cidx(x, y, z)];
                if (l == 0)
                    continue;
                for (const auto& d : dirs) {
                    const int nx = x + d[0], ny = y + d[1], nz = z + d[2];
                    const int ci = cidx(nx, ny, nz);
                    if (solid[ci] || cache[ci] >= l - 1)
                        continue;
                    cache[ci] = static_cast<uint8_t>(l - 1);
                    next.insert(next.end(), { nx, ny, nz });
                }
            }
            std::swap(cur, next);
        }
        for (int z = 0; z < kCube; ++z)
            for (int y = 0; y < kCube; ++y)
                for (int x = 0; x < kCube; ++x) {
                    const int wx = sx + x - kMaxDistance, wy = sy + y - kMaxDistance, wz = sz + z - kMaxDistance;
                    if (wx < 0 || wy < 0 || wz < 0 || wx >= static_cast<int>(W) || wy >= static_cast<int>(H)
                        || wz >= static_cast<int>(D))
                        continue;
                    uint8_t& out = light[vidx(W, H, wx, wy, wz)];
                    out = std::max(out, cache[cidx(x, y, z)]);
                }
    }
}

// Multi-source breadth-first distance to the nearest source through
// non-opaque cells; level = max(0, 15 - distance).
void multi_source(uint32_t W, uint32_t H, uint32_t D, const uint8_t* blocks, const std::vector<std::size_t>& seeds,
    uint8_t* light)
{
    const std::size_t vol = static_cast<std::size_t>(W) * H * D;
    std::vector<int8_t> dist(vol, -1);
    std::vector<std::size_t> cur, next;
    for (std::size_t s : seeds) {
        if (dist[s] < 0) {
            dist[s] = 0;
            cur.push_back(s);
        }
    }
    for (int d = 0; d < kMaxDistance && !cur.empty(); ++d) {
        next.clear();
        for (std::size_t i : cur) {
            const int x = static_cast<int>(i % W);
            const int y = static_cast<int>((i / W) % H);
            const int z = static_cast<int>(i / (static_cast<std::size_t>(W) * H));
            const int nb[6][3] = { { x - 1, y, z }, { x + 1, y, z }, { x, y - 1, z }, { x, y + 1, z }, { x, y, z - 1 }, { x, y, z + 1 } };
            for (const auto& n : nb) {
                if (n[0] < 0 || n[1] < 0 || n[2] < 0 || n[0] >= static_cast<int>(W) || n[1] >= static_cast<int>(H)
                    || n[2] >= static_cast<int>(D))
                    continue;
                const std::size_t j = vidx(W, H, n[0], n[1], n[2]);
                if (dist[j] >= 0 || opaque(blocks[j]))
                    continue;
                dist[j] = static_cast<int8_t>(d + 1);
                next.push_back(j);
            }
        }
        std::swap(cur, next);
    }
    for (std::size_t i = 0; i < vol; ++i)
        light[i] = dist[i] < 0 ? 0 : static_cast<uint8_t>(15 - dist[i]);
}

} // namespace

extern "C" {

// src/utility/Hash.h:10-24 (two- and three-argument hashCombine).
uint32_t orc_hash_combine2(uint32_t a, uint32_t b)
{
    a ^= b + 0x9e3779b9u + (a << 6) + (a >> 2);
    return a;
}

uint32_t orc_hash_combine3(uint32_t a, uint32_t b, uint32_t c) { return orc_hash_combine2(a, orc_hash_combine2(b, c)); }

// src/utility/Hash.h:26-34
uint32_t orc_hash(uint32_t v)
{
    v ^= v >> 16U;
    v *= 0x7feb352dU;
    v ^= v >> 15U;
    v *= 0x846ca68bU;
    v ^= v >> 16U;
    return v;
}

// src/utility/Hash.h:36-41 with the default range 4096.
int32_t orc_seed_offset(uint32_t seed, uint32_t salt)
{
    return static_cast<int32_t>(orc_hash_combine2(seed, salt) % (4096U * 2U + 1U)) - 4096;
}

int32_t orc_terrain_height(const orc_world_params* p, int32_t x, int32_t z)
{
    switch (p->terrain_mode) {
    case ORC_TERRAIN_REFERENCE:
        return static_cast<int32_t>(terrain_height_reference(p->seed, x, z));
    case ORC_TERRAIN_FBM:
        return p->fbm_base + static_cast<int32_t>(std::round(p->fbm_amplitude * fbm(p->seed, x, z)));
    default:
        return p->fbm_base;
    }
}

void orc_build_blocks(const orc_world_params* p, const int32_t* ovr_xyz, const uint8_t* ovr_block, uint32_t n_ovr,
    uint8_t* blocks, int16_t* height_map)
{
    const uint32_t W = p->width, H = p->height, D = p->depth;
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t x = 0; x < W; ++x) {
            const int32_t h = orc_terrain_height(p, p->origin_x + static_cast<int32_t>(x), p->origin_z + static_cast<int32_t>(z));
            for (uint32_t y = 0; y < H; ++y)
                blocks[vidx(W, H, x, y, z)] = layer_block(p->origin_y + static_cast<int32_t>(y), h);
        }
    for (uint32_t i = 0; i < n_ovr; ++i) {
        const int32_t x = ovr_xyz[3 * i] - p->origin_x, y = ovr_xyz[3 * i + 1] - p->origin_y, z = ovr_xyz[3 * i + 2] - p->origin_z;
        if (x < 0 || y < 0 || z < 0 || x >= static_cast<int32_t>(W) || y >= static_cast<int32_t>(H) || z >= static_cast<int32_t>(D))
            continue;
        blocks[vidx(W, H, x, y, z)] = ovr_block[i];
    }
    // src/world/WorldGenerator.cu:208-218: highest solid world y, origin_y - 1 if none.
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t x = 0; x < W; ++x) {
            int32_t top = p->origin_y - 1;
            for (int32_t y = static_cast<int32_t>(H) - 1; y >= 0; --y)
                if (opaque(blocks[vidx(W, H, x, y, z)])) {
                    top = p->origin_y + y;
                    break;
                }
            height_map[x + W * z] = static_cast<int16_t>(top);
        }
}

void orc_light_per_source(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, const uint8_t* blocks,
    const int16_t* height_map, uint8_t* block_light, uint8_t* sky_light)
{
    const std::size_t vol = static_cast<std::size_t>(W) * H * D;
    std::memset(block_light, 0, vol);
    // Block light: every torch is a level-15 source (src/world/WorldGenerator.cu:196-206).
    std::vector<int32_t> sources;
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t y = 0; y < H; ++y)
            for (uint32_t x = 0; x < W; ++x)
                if (blocks[vidx(W, H, x, y, z)] == Torch)
                    sources.insert(sources.end(), { static_cast<int32_t>(x), static_cast<int32_t>(y), static_cast<int32_t>(z) });
    propagate_from_sources(W, H, D, blocks, sources, block_light);

    // Sky: vertical fill above the height map (src/world/WorldGenerator.cu:490-504) ...
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t y = 0; y < H; ++y)
            for (uint32_t x = 0; x < W; ++x)
                sky_light[vidx(W, H, x, y, z)] = origin_y + static_cast<int32_t>(y) > height_map[x + W * z] ? 15 : 0;
    // ... seeds at lit cells beside a darker neighbour column whose cell is
    // not opaque (src/world/WorldGenerator.cu:506-588) ...
    sources.clear();
    static const int dirs[4][2] = { { 1, 0 }, { -1, 0 }, { 0, 1 }, { 0, -1 } };
    std::vector<uint8_t> mark(H);
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t x = 0; x < W; ++x) {
            std::fill(mark.begin(), mark.end(), 0);
            const int cur = height_map[x + W * z] - origin_y;
            for (const auto& d : dirs) {
                const int nx = static_cast<int>(x) + d[0], nz = static_cast<int>(z) + d[1];
                if (nx < 0 || nz < 0 || nx >= static_cast<int>(W) || nz >= static_cast<int>(D))
                    continue;
                const int nh = height_map[nx + W * nz] - origin_y;
                for (int y = cur + 1; y < nh; ++y)
                    if (!opaque(blocks[vidx(W, H, nx, y, nz)]))
                        mark[y] = 1;
            }
            for (uint32_t y = 0; y < H; ++y)
                if (mark[y])
                    sources.insert(sources.end(), { static_cast<int32_t>(x), static_cast<int32_t>(y), static_cast<int32_t>(z) });
        }
    // ... each propagated like a torch and max-merged.
    propagate_from_sources(W, H, D, blocks, sources, sky_light);
}

void orc_light_multi_source(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, const uint8_t* blocks,
    const int16_t* height_map, uint8_t* block_light, uint8_t* sky_light)
{
    const std::size_t vol = static_cast<std::size_t>(W) * H * D;
    std::vector<std::size_t> seeds;
    for (std::size_t i = 0; i < vol; ++i)
        if (blocks[i] == Torch)
            seeds.push_back(i);
    multi_source(W, H, D, blocks, seeds, block_light);
    seeds.clear();
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t y = 0; y < H; ++y)
            for (uint32_t x = 0; x < W; ++x)
                if (origin_y + static_cast<int32_t>(y) > height_map[x + W * z])
                    seeds.push_back(vidx(W, H, x, y, z));
    multi_source(W, H, D, blocks, seeds, sky_light);
}

uint32_t orc_render_voxels(uint32_t W, uint32_t H, uint32_t D, const uint8_t* blocks, const uint8_t* block_light,
    const uint8_t* sky_light, uint32_t* voxels, uint32_t max_voxels)
{
    uint32_t count = 0;
    for (uint32_t z = 0; z < D; ++z)
        for (uint32_t y = 0; y < H; ++y)
            for (uint32_t x = 0; x < W; ++x) {
                const uint8_t b = blocks[vidx(W, H, x, y, z)];
                if (b == Air)
                    continue;
                // Neighbour order left, right, top, bottom, front, back
                // (src/world/Voxel.h:10-17, src/world/WorldGenerator.cu:254-259).
                const int nb[6][3] = { { (int)x - 1, (int)y, (int)z }, { (int)x + 1, (int)y, (int)z },
                    { (int)x, (int)y + 1, (int)z }, { (int)x, (int)y - 1, (int)z }, { (int)x, (int)y, (int)z + 1 },
                    { (int)x, (int)y, (int)z - 1 } };
                uint8_t nbBlock[6], nbBlockLight[6], nbSky[6];
                for (int f = 0; f < 6; ++f) {
                    const int* n = nb[f];
                    if (n[0] < 0 || n[1] < 0 || n[2] < 0 || n[0] >= (int)W || n[1] >= (int)H || n[2] >= (int)D) {
                        nbBlock[f] = Air;
                        nbBlockLight[f] = 0;
                        nbSky[f] = 0;
                    } else {
                        const std::size_t j = vidx(W, H, n[0], n[1], n[2]);
                        nbBlock[f] = blocks[j];
                        nbBlockLight[f] = block_light[j];
                        nbSky[f] = sky_light[j];
                    }
                }
                uint32_t faces = 0, bl = 0, sl = 0;
                if (b == Torch) {
                    faces = 0x2 | 0x1 | 0x4 | 0x10 | 0x20; // every face but the bottom
                    bl = 0xFFFFFFu;
                } else {
                    bool all_opaque = true;
                    for (int f = 0; f < 6; ++f)
                        all_opaque = all_opaque && opaque(nbBlock[f]);
                    if (all_opaque)
                        continue;
                    for (int f = 0; f < 6; ++f) {
                        if (!opaque(nbBlock[f]))
                            faces |= 1u << f;
                        bl |= static_cast<uint32_t>(nbBlockLight[f]) << (4 * f);
                    }
                }
                for (int f = 0; f < 6; ++f)
                    sl |= static_cast<uint32_t>(nbSky[f]) << (4 * f);
                if (count < max_voxels) {
                    voxels[3 * count] = static_cast<uint32_t>(b) | (faces << 5) | (z << 11) | (y << 17) | (x << 26);
                    voxels[3 * count + 1] = bl;
                    voxels[3 * count + 2] = sl;
                }
                ++count;
            }
    return count;
}

void orc_convert_rgba8(const uint8_t* rgba, float* nchw, uint32_t batch, uint32_t width, uint32_t height)
{
    const std::size_t plane = static_cast<std::size_t>(width) * height;
    const float inv255 = 1.0f / 255.0f;
    for (uint32_t n = 0; n < batch; ++n)
        for (std::size_t p = 0; p < plane; ++p) {
            const uint8_t* px = rgba + 4 * (n * plane + p);
            float* out = nchw + 3 * n * plane + p;
            out[0] = static_cast<float>(px[0]) * inv255;
            out[plane] = static_cast<float>(px[1]) * inv255;
            out[2 * plane] = static_cast<float>(px[2]) * inv255;
        }
}

// src/world/Lighting.cpp:21-49 (integer trait) with the tick constants of
// src/world/WorldTime.h:10-18.
uint8_t orc_sky_light_at_time(uint32_t t)
{
    const int sunsetStart = 12000, sunsetEnd = 13702, sunriseStart = 22300, sunriseEnd = 23961;
    const int tt = static_cast<int>(t);
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

uint32_t orc_permute(uint32_t i, uint32_t n, uint32_t key)
{
    uint32_t bits = 2;
    while ((1u << bits) < n)
        bits += 2;
    const uint32_t half = bits / 2, mask = (1u << half) - 1u;
    uint32_t v = i;
    for (uint32_t guard = 0; guard <= (1u << bits); ++guard) {
        uint32_t l = v >> half, r = v & mask;
        for (uint32_t round = 0; round < 4; ++round) {
            const uint32_t f = orc_hash(orc_hash_combine2(key + round, r)) & mask;
            const uint32_t nl = r;
            r = l ^ f;
            l = nl;
        }
        v = (l << half) | r;
        if (v < n)
            return v;
    }
    return i % n;
}

uint32_t orc_place_torches(const orc_world_params* p, uint32_t count, uint32_t key, int32_t* out_xyz)
{
    const uint32_t columns = p->width * p->depth;
    const uint32_t n = std::min(count, columns);
    uint32_t placed = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t c = orc_permute(i, columns, key);
        const int32_t x = static_cast<int32_t>(c % p->width), z = static_cast<int32_t>(c / p->width);
        const int32_t wx = p->origin_x + x, wz = p->origin_z + z;
        int32_t h = orc_terrain_height(p, wx, wz) - p->origin_y;
        h = std::clamp<int32_t>(h, -1, static_cast<int32_t>(p->height) - 1);
        const int32_t y = h + 1;
        if (y >= static_cast<int32_t>(p->height))
            continue;
        out_xyz[3 * placed] = wx;
        out_xyz[3 * placed + 1] = p->origin_y + y;
        out_xyz[3 * placed + 2] = wz;
        ++placed;
    }
    return placed;
}

uint32_t orc_apply_edits(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, uint8_t* blocks, int16_t* height_map,
    const int32_t* edit_xyz, const uint8_t* edit_kind, const uint8_t* edit_block, uint32_t n_edits)
{
    uint32_t changed = 0;
    // World::setBlock, src/world/World.cpp:239-287, on a dense region.
    auto set = [&](auto&& self, int x, int y, int z, uint8_t block) -> void {
        if (y < 0 || y >= static_cast<int>(H) || x < 0 || z < 0 || x >= static_cast<int>(W) || z >= static_cast<int>(D))
            return;
        uint8_t& cell = blocks[vidx(W, H, x, y, z)];
        const uint8_t old = cell;
        if (old == block)
            return;
        cell = block;
        ++changed;
        int16_t& hm = height_map[x + W * z];
        int top = hm - origin_y;
        if (opaque(block) && y > top)
            top = y;
        else if (!opaque(block) && opaque(old) && y == top) {
            top = -1;
            for (int yy = y - 1; yy >= 0; --yy)
                if (opaque(blocks[vidx(W, H, x, yy, z)])) {
                    top = yy;
                    break;
                }
        }
        hm = static_cast<int16_t>(top + origin_y);
        if (opaque(old) && !opaque(block) && y + 1 < static_cast<int>(H) && blocks[vidx(W, H, x, y + 1, z)] == Torch)
            self(self, x, y + 1, z, Air);
    };
    for (uint32_t i = 0; i < n_edits; ++i) {
        const int x = edit_xyz[3 * i], y = edit_xyz[3 * i + 1], z = edit_xyz[3 * i + 2];
        if (edit_kind[i] == 1) {
            if (y < 0 || y >= static_cast<int>(H) || x < 0 || z < 0 || x >= static_cast<int>(W) || z >= static_cast<int>(D))
                continue;
            if (blocks[vidx(W, H, x, y, z)] == Torch)
                set(set, x, y, z, Air);
        } else {
            set(set, x, y, z, edit_block[i]);
        }
    }
    return changed;
}

} // extern "C"

// ---------------------------------------------------------------- frames --
// CPU restatement of the voxel pipeline's shading for one region, ray-cast
// per pixel centre: shaders/voxel.vert.hlsl:110-158 (faces, torch box, face
// light), shaders/lighting.hlsl:3-30, shaders/mesh.frag.hlsl:12-82 (texels,
// sRGB palette, fog mix), shaders/projection.hlsl (camera), an sRGB target.
// Volumes in the reference layout x + W * (y + H * z).
namespace {

struct RenderParamsC {
    float origin[3], forward[3], right[3], up[3];
    float far_plane, fov_radians, fog_start, fog_end;
    float sky_color[3];
    uint32_t sky_light_dimming;
    float sky_light_direction[3];
    uint32_t reserved;
};

enum { kLeft = 0, kRight, kTop, kBottom, kFront, kBack };

float frac_(float x) { return x - std::floor(x); }
float sat_(float x) { return std::fmin(std::fmax(x, 0.0f), 1.0f); }
float lerp_(float a, float b, float t) { return a + t * (b - a); }

float hash21_(float px, float py)
{
    float x = frac_(px * 0.1031f), y = frac_(py * 0.1031f), z = frac_(px * 0.1031f);
    const float d = x * (y + 33.33f) + y * (z + 33.33f) + z * (x + 33.33f);
    x += d;
    y += d;
    z += d;
    return frac_((x + y) * z);
}

void texel_(int mat, float u, float v, float wx, float wz, float rgb[3])
{
    float tx, ty;
    if (mat == 0) {
        tx = std::floor(wx * 16.0f);
        ty = std::floor(wz * 16.0f);
    } else {
        tx = std::floor(sat_(u) * 15.999f);
        ty = std::floor(sat_(v) * 15.999f);
    }
    const float n = hash21_(tx + mat * 17.0f, ty + mat * 17.0f);
    float c[3];
    auto mix3 = [&](float a0, float a1, float a2, float b0, float b1, float b2) {
        c[0] = lerp_(a0, b0, n);
        c[1] = lerp_(a1, b1, n);
        c[2] = lerp_(a2, b2, n);
    };
    if (mat == 0) { // grass top
        const float blade = hash21_(tx * 1.7f + 4.0f, ty * 1.7f + 4.0f) >= 0.68f ? 1.0f : 0.0f;
        mix3(0.22f, 0.50f, 0.18f, 0.36f, 0.64f, 0.27f);
        c[0] += blade * 0.02f;
        c[1] += blade * 0.04f;
        c[2] += blade * 0.01f;
    } else if (mat == 1) {
        mix3(0.35f, 0.20f, 0.10f, 0.56f, 0.36f, 0.18f);
    } else if (mat == 2) {
        mix3(0.43f, 0.44f, 0.44f, 0.57f, 0.58f, 0.58f);
    } else if (mat == 3) { // grass side
        const float dirt[3] = { lerp_(0.32f, 0.48f, n), lerp_(0.20f, 0.31f, n), lerp_(0.11f, 0.17f, n) };
        const float grass[3] = { lerp_(0.18f, 0.30f, n), lerp_(0.46f, 0.58f, n), lerp_(0.15f, 0.21f, n) };
        float chance = 1.0f;
        if (ty >= 15.0f)
            chance = 0.0f;
        else if (ty >= 14.0f)
            chance = 0.12f;
        else if (ty >= 13.0f)
            chance = 0.32f;
        else if (ty >= 12.0f)
            chance = 0.58f;
        const float m = hash21_(tx + 11.0f, ty + 11.0f) >= 1.0f - chance ? 1.0f : 0.0f;
        for (int k = 0; k < 3; ++k)
            c[k] = lerp_(grass[k], dirt[k], m);
    } else if (mat == 6) { // torch side
        const float wood[3] = { lerp_(0.46f, 0.58f, n), lerp_(0.25f, 0.34f, n), lerp_(0.10f, 0.16f, n) };
        const float ember[3] = { lerp_(1.00f, 1.00f, n), lerp_(0.52f, 0.88f, n), lerp_(0.08f, 0.24f, n) };
        const float e = v >= 0.72f ? 1.0f : 0.0f;
        for (int k = 0; k < 3; ++k)
            c[k] = lerp_(wood[k], ember[k], e);
    } else { // torch top
        mix3(1.00f, 0.52f, 0.08f, 1.00f, 0.88f, 0.24f);
    }
    for (int k = 0; k < 3; ++k)
        rgb[k] = std::pow(sat_(c[k]), 2.2f);
}

float face_dot_(int f, const float v[3])
{
    switch (f) {
    case kLeft: return -v[0];
    case kRight: return v[0];
    case kTop: return v[1];
    case kBottom: return -v[1];
    case kFront: return v[2];
    default: return -v[2];
    }
}

float face_sky_(int f, const RenderParamsC& p)
{
    const float direct = lerp_(0.4f, 1.0f, sat_(face_dot_(f, p.sky_light_direction)));
    const float t = sat_(p.sky_light_direction[1] / 0.6f);
    const float fallback = 1.0f - t * t * (3.0f - 2.0f * t);
    if (fallback < 1e-3f)
        return direct;
    const float k = 1.0f / std::sqrt(1.09f);
    const float fd[3] = { 0.0f, k, 0.3f * k };
    return lerp_(direct, lerp_(0.4f, 1.0f, sat_(face_dot_(f, fd))), fallback);
}

float face_block_(int f)
{
    const float ka = 1.0f / std::sqrt(0.35f * 0.35f + 0.85f * 0.85f + 0.45f * 0.45f);
    const float fa = 1.0f / std::sqrt(0.55f * 0.55f + 0.65f * 0.65f + 0.25f * 0.25f);
    const float key[3] = { 0.35f * ka, 0.85f * ka, 0.45f * ka }, fill[3] = { -0.55f * fa, 0.65f * fa, -0.25f * fa };
    return 0.45f + sat_(face_dot_(f, key)) * 0.40f + sat_(face_dot_(f, fill)) * 0.15f;
}

uint32_t srgb8_(float c)
{
    c = sat_(c);
    const float s = c <= 0.0031308f ? 12.92f * c : 1.055f * std::pow(c, 1.0f / 2.4f) - 0.055f;
    return static_cast<uint32_t>(std::lrint(s * 255.0f));
}

} // namespace

extern "C" void orc_render_frame(uint32_t W, uint32_t H, uint32_t D, int32_t ox, int32_t oy, int32_t oz,
    const uint8_t* blocks, const uint8_t* block_light, const uint8_t* sky_light, const void* params, uint32_t width,
    uint32_t height, uint8_t* out_rgba)
{
    RenderParamsC p;
    std::memcpy(&p, params, sizeof(p));
    const int dims[3] = { static_cast<int>(W), static_cast<int>(H), static_cast<int>(D) };
    auto inside = [&](const int c[3]) {
        return c[0] >= 0 && c[1] >= 0 && c[2] >= 0 && c[0] < dims[0] && c[1] < dims[1] && c[2] < dims[2];
    };
    auto idx = [&](const int c[3]) { return static_cast<size_t>(c[0]) + W * (static_cast<size_t>(c[1]) + H * c[2]); };
    auto block = [&](const int c[3]) -> uint8_t { return inside(c) ? blocks[idx(c)] : 0; };
    auto opaque = [](uint8_t b) { return b != 0 && b != 4; };
    const float t = std::tan(p.fov_radians * 0.5f);
    const float aspect = static_cast<float>(width) / static_cast<float>(height);
    const float o[3] = { p.origin[0] - ox, p.origin[1] - oy, p.origin[2] - oz };
    const int off[6][3] = { { -1, 0, 0 }, { 1, 0, 0 }, { 0, 1, 0 }, { 0, -1, 0 }, { 0, 0, 1 }, { 0, 0, -1 } };
    const float kNear = 0.05f;
    // The walk stops at the fog end, where faces take the sky colour.
    const float far = p.fog_end > p.fog_start ? std::fmin(p.far_plane, p.fog_end) : p.far_plane;
    for (uint32_t py = 0; py < height; ++py)
        for (uint32_t px = 0; px < width; ++px) {
            const float xn = (px + 0.5f) / width * 2.0f - 1.0f, yn = (py + 0.5f) / height * 2.0f - 1.0f;
            const float vx = xn * aspect * t, vy = -yn * t;
            float d[3];
            for (int k = 0; k < 3; ++k)
                d[k] = p.right[k] * vx + p.up[k] * vy + p.forward[k];
            float s0 = 0.0f, s1 = far;
            int entry_axis = -1;
            for (int k = 0; k < 3; ++k) {
                if (std::fabs(d[k]) < 1e-20f) {
                    if (o[k] < 0.0f || o[k] >= dims[k])
                        s1 = -1.0f;
                } else {
                    float ta = (0.0f - o[k]) / d[k], tb = (dims[k] - o[k]) / d[k];
                    if (ta > tb)
                        std::swap(ta, tb);
                    if (ta > s0) {
                        s0 = ta;
                        entry_axis = k;
                    }
                    s1 = std::fmin(s1, tb);
                }
            }
            // hit: depth, face, block, owner cell, neighbour cell, box coordinates
            float hs = -1.0f, hl[3] = { 0, 0, 0 };
            int hf = -1, hn[3] = { 0, 0, 0 };
            uint8_t hb = 0;
            auto face_hit = [&](const int* owner, const int* other, int ax, float sh) {
                const int dir = other[ax] - owner[ax];
                hs = sh;
                hf = ax == 0 ? (dir > 0 ? kRight : kLeft) : (ax == 1 ? (dir > 0 ? kTop : kBottom) : (dir > 0 ? kFront : kBack));
                hb = block(owner);
                for (int k = 0; k < 3; ++k) {
                    hn[k] = other[k];
                    hl[k] = sat_(o[k] + d[k] * sh - owner[k]);
                }
                hl[ax] = dir > 0 ? 1.0f : 0.0f;
            };
            if (s0 <= s1) {
                int c[3], st[3];
                float tmax[3], tdel[3];
                for (int k = 0; k < 3; ++k) {
                    int ck = static_cast<int>(std::floor(o[k] + d[k] * s0));
                    ck = std::min(std::max(ck, 0), dims[k] - 1);
                    c[k] = ck;
                    if (d[k] > 0.0f) {
                        st[k] = 1;
                        tdel[k] = 1.0f / d[k];
                        tmax[k] = (ck + 1 - o[k]) / d[k];
                    } else if (d[k] < 0.0f) {
                        st[k] = -1;
                        tdel[k] = -1.0f / d[k];
                        tmax[k] = (ck - o[k]) / d[k];
                    } else {
                        st[k] = 0;
                        tdel[k] = 3.0e38f;
                        tmax[k] = 3.0e38f;
                    }
                }
                float s_cell = s0;
                if (entry_axis >= 0 && s0 >= kNear && s0 <= far && opaque(block(c))) {
                    int out_c[3] = { c[0], c[1], c[2] };
                    out_c[entry_axis] -= st[entry_axis];
                    face_hit(c, out_c, entry_axis, s0);
                }
                const int max_steps = dims[0] + dims[1] + dims[2] + 3;
                for (int it = 0; it < max_steps && hs < 0.0f; ++it) {
                    const uint8_t cur = block(c);
                    const int ax = tmax[0] <= tmax[1] ? (tmax[0] <= tmax[2] ? 0 : 2) : (tmax[1] <= tmax[2] ? 1 : 2);
                    const float s_cross = tmax[ax];
                    if (cur == 4) {
                        const float lo[3] = { c[0] + 0.4375f, static_cast<float>(c[1]), c[2] + 0.4375f };
                        const float hi[3] = { c[0] + 0.5625f, c[1] + 0.65f, c[2] + 0.5625f };
                        float tin = -3.0e38f, tout = 3.0e38f;
                        int fin = -1, fout = -1;
                        for (int k = 0; k < 3; ++k) {
                            if (d[k] == 0.0f) {
                                if (o[k] < lo[k] || o[k] > hi[k])
                                    tin = 3.0e38f;
                                continue;
                            }
                            float ta = (lo[k] - o[k]) / d[k], tb = (hi[k] - o[k]) / d[k];
                            int fa = k == 0 ? kLeft : (k == 1 ? kBottom : kBack);
                            int fb = k == 0 ? kRight : (k == 1 ? kTop : kFront);
                            if (ta > tb) {
                                std::swap(ta, tb);
                                std::swap(fa, fb);
                            }
                            if (ta > tin) {
                                tin = ta;
                                fin = fa;
                            }
                            if (tb < tout) {
                                tout = tb;
                                fout = fb;
                            }
                        }
                        const float lo_s = std::fmax(s_cell, kNear);
                        if (tin <= tout) {
                            float sh = -1.0f;
                            int fh = -1;
                            if (fin >= 0 && fin != kBottom && tin >= lo_s && tin <= s_cross)
                                sh = tin, fh = fin;
                            else if (fout >= 0 && fout != kBottom && tout >= lo_s && tout <= s_cross)
                                sh = tout, fh = fout;
                            if (fh >= 0 && sh <= far) {
                                hs = sh;
                                hf = fh;
                                hb = 4;
                                for (int k = 0; k < 3; ++k)
                                    hn[k] = c[k] + off[fh][k];
                                hl[0] = sat_((o[0] + d[0] * sh - lo[0]) / 0.125f);
                                hl[1] = sat_((o[1] + d[1] * sh - lo[1]) / 0.65f);
                                hl[2] = sat_((o[2] + d[2] * sh - lo[2]) / 0.125f);
                                break;
                            }
                        }
                    }
                    if (s_cross > s1 + 1e-4f || s_cross > far)
                        break;
                    int nxt[3] = { c[0], c[1], c[2] };
                    nxt[ax] += st[ax];
                    const uint8_t nb = block(nxt);
                    if (s_cross >= kNear && opaque(cur) != opaque(nb)) {
                        if (opaque(cur))
                            face_hit(c, nxt, ax, s_cross);
                        else
                            face_hit(nxt, c, ax, s_cross);
                        break;
                    }
                    for (int k = 0; k < 3; ++k)
                        c[k] = nxt[k];
                    s_cell = s_cross;
                    tmax[ax] += tdel[ax];
                    if (!inside(c))
                        break;
                }
            }
            float rgb[3];
            if (hs < 0.0f) {
                for (int k = 0; k < 3; ++k)
                    rgb[k] = p.sky_color[k];
            } else {
                uint32_t sky = 0, blk = 0;
                if (inside(hn)) {
                    sky = sky_light[idx(hn)];
                    blk = block_light[idx(hn)];
                }
                if (hb == 4)
                    blk = 15;
                const uint32_t cur_sky = sky - std::min(sky, p.sky_light_dimming);
                const float light = std::fmax(cur_sky * face_sky_(hf, p), blk * face_block_(hf)) / 15.0f;
                float u, v;
                switch (hf) {
                case kLeft:
                case kRight: u = hl[2]; v = hl[1]; break;
                case kTop: u = hl[0]; v = hl[2]; break;
                case kBottom: u = hl[2]; v = hl[0]; break;
                default: u = hl[0]; v = hl[1]; break;
                }
                int mat;
                if (hb == 1)
                    mat = hf == kTop ? 0 : (hf == kBottom ? 1 : 3);
                else if (hb == 2)
                    mat = 1;
                else if (hb == 3)
                    mat = 2;
                else
                    mat = hf == kTop ? 7 : 6;
                float alb[3];
                texel_(mat, u, v, o[0] + d[0] * hs + ox, o[2] + d[2] * hs + oz, alb);
                const float fog = sat_((hs - p.fog_start) / std::fmax(p.fog_end - p.fog_start, 0.001f));
                for (int k = 0; k < 3; ++k)
                    rgb[k] = lerp_(sat_(alb[k] * light), p.sky_color[k], fog);
            }
            uint8_t* q = out_rgba + (static_cast<size_t>(py) * width + px) * 4;
            q[0] = static_cast<uint8_t>(srgb8_(rgb[0]));
            q[1] = static_cast<uint8_t>(srgb8_(rgb[1]));
            q[2] = static_cast<uint8_t>(srgb8_(rgb[2]));
            q[3] = 255;
        }
}
