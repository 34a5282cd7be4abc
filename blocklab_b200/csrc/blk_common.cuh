// Device-side primitives shared by the world-state kernels: hashing, terrain
// heights, block predicates, device error flags.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace blk {

constexpr int kMaxDistance = 14;   // light reach, src/world/WorldGenerator.cu:22
constexpr int kHalo = kMaxDistance;

enum : uint8_t { Air = 0, Grass = 1, Dirt = 2, Stone = 3, Torch = 4 };

// Opaque == solid == not Air and not Torch (src/world/Block.h:30-34).
__host__ __device__ inline bool is_opaque(uint8_t b) { return b != Air && b != Torch; }

// Device error flag bits (ORed into the context's flag word).
enum : uint32_t {
    kFlagOverrideList = 1u << 0,   // per-column override list longer than supported
    kFlagBandTooWide = 1u << 1,    // light band wider than the compiled maximum
    kFlagEditOverflow = 1u << 2,   // changed-cell list of an edit batch overflowed
    kFlagPermuteGuard = 1u << 3,   // permutation walk hit its iteration bound
    kFlagEnvIndex = 1u << 4,       // an env index of a partial reset is out of range
    kFlagRelightRegion = 1u << 5,  // a relight region held more columns than its size class
};

// src/utility/Hash.h:10-24
__host__ __device__ inline uint32_t hash_combine2(uint32_t a, uint32_t b)
{
    a ^= b + 0x9e3779b9u + (a << 6) + (a >> 2);
    return a;
}
__host__ __device__ inline uint32_t hash_combine3(uint32_t a, uint32_t b, uint32_t c)
{
    return hash_combine2(a, hash_combine2(b, c));
}
// src/utility/Hash.h:26-34
__host__ __device__ inline uint32_t hash32(uint32_t v)
{
    v ^= v >> 16U;
    v *= 0x7feb352dU;
    v ^= v >> 15U;
    v *= 0x846ca68bU;
    v ^= v >> 16U;
    return v;
}
// src/utility/Hash.h:36-41
__host__ __device__ inline int32_t seed_offset(uint32_t seed, uint32_t salt)
{
    return static_cast<int32_t>(hash_combine2(seed, salt) % (4096U * 2U + 1U)) - 4096;
}

// Reference terrain, written with the same expression shape as
// src/world/WorldGenerator.cu:112-127 so that nvcc makes the same choices
// (fast __sinf/__cosf, contraction) as for the reference's CUDA build.
__device__ inline float ref_value_noise(uint32_t seed, int32_t x, int32_t z)
{
    const uint32_t hash = hash_combine3(seed, static_cast<uint32_t>(x), static_cast<uint32_t>(z));
    return static_cast<float>(hash & 0x00ffffffU) / static_cast<float>(0x00ffffffU) * 2.0f - 1.0f;
}

__device__ inline float ref_terrain_height(uint32_t seed, int32_t x, int32_t z)
{
    const int32_t sampleX = x + seed_offset(seed, 0x4f1bbc21U);
    const int32_t sampleZ = z + seed_offset(seed, 0x9a7c15d3U);
    const float low = __sinf(static_cast<float>(sampleX) * 0.17f) * 2.2f;
    const float high = __cosf(static_cast<float>(sampleZ) * 0.13f) * 1.8f;
    const float diagonal = __sinf(static_cast<float>(sampleX + sampleZ) * 0.08f) * 2.0f;
    const float rough = ref_value_noise(seed, sampleX / 3, sampleZ / 3) * 0.55f;
    return 9.0f + low + high + diagonal + rough;
}

// Lattice value of the fBm terrain in [-1, 1]: the reference's hash finalizer
// (src/utility/Hash.h:26-34) over hash_combine(octave seed, x, z), evaluated
// with explicitly rounded single operations (no contraction) so the CPU
// oracle reproduces it bit for bit. Without the finalizer hash_combine of
// small lattice coordinates changes only low bits and the terrain is flat.
__device__ inline float fbm_lattice(uint32_t seed, int32_t x, int32_t z)
{
    const uint32_t h = hash32(hash_combine3(seed, static_cast<uint32_t>(x), static_cast<uint32_t>(z)));
    const float q = __fdiv_rn(static_cast<float>(h & 0x00ffffffU), 16777215.0f);
    return __fsub_rn(__fmul_rn(q, 2.0f), 1.0f);
}

// Cell of octave o (lattice spacing 64 >> o) holding world coordinate v: the
// lattice index and the smoothstep weight of v inside the cell.
__device__ inline void fbm_cell(int o, int32_t v, int32_t& i, float& w)
{
    const float scale = 1.0f / static_cast<float>(64 >> o); // exact power of two
    const float f = __fmul_rn(static_cast<float>(v), scale);
    const float fl = floorf(f);
    i = static_cast<int32_t>(fl);
    const float t = __fsub_rn(f, fl);
    w = __fmul_rn(__fmul_rn(t, t), __fsub_rn(3.0f, __fmul_rn(2.0f, t)));
}

// Bilinear mix of one octave's four corner values.
__device__ inline float fbm_mix(float v00, float v10, float v01, float v11, float wx, float wz)
{
    const float a = __fadd_rn(v00, __fmul_rn(__fsub_rn(v10, v00), wx));
    const float b = __fadd_rn(v01, __fmul_rn(__fsub_rn(v11, v01), wx));
    return __fadd_rn(a, __fmul_rn(__fsub_rn(b, a), wz));
}

__device__ inline uint32_t fbm_octave_seed(uint32_t seed, int o)
{
    return hash32(hash_combine2(seed, static_cast<uint32_t>(o)));
}

// 4-octave value-noise fBm in [-1, 1]: lattice spacing 64 >> o, lacunarity 2,
// gain 0.5, smoothstep-weighted bilinear interpolation, normalised by 1.875;
// octave o uses the seed hash(hash_combine(seed, o)).
__device__ inline float fbm(uint32_t seed, int32_t x, int32_t z)
{
    float acc = 0.0f;
    float amp = 1.0f;
#pragma unroll
    for (int o = 0; o < 4; ++o) {
        const uint32_t s = fbm_octave_seed(seed, o);
        int32_t ix, iz;
        float wx, wz;
        fbm_cell(o, x, ix, wx);
        fbm_cell(o, z, iz, wz);
        const float n = fbm_mix(fbm_lattice(s, ix, iz), fbm_lattice(s, ix + 1, iz), fbm_lattice(s, ix, iz + 1),
            fbm_lattice(s, ix + 1, iz + 1), wx, wz);
        acc = __fadd_rn(acc, __fmul_rn(amp, n));
        amp = __fmul_rn(amp, 0.5f);
    }
    return __fdiv_rn(acc, 1.875f);
}

struct TerrainParams {
    int32_t mode;       // blk_terrain_mode
    int32_t base;
    float amplitude;
    int32_t height;     // H
};

// Surface (highest terrain block) of world column (wx, wz) as a y local to a
// region whose cell 0 lies at world y `oy`, not clamped: the layer rule needs
// the true surface even when it lies outside the region. Callers clamp to
// [-1, H-1] where they need a cell index.
__device__ inline int32_t terrain_top_local(const TerrainParams& t, uint32_t seed, int32_t wx, int32_t wz, int32_t oy)
{
    int32_t h;
    if (t.mode == 0)
        h = static_cast<int32_t>(ref_terrain_height(seed, wx, wz));
    else if (t.mode == 1)
        h = t.base + static_cast<int32_t>(roundf(__fmul_rn(t.amplitude, fbm(seed, wx, wz))));
    else
        h = t.base;
    return h - oy;
}

__device__ inline int32_t clamp_top(int32_t top, int32_t height)
{
    return top < -1 ? -1 : (top > height - 1 ? height - 1 : top);
}

// Terrain layer rule on local coordinates (src/world/WorldGenerator.cu:129-140).
__device__ inline uint8_t layer_block(int32_t y, int32_t top)
{
    if (y > top)
        return Air;
    if (y == top)
        return Grass;
    if (y > top - 4)
        return Dirt;
    return Stone;
}

// Keyed permutation of [0, n) by a 4-round Feistel network with cycle walking.
// Returns false if the walk exceeded its bound (cannot happen for a bijection;
// kept as a guard).
__device__ inline bool permute(uint32_t i, uint32_t n, uint32_t key, uint32_t& out)
{
    uint32_t bits = 2;
    while ((1u << bits) < n)
        bits += 2;
    const uint32_t half = bits / 2, mask = (1u << half) - 1u;
    uint32_t v = i;
    for (uint32_t guard = 0; guard <= (1u << bits); ++guard) {
        uint32_t l = v >> half, r = v & mask;
#pragma unroll
        for (uint32_t round = 0; round < 4; ++round) {
            const uint32_t f = hash32(hash_combine2(key + round, r)) & mask;
            const uint32_t nl = r;
            r = l ^ f;
            l = nl;
        }
        v = (l << half) | r;
        if (v < n) {
            out = v;
            return true;
        }
    }
    out = i % n;
    return false;
}

} // namespace blk
