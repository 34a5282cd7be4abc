// CPU restatement of the reference world-state path (generation, sky fill,
// flood-fill light, render voxel list, observation conversion, day/night
// dimming) used ONLY as a test oracle and as the timed CPU baseline.
// The product never links, loads or calls anything declared here.
//
// Layouts follow the reference: volumes are indexed x + W*(y + H*z)
// (src/world/WorldGenerator.cu:183), height maps x + W*z (:218).
// Block ids follow the reference enum Air=0 Grass=1 Dirt=2 Stone=3 Torch=4
// (src/world/Block.h:11-19).
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum orc_terrain_mode {
    ORC_TERRAIN_REFERENCE = 0, // sin/cos + value noise, src/world/WorldGenerator.cu:112-140
    ORC_TERRAIN_FBM = 1,       // 4-octave value-noise fBm (this project's documented spec)
    ORC_TERRAIN_FLAT = 2,      // every column at height `fbm_base` (test worlds)
};

typedef struct orc_world_params {
    uint32_t seed;
    int32_t origin_x, origin_y, origin_z; // world coordinate of local (0,0,0)
    uint32_t width, height, depth;        // W (x), H (y), D (z)
    int32_t terrain_mode;                 // orc_terrain_mode
    int32_t fbm_base;                     // fBm: surface = base + round(amplitude * fbm)
    float fbm_amplitude;
} orc_world_params;

// Hash primitives (src/utility/Hash.h:10-41).
uint32_t orc_hash_combine2(uint32_t a, uint32_t b);
uint32_t orc_hash_combine3(uint32_t a, uint32_t b, uint32_t c);
uint32_t orc_hash(uint32_t v);
int32_t orc_seed_offset(uint32_t seed, uint32_t salt);

// Terrain surface height of world column (x, z) before clamping to the region.
int32_t orc_terrain_height(const orc_world_params* p, int32_t x, int32_t z);

// Dense block ids of the region with the override list applied
// (src/world/WorldGenerator.cu:142-219); overrides are world coordinates,
// at most one per cell. Also writes the height map (highest solid local y,
// -1 for an empty column; stored as world y like the reference, i.e. plus origin_y).
void orc_build_blocks(const orc_world_params* p, const int32_t* ovr_xyz, const uint8_t* ovr_block,
    uint32_t n_ovr, uint8_t* blocks, int16_t* height_map);

// Block and sky light of a dense block volume, restating the reference's
// per-source breadth-first propagation (src/world/WorldGenerator.cu:364-588).
// `height_map` holds world y (origin_y - 1 for empty columns).
void orc_light_per_source(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, const uint8_t* blocks,
    const int16_t* height_map, uint8_t* block_light, uint8_t* sky_light);

// The same light fields computed as one multi-source breadth-first search per
// light type (exact shortest-path form of the same definition). Independent
// second implementation used to cross-check the first.
void orc_light_multi_source(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, const uint8_t* blocks,
    const int16_t* height_map, uint8_t* block_light, uint8_t* sky_light);

// Render voxel list (src/world/WorldGenerator.cu:221-303): writes the 12-byte
// voxels in ascending volume-index order (the reference order is
// nondeterministic). Returns the number of visible voxels (all written when
// <= max_voxels).
uint32_t orc_render_voxels(uint32_t W, uint32_t H, uint32_t D, const uint8_t* blocks, const uint8_t* block_light,
    const uint8_t* sky_light, uint32_t* voxels, uint32_t max_voxels);

// RGBA8 -> float32 NCHW, x * (1/255) (src/environment/CudaObservation.cu:13-30).
void orc_convert_rgba8(const uint8_t* rgba, float* nchw, uint32_t batch, uint32_t width, uint32_t height);

// Integer sky level for a day tick (src/world/Lighting.cpp:21-49).
uint8_t orc_sky_light_at_time(uint32_t tick);

// Torch placement used by the benchmark worlds: `count` distinct columns from
// a keyed permutation of the W*D columns, torch at surface height + 1.
// Writes up to `count` world (x, y, z) triples; returns how many were placed.
uint32_t orc_place_torches(const orc_world_params* p, uint32_t count, uint32_t key, int32_t* out_xyz);

// One keyed pseudo-random permutation step over [0, n): the column index of
// the i-th torch.
uint32_t orc_permute(uint32_t i, uint32_t n, uint32_t key);

// Sequential edit semantics of World::setBlock (src/world/World.cpp:239-287)
// on a dense region: y outside [0, H) rejected, same block is a no-op, and
// digging the solid support under a torch removes the torch. `kind`:
// 0 = set block `block`, 1 = remove torch (cell becomes Air only if it holds a
// torch). Coordinates are local. Updates blocks and height_map (world y).
// Returns the number of cells actually changed.
uint32_t orc_apply_edits(uint32_t W, uint32_t H, uint32_t D, int32_t origin_y, uint8_t* blocks, int16_t* height_map,
    const int32_t* edit_xyz, const uint8_t* edit_kind, const uint8_t* edit_block, uint32_t n_edits);

// Ray-cast RGBA8 sRGB frame (height x width x 4) of one region with the
// voxel pipeline's shading (shaders/voxel.vert.hlsl:110-158,
// shaders/lighting.hlsl:3-30, shaders/mesh.frag.hlsl:12-82, shaders/fog.hlsl);
// `params` is a blk_render_params record (include/blk_world.h).
void orc_render_frame(uint32_t W, uint32_t H, uint32_t D, int32_t ox, int32_t oy, int32_t oz, const uint8_t* blocks,
    const uint8_t* block_light, const uint8_t* sky_light, const void* params, uint32_t width, uint32_t height,
    uint8_t* out_rgba);

#ifdef __cplusplus
}
#endif
