/*
 * blk_world.h — C ABI of the B200 world-state library (libblk_world.so).
 *
 * The library owns, per GPU context, a batch of `num_envs` independent voxel
 * regions (W x H x D each) resident in HBM, and exposes the reference's
 * world-state hot path over them:
 *   generation (seed + sparse override overlay -> block ids, height map),
 *   sky-light column fill and 6-neighbour flood-fill block/sky light,
 *   exact incremental relight after edits,
 *   the render voxel list, day/night effective light,
 *   and the RGBA8 -> float32 NCHW observation conversion.
 *
 * Conventions
 *   - Every entry point returns an int status (BLK_OK == 0); nothing aborts.
 *     blk_last_error() returns the message of the last failure on the
 *     calling thread.
 *   - All work is enqueued on the caller's stream (cudaStream_t passed as
 *     uintptr_t; 0 = legacy default stream). Calls are asynchronous unless
 *     stated otherwise; device-side error flags are reported by blk_sync().
 *   - Array arguments may live in host memory (pageable or pinned) or device
 *     memory; the library detects which and stages host data itself.
 *   - One context per GPU per host thread; a context is not thread-safe.
 *
 * Block ids are the reference's (src/world/Block.h:11-19):
 *   Air=0 Grass=1 Dirt=2 Stone=3 Torch=4. Opaque == solid == not Air/Torch.
 * Light bytes pack sky<<4 | block, each 0..15.
 *
 * Device layout of the world arrays (per env, column-major, y fastest):
 *   ids[env][z][x][y], light[env][z][x][y]  (uint8)
 *   height_map[env][z][x]                   (int16, world y of the highest
 *                                            solid block, origin_y-1 if none)
 * so one column of H cells is H contiguous bytes.
 */
#ifndef BLK_WORLD_H
#define BLK_WORLD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum blk_status {
    BLK_OK = 0,
    BLK_ERR_INVALID_ARGUMENT = 1,
    BLK_ERR_CUDA = 2,
    BLK_ERR_OUT_OF_MEMORY = 3,
    BLK_ERR_CAPACITY = 4,     /* an input exceeds a documented limit */
    BLK_ERR_DEVICE_FLAG = 5,  /* a kernel reported an internal limit or bound */
    BLK_ERR_NOT_READY = 6,    /* world not generated yet */
};

enum blk_terrain_mode {
    BLK_TERRAIN_REFERENCE = 0, /* reference sin/cos + value-noise heights */
    BLK_TERRAIN_FBM = 1,       /* 4-octave value-noise fBm: base + round(amplitude * fbm) */
    BLK_TERRAIN_FLAT = 2,      /* every column at height `fbm_base` */
};

enum blk_block {
    BLK_AIR = 0,
    BLK_GRASS = 1,
    BLK_DIRT = 2,
    BLK_STONE = 3,
    BLK_TORCH = 4,
};

enum blk_edit_kind {
    BLK_EDIT_SET = 0,          /* World::setBlock(pos, block) */
    BLK_EDIT_REMOVE_TORCH = 1, /* setBlock(pos, Air) only if the cell holds a torch */
};

typedef struct blk_world_config {
    uint32_t num_envs;
    uint32_t width;    /* W: x extent, 1..4096 */
    uint32_t height;   /* H: y extent, multiple of 32, 32..256 */
    uint32_t depth;    /* D: z extent, 1..4096 */
    int32_t origin_x;  /* world coordinate of local (0, 0, 0) of every env until */
    int32_t origin_y;  /* blk_generate / blk_generate_envs gives it its own      */
    int32_t origin_z;
    int32_t terrain_mode;   /* blk_terrain_mode */
    int32_t fbm_base;
    float fbm_amplitude;
    uint32_t max_overrides; /* capacity of one blk_generate override list, at most 2^26 */
    uint32_t max_edits;     /* capacity of one blk_apply_edits list */
} blk_world_config;

/* One sparse override / edit; world coordinates. Mirrors the reference's
 * BlockOverride {IVec3 coord; Block block} (src/world/Block.h:55-58) plus the
 * env index of the batch and the edit kind. */
typedef struct blk_override {
    int32_t x, y, z;
    uint16_t env;
    uint8_t block; /* blk_block */
    uint8_t kind;  /* blk_edit_kind; ignored by blk_generate */
} blk_override;

typedef struct blk_world_views {
    uint8_t* ids;          /* device, num_envs * D * W * H */
    uint8_t* light;        /* device, same shape, sky<<4 | block */
    int16_t* height_map;   /* device, num_envs * D * W */
    const int32_t* env_origins; /* device, num_envs * 4: x, y, z (world coordinates of
                                   the env's local (0, 0, 0)) and one unused word */
    uint64_t env_stride;   /* bytes between envs in ids/light */
    uint32_t num_envs, width, height, depth;
} blk_world_views;

typedef struct blk_ctx blk_ctx;

/* Context lifetime. Replaces the reference's WorldGenerator constructor /
 * destructor (src/world/WorldGenerator.h:69-72, src/world/WorldGenerator.cu:594-619);
 * allocates the resident world arrays for `num_envs` regions. */
int blk_ctx_create(int device, const blk_world_config* config, blk_ctx** out);
int blk_ctx_destroy(blk_ctx* ctx);

/* Message of the last failure on this thread ("" if none). */
const char* blk_last_error(void);

/* Device pointers of the resident world arrays (valid until destroy). */
int blk_views(blk_ctx* ctx, blk_world_views* out);

/* Full generation + light of every env: terrain from env_seeds[num_envs],
 * sparse overrides applied (at most one per cell; with duplicates the
 * latest in list order wins), height map, sky column fill, block and sky
 * flood fill. Replaces WorldGenerator::generate
 * (src/world/WorldGenerator.h:79-82, src/world/WorldGenerator.cu:673-829) for
 * a whole batch at once. env_origins, when not NULL, holds num_envs * 3
 * int32 (x, y, z): the world coordinates of each env's region corner, which
 * the reference sets per call to the agent's block minus the half extent
 * (src/world/WorldGenerator.cpp:13-21); the origins stay until the next call
 * that gives them. NULL keeps every env's current origin (initially the
 * configuration's). Override, edit and query coordinates are world
 * coordinates; overrides outside their env's region are ignored. */
int blk_generate(blk_ctx* ctx, const uint32_t* env_seeds, const int32_t* env_origins, const blk_override* overrides,
    uint32_t n_overrides, uintptr_t stream);

/* Regenerates and relights only the envs listed in env_ids[n_envs] (distinct
 * indices; out-of-range ones are skipped and reported by blk_sync), with
 * seeds env_seeds[n_envs], origins env_origins[n_envs * 3] (NULL keeps their
 * current origins) and the overrides of those envs (records of other envs are
 * ignored); every other env keeps its state. The batched per-env reset the
 * reference leaves for later (include/blocklab/environment/Environment.h:33),
 * and the regeneration of an env whose agent left its cached region
 * (src/graphics/Renderer.cpp:1115-1141); requires a prior blk_generate. Arrays
 * may be host or device memory. */
int blk_generate_envs(blk_ctx* ctx, const uint32_t* env_ids, uint32_t n_envs, const uint32_t* env_seeds,
    const int32_t* env_origins, const blk_override* overrides, uint32_t n_overrides, uintptr_t stream);

/* Writes up to `per_env` torch overrides per env at distinct pseudo-random
 * columns, one cell above the terrain surface (benchmark world construction).
 * `out` is device memory of num_envs*per_env entries; *out_count (device)
 * receives the number written. Keyed by env_seeds (host or device). */
int blk_place_torches(blk_ctx* ctx, const uint32_t* env_seeds, uint32_t per_env, blk_override* out,
    uint32_t* out_count, uintptr_t stream);

/* Applies edits with World::setBlock semantics (src/world/World.cpp:239-287),
 * sequentially per env in list order, then relights exactly the cells whose
 * light can change. The reference instead regenerates and relights the whole
 * region on any edit (src/graphics/Renderer.cpp:1121-1141). */
int blk_apply_edits(blk_ctx* ctx, const blk_override* edits, uint32_t n_edits, uintptr_t stream);

/* Render voxel list of one env in the reference's 12-byte Voxel format and
 * TerrainHeader (src/world/WorldGenerator.cu:27-67, :171-178, :221-303;
 * shaders/voxel.vert.hlsl:14-24). Voxels are written in ascending
 * (z, y, x) order. `voxels`, `count` and `header` are device memory. The
 * packing holds x, z < 64 and y < 512, as in the reference. The header holds
 * the env's current origin. */
int blk_build_render_voxels(blk_ctx* ctx, uint32_t env, void* voxels, uint32_t max_voxels, uint32_t* count,
    int32_t* header, uintptr_t stream);

/* No counterpart in the reference (an addition of this library). The render
 * voxel list of blk_build_render_voxels for one world held in caller-owned
 * device memory (ids and light of one env in this library's layout,
 * [depth][width][height] with height fastest, e.g. a blk_views env slice),
 * without allocating anything: the row scratch is a fixed device array of
 * 2 x 32768 words inside the library. For callers that cannot allocate
 * device memory at call time, e.g. a renderer recording its frame work.
 * Limits: width, depth <= 64 and height <= 512 (the reference packing) and
 * depth * height <= 32768 rows; larger regions return BLK_ERR_CAPACITY.
 * The world must live on the current device (its scratch is used; another
 * device's world returns BLK_ERR_INVALID_ARGUMENT). Each call outside a stream
 * capture looks up the scratch array's device address with that device
 * current (a query that allocates nothing, so it stays right across a
 * cudaDeviceReset); a call inside a capture reuses the address of the
 * device's last call outside one, so the first call on a device must come
 * before any stream capture. Nothing has to start at zero. All calls on a
 * device share the scratch: calls that overlap in time (other streams or host
 * threads) race, so order them. `voxels`, `count` and `header` are device
 * memory. */
int blk_build_render_voxels_static(const uint8_t* ids, const uint8_t* light, uint32_t width, uint32_t height,
    uint32_t depth, int32_t origin_x, int32_t origin_y, int32_t origin_z, void* voxels, uint32_t max_voxels,
    uint32_t* count, int32_t* header, uintptr_t stream);

/* Day/night effective light: out[i] = (sky - min(sky, dimming[env])) << 4 | block
 * for every cell, dimming = 15 - skyLightAtTime(t) as the reference renderer
 * applies it per face (src/graphics/Renderer.cpp:803, shaders/voxel.vert.hlsl:151).
 * `dimming` holds num_envs bytes; `out` is device memory shaped like light. */
int blk_effective_light(blk_ctx* ctx, const uint8_t* dimming, uint8_t* out, uintptr_t stream);

/* Integer sky level at a day tick (src/world/Lighting.cpp:21-49). Host only. */
uint8_t blk_sky_light_at_time(uint32_t tick);

/* Sparse queries of the resident worlds. They replace the reference's copy of
 * the whole block cache to the host after every generation
 * (src/world/WorldGenerator.cu:798-815, src/world/World.cpp:149-183), which its
 * physics then reads through World::block (src/world/World.cpp:221-231),
 * World::terrainHeight (src/world/World.h:56, src/world/World.cpp:67-78) and
 * World::hasSolidBlockInArea (src/world/World.cpp:289-307). Queries use world
 * coordinates; queries and outputs are device memory. */
typedef struct blk_cell_query {
    int32_t x, y, z;
    uint32_t env;
} blk_cell_query;

typedef struct blk_box_query {
    int32_t min_x, min_y, min_z;
    int32_t max_x, max_y, max_z; /* inclusive */
    uint32_t env;
    uint32_t reserved;
} blk_box_query;

/* Per query i: out_block[i] = block id, or 255 outside the region (where
 * World::block returns null); out_light[i] = sky << 4 | block light, 0 outside;
 * out_height[i] = world y of the highest solid block of column (x, z), or
 * INT32_MIN when the column is outside the region. Any output may be NULL. */
int blk_query_cells(blk_ctx* ctx, const blk_cell_query* queries, uint32_t n, uint8_t* out_block, uint8_t* out_light,
    int32_t* out_height, uintptr_t stream);

/* out_solid[i] = 1 if the box of query i, clipped to the region, holds a solid
 * (opaque) block, else 0 (World::hasSolidBlockInArea). */
int blk_query_solid(blk_ctx* ctx, const blk_box_query* queries, uint32_t n, uint8_t* out_solid, uintptr_t stream);

/* Snapshot of one env's overlay: every cell whose block differs from the
 * generated terrain, as blk_override records (world coordinates, env = `env`),
 * in ascending (z, x, y) order. blk_generate with the env's seed and these
 * overrides rebuilds the same world (ids, light, height map). The reference
 * keeps the overlay as World's override columns (src/world/World.h:143,
 * src/world/World.cpp:239-287). `out` (capacity entries) and `count` are device
 * memory; *count receives the full size even when it exceeds the capacity. */
int blk_snapshot_overrides(blk_ctx* ctx, uint32_t env, blk_override* out, uint32_t capacity, uint32_t* count,
    uintptr_t stream);

/* Camera and sky of one env's frame: the reference's RenderParams
 * (shaders/render_params.hlsl, filled by Renderer::buildRenderParams,
 * src/graphics/Renderer.cpp:773-808) without the viewport and frame fields. */
typedef struct blk_render_params {
    float origin[3];   /* eye position, world coordinates */
    float forward[3];  /* unit view direction */
    float right[3];
    float up[3];
    float far_plane;   /* 48 in the reference */
    float fov_radians; /* vertical field of view, pi / 2.25 in the reference */
    float fog_start, fog_end;
    float sky_color[3];
    uint32_t sky_light_dimming; /* 15 - skyLightAtTime(t) */
    float sky_light_direction[3];
    uint32_t reserved;
} blk_render_params;

/* Render parameters of an agent standing at (x, y, z) (feet) looking along
 * yaw / pitch (radians) at day tick `tick` (0..23999): eye 1.62 above the
 * feet, the reference's projection and fog constants, sky colour, light
 * direction and dimming at that tick (src/graphics/Renderer.cpp:76-80,773-808;
 * src/world/Lighting.cpp:53-118). Host only. */
void blk_render_params_at(float x, float y, float z, float yaw, float pitch, uint32_t tick, blk_render_params* out);

/* Frames of every env, RGBA8 sRGB, shape (num_envs, height, width, 4): the
 * first face along each pixel's view ray, shaded as the reference's voxel
 * pipeline shades it (shaders/voxel.vert.hlsl:110-158, shaders/lighting.hlsl,
 * shaders/mesh.frag.hlsl:12-82, shaders/fog.hlsl), sky colour where no face
 * lies within the far plane. Only the world region is drawn (no mobs, drops
 * or held items). `params` holds num_envs entries (host or device memory);
 * `out_rgba` is device memory. */
int blk_render_frames(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height,
    uint8_t* out_rgba, uintptr_t stream);

/* The same frames written straight into the float32 NCHW observation tensor
 * (num_envs, 3, height, width), equal to blk_convert_rgba8_to_float_nchw of
 * the RGBA8 frames (src/environment/CudaObservation.cu:13-44) without the
 * round trip through them; `out_rgba` may also be given (else NULL). Both are
 * device memory. */
int blk_render_observations(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height,
    float* out_nchw, uint8_t* out_rgba, uintptr_t stream);

/* Copies env range [env_begin, env_begin + n_envs) of the world arrays to
 * caller memory in the device layout (any of the outputs may be NULL).
 * Replaces the per-generation cache readback (src/world/WorldGenerator.cu:798-815). */
int blk_readback(blk_ctx* ctx, uint32_t env_begin, uint32_t n_envs, uint8_t* ids, uint8_t* light,
    int16_t* height_map, uintptr_t stream);

/* Waits for `stream` and reports any device-side flag raised since the last
 * call (BLK_ERR_DEVICE_FLAG with a message). */
int blk_sync(blk_ctx* ctx, uintptr_t stream);

/* Per-phase device timing (CUDA events recorded on the call's own stream
 * around each phase while enabled). The reference has no tracing of its own;
 * this replaces ad-hoc timing of its benchmark (src/app/benchmark.cpp:341-377). */
typedef struct blk_profile {
    double generate_prep_ms;  /* override column-CSR build of blk_generate */
    double generate_tiles_ms; /* fused generation + light tile kernel */
    double edits_prep_ms;     /* edit grouping + setBlock application */
    double relight_ms;        /* dirty-window compaction + relight tile kernel */
    uint64_t generate_calls;
    uint64_t edit_calls;
} blk_profile;

int blk_profile_enable(blk_ctx* ctx, int enable);
/* Waits for the recorded events and returns the accumulated times; reset != 0
 * clears the accumulators afterwards. */
int blk_profile_read(blk_ctx* ctx, blk_profile* out, int reset);

/* Generation path. BLK_GENERATION_SURFACE generates each tile with the surface
 * kernel, which lights one 32-row word per column starting at the column's
 * first open row, and hands the tiles it cannot prove exact (caves, overhangs,
 * tall light, steep steps between columns) to the tile kernel;
 * BLK_GENERATION_TILES runs the tile kernel on every tile. BLK_GENERATION_AUTO
 * (the default) takes the tile kernel for steep fBm terrain (amplitude above
 * 80, where most tiles would be handed over) and the surface kernel otherwise.
 * All give the same worlds. No counterpart in the reference, whose generator
 * has one path (src/world/WorldGenerator.cu:673-829). */
typedef enum blk_generation_path {
    BLK_GENERATION_SURFACE = 0,
    BLK_GENERATION_TILES = 1,
    BLK_GENERATION_AUTO = 2
} blk_generation_path;

int blk_set_generation_path(blk_ctx* ctx, int path);
/* Number of tiles of the last blk_generate / blk_generate_envs that the surface
 * kernel left to the tile kernel (waits for the context's device). */
int blk_generation_fallback_tiles(blk_ctx* ctx, uint32_t* count);

/* RGBA8 -> float32 NCHW with the alpha channel dropped, value * (1.0f/255.0f).
 * Same signature and meaning as the reference's convertRgba8ToFloatNchw
 * (src/environment/CudaObservation.h:7-8); both pointers are device memory.
 * Returns a status instead of aborting. */
int blk_convert_rgba8_to_float_nchw(const void* rgba8, float* nchw, uint32_t batch, uint32_t width, uint32_t height,
    uintptr_t stream);

#ifdef __cplusplus
}
#endif

#endif /* BLK_WORLD_H */
