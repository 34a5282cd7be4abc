// Internal context and launch declarations of libblk_world.so.
#pragma once

#include "../../include/blk_world.h"
#include "blk_common.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>
#include <vector>

// Size classes of the region relight kernels (blk_relight.cu): one item list,
// side stream and scratch area each.
constexpr int kRegionLists = 6;

struct blk_ctx {
    int device = 0;
    blk_world_config cfg {};
    uint32_t tiles_x = 0, tiles_z = 0;
    uint64_t columns_per_env = 0;
    uint64_t env_stride = 0;          // bytes per env in ids / light

    uint8_t* ids = nullptr;           // [env][z][x][y]
    uint8_t* light = nullptr;         // [env][z][x][y], sky<<4 | block
    int16_t* hmap = nullptr;          // [env][z][x], world y

    uint32_t* seeds = nullptr;        // [env]
    int4* origins = nullptr;          // [env] world coordinates of each env's local (0, 0, 0); w unused
    int32_t* origin_stage = nullptr;  // [env * 3] staging of host-resident origin lists
    int16_t* terrain_top = nullptr;   // [env][z][x] local terrain surface, clamped to [-1, H+4]
    uint16_t* halo_order = nullptr;   // halo columns of a tile by cone distance
    bool generated = false;

    // Override column CSR (generation input).
    blk_override* ovr = nullptr;      // staging of host-resident override lists
    uint32_t* col_count = nullptr;    // [env * columns + 1]
    bool counts_zero = false;         // col_count is all zero (a generation's scatter leaves it so)
    uint32_t* col_offset = nullptr;   // [env * columns + 1]
    uint64_t* entries = nullptr;      // [max_overrides], key y<<40 | order<<8 | block
    uint8_t* ovr_owner = nullptr;     // [max_overrides], 1 for the override owning its column segment
    uint4* col_summary = nullptr;     // [env * columns] generation column summaries (see column_summary_kernel)
    uint8_t* env_mask = nullptr;      // [num_envs] envs of a partial reset
    uint32_t* env_list = nullptr;     // [num_envs] staging of a partial reset's env ids
    uint32_t* seed_list = nullptr;    // [num_envs] staging of a partial reset's seeds
    uint32_t* scan_partials = nullptr;
    uint64_t scan_blocks = 0;

    // Edits (incremental relight).
    blk_override* edits = nullptr;        // staging of host-resident edit lists
    uint32_t* edit_env_count = nullptr;   // [num_envs + 1]
    uint32_t* edit_env_offset = nullptr;  // [num_envs + 1]
    uint32_t* edit_order = nullptr;       // [max_edits] edit indices grouped by env, stable
    uint4* edit_changes = nullptr;        // [2 * max_edits] cells each edit changed (see apply_edits_kernel)
    uint32_t* dirty_window = nullptr;     // [num_envs * tiles] packed ylo | yhi<<16, 0xFFFFFFFF = clean
    uint32_t* dirty_list = nullptr;       // [num_envs * tiles] dirty tile ids
    uint32_t* dirty_count = nullptr;      // [1]
    uint4* region_lists = nullptr;        // [kRegionLists][region_capacity][2] relight items by size class (see blk_relight.cu)
    uint32_t region_capacity = 0;         // items per list, and footprint centres of all items
    uint32_t* region_centres = nullptr;   // [region_capacity] footprint centres of the items (x | z << 16)
    uint32_t* region_counts = nullptr;    // [kRegionLists + 1]: items per list, then centres used
    cudaStream_t relight_streams[kRegionLists] = {}; // side streams of the region kernels (forked from the caller's stream)
    cudaEvent_t relight_fork = nullptr;
    cudaEvent_t relight_join[kRegionLists] = {};
    uint32_t box_capacity = 0;            // 2 * max_edits (an edit changes at most two cells)
    uint32_t* h_dirty_count = nullptr;    // pinned [1]

    // Generation: the surface kernel's tiles left to the tile kernel.
    uint32_t* fallback_list = nullptr;    // [num_envs * tiles] tile ids
    uint32_t* fallback_count = nullptr;   // [2]: their number, then the surface kernel's tile cursor
    int generation_path = BLK_GENERATION_AUTO;

    uint32_t* park = nullptr;             // tile-kernel scratch: 16 words x 1024 threads per CTA
    uint32_t park_ctas = 0;
    blk_render_params* render_params = nullptr; // [num_envs] staging of host-resident render parameters
    uint32_t* flags = nullptr;            // device error flag word
    uint32_t* h_flags = nullptr;          // pinned mirror

    // Phase timing (blk_profile_*): event triples (start, mid, end) per call.
    bool profiling = false;
    struct Mark {
        cudaEvent_t e[3];
        int kind; // 0 generate, 1 edits
    };
    std::vector<Mark> marks;
    blk_profile prof {};
};

namespace blk {

// Region relight (blk_relight.cu): inputs of the per-env region build.
struct RegionBuildArgs {
    const uint4* changes;       // change records of the edit step (two per env-grouped edit position)
    const uint32_t* env_offset; // [num_envs + 1] edit positions per env
    uint32_t num_envs;
    int32_t W, H, D;
    uint4* lists[kRegionLists]; // relight item lists by size class, two uint4 per item
    uint32_t* counts;           // [kRegionLists + 1]: items per list, then centres used
    uint32_t capacity;          // entries per list, and of the centre array
    uint32_t* centres;          // footprint centres of the items (x | z << 16)
    uint32_t* win_lo;           // tile path: per env tile dirty rows (atomicMin / atomicMax)
    uint32_t* win_hi;
    int32_t tiles_x, tiles_z;
    uint32_t* flags;
};

struct RegionRelightArgs {
    const uint8_t* ids;
    uint8_t* light;
    const int16_t* hmap;
    const int4* origins;
    int32_t W, H, D;
    uint64_t env_stride;
    uint64_t columns;           // per env
    const uint4* regions;       // this kernel's item list (two uint4 per item) and its count
    const uint32_t* count;
    uint32_t capacity;
    const uint32_t* centres;    // footprint centres (x | z << 16) the items point into
    uint32_t* flags;
};

int launch_region_build(blk_ctx* ctx, const RegionBuildArgs& a, cudaStream_t stream);
int launch_region_relight(blk_ctx* ctx, const cudaStream_t (&side)[kRegionLists]);

void set_error(const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

// Copies `bytes` from host or device memory `src` into the device buffer
// `staging` (when src is host memory) and returns the device pointer to use.
bool device_memory(const void* p);
int stage_input(const void* src, size_t bytes, void* staging, cudaStream_t stream, const void** out);

TerrainParams terrain_params(const blk_ctx* ctx);

int launch_relight(blk_ctx* ctx, cudaStream_t stream);
// env_mask (device, one byte per env) restricts the work to the envs set in it; nullptr = all.
int launch_terrain(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask = nullptr);
int launch_column_summary(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask = nullptr);
// Terrain surfaces plus generation column summaries; needs the override CSR.
int launch_surface(blk_ctx* ctx, cudaStream_t stream, const uint8_t* env_mask = nullptr);
// Mode 0 over a tile list (ctx->dirty_list, n_tiles entries, 0xFFFFFFFF = skip) when `listed`.
int launch_tiles(blk_ctx* ctx, int mode, uint32_t n_tiles, cudaStream_t stream, bool listed = false);
// Generation of all tiles (or the listed ones) on ctx->generation_path: the
// surface kernel, then the tile kernel over the tiles it left.
int launch_generation(blk_ctx* ctx, uint32_t n_tiles, cudaStream_t stream, bool listed = false);
// The path launch_generation takes (BLK_GENERATION_SURFACE or BLK_GENERATION_TILES).
int generation_path_of(const blk_ctx* ctx);
int launch_render(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height, uint8_t* out,
    float* out_nchw, cudaStream_t stream);
void halo_order_table(uint16_t* out);
int halo_order_size();

// Phase marks for blk_profile: begin() returns a mark index or -1 when off.
int prof_begin(blk_ctx* ctx, int kind, cudaStream_t stream);
void prof_mark(blk_ctx* ctx, int mark, int which, cudaStream_t stream);

} // namespace blk
