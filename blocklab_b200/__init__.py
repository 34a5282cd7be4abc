"""B200-native world-state hot path of the BlockLab environment.

Generation over the sparse override overlay, sky column fill, 6-neighbour
flood-fill block/sky light with exact incremental relight, render voxel list,
day/night effective light and the RGBA8 -> float32 NCHW observation
conversion, as hand-written sm_100a CUDA behind a C ABI (include/blk_world.h).
"""
from ._native import (AIR, DIRT, EDIT_REMOVE_TORCH, EDIT_SET, GRASS, STONE, TERRAIN_FBM, TERRAIN_FLAT,
                      TERRAIN_REFERENCE, TORCH, BlkError)
from .observation import convert_rgba8_to_float_nchw
from .world import (BOX_QUERY_DTYPE, CELL_QUERY_DTYPE, OVERRIDE_DTYPE, RENDER_PARAMS_DTYPE, WorldBatch, WorldConfig,
                    load_snapshot, make_overrides, render_params_at, save_snapshot, sky_light_at_time,
                    sky_light_dimming, torch_key)

__all__ = [
    "AIR", "GRASS", "DIRT", "STONE", "TORCH", "EDIT_SET", "EDIT_REMOVE_TORCH", "TERRAIN_REFERENCE", "TERRAIN_FBM",
    "TERRAIN_FLAT", "BlkError", "convert_rgba8_to_float_nchw", "OVERRIDE_DTYPE", "WorldBatch", "WorldConfig",
    "make_overrides", "sky_light_at_time", "sky_light_dimming", "torch_key", "CELL_QUERY_DTYPE", "BOX_QUERY_DTYPE",
    "save_snapshot", "load_snapshot", "RENDER_PARAMS_DTYPE", "render_params_at",
]
