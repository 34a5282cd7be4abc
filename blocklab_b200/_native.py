"""ctypes binding of libblk_world.so (include/blk_world.h).

The shared library is the product: every compute call below goes to CUDA
kernels in it. If the library is missing or fails to load, importing this
module raises — there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libblk_world.so")

BLK_OK = 0
STATUS_NAMES = {
    0: "BLK_OK",
    1: "BLK_ERR_INVALID_ARGUMENT",
    2: "BLK_ERR_CUDA",
    3: "BLK_ERR_OUT_OF_MEMORY",
    4: "BLK_ERR_CAPACITY",
    5: "BLK_ERR_DEVICE_FLAG",
    6: "BLK_ERR_NOT_READY",
}

TERRAIN_REFERENCE, TERRAIN_FBM, TERRAIN_FLAT = 0, 1, 2
AIR, GRASS, DIRT, STONE, TORCH = 0, 1, 2, 3, 4
EDIT_SET, EDIT_REMOVE_TORCH = 0, 1


class BlkError(RuntimeError):
    """A non-zero status from the C ABI."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class WorldConfigC(ctypes.Structure):
    _fields_ = [
        ("num_envs", ctypes.c_uint32),
        ("width", ctypes.c_uint32),
        ("height", ctypes.c_uint32),
        ("depth", ctypes.c_uint32),
        ("origin_x", ctypes.c_int32),
        ("origin_y", ctypes.c_int32),
        ("origin_z", ctypes.c_int32),
        ("terrain_mode", ctypes.c_int32),
        ("fbm_base", ctypes.c_int32),
        ("fbm_amplitude", ctypes.c_float),
        ("max_overrides", ctypes.c_uint32),
        ("max_edits", ctypes.c_uint32),
    ]


class OverrideC(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_int32),
        ("y", ctypes.c_int32),
        ("z", ctypes.c_int32),
        ("env", ctypes.c_uint16),
        ("block", ctypes.c_uint8),
        ("kind", ctypes.c_uint8),
    ]


class WorldViewsC(ctypes.Structure):
    _fields_ = [
        ("ids", ctypes.c_void_p),
        ("light", ctypes.c_void_p),
        ("height_map", ctypes.c_void_p),
        ("env_origins", ctypes.c_void_p),
        ("env_stride", ctypes.c_uint64),
        ("num_envs", ctypes.c_uint32),
        ("width", ctypes.c_uint32),
        ("height", ctypes.c_uint32),
        ("depth", ctypes.c_uint32),
    ]


class ProfileC(ctypes.Structure):
    _fields_ = [
        ("generate_prep_ms", ctypes.c_double),
        ("generate_tiles_ms", ctypes.c_double),
        ("edits_prep_ms", ctypes.c_double),
        ("relight_ms", ctypes.c_double),
        ("generate_calls", ctypes.c_uint64),
        ("edit_calls", ctypes.c_uint64),
    ]


assert ctypes.sizeof(OverrideC) == 16

# Every symbol include/blk_world.h declares, with its ctypes signature.
_VP, _U32, _I32, _UP = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int32, ctypes.c_size_t
SIGNATURES = {
    "blk_ctx_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(WorldConfigC), ctypes.POINTER(ctypes.c_void_p)]),
    "blk_ctx_destroy": (ctypes.c_int, [_VP]),
    "blk_last_error": (ctypes.c_char_p, []),
    "blk_views": (ctypes.c_int, [_VP, ctypes.POINTER(WorldViewsC)]),
    "blk_generate": (ctypes.c_int, [_VP, _VP, _VP, _VP, _U32, _UP]),
    "blk_place_torches": (ctypes.c_int, [_VP, _VP, _U32, _VP, _VP, _UP]),
    "blk_apply_edits": (ctypes.c_int, [_VP, _VP, _U32, _UP]),
    "blk_build_render_voxels": (ctypes.c_int, [_VP, _U32, _VP, _U32, _VP, _VP, _UP]),
    "blk_build_render_voxels_static": (ctypes.c_int, [_VP, _VP, _U32, _U32, _U32, ctypes.c_int32, ctypes.c_int32,
                                                      ctypes.c_int32, _VP, _U32, _VP, _VP, _UP]),
    "blk_effective_light": (ctypes.c_int, [_VP, _VP, _VP, _UP]),
    "blk_sky_light_at_time": (ctypes.c_uint8, [_U32]),
    "blk_readback": (ctypes.c_int, [_VP, _U32, _U32, _VP, _VP, _VP, _UP]),
    "blk_sync": (ctypes.c_int, [_VP, _UP]),
    "blk_profile_enable": (ctypes.c_int, [_VP, ctypes.c_int]),
    "blk_profile_read": (ctypes.c_int, [_VP, ctypes.POINTER(ProfileC), ctypes.c_int]),
    "blk_convert_rgba8_to_float_nchw": (ctypes.c_int, [_VP, _VP, _U32, _U32, _U32, _UP]),
    "blk_query_cells": (ctypes.c_int, [_VP, _VP, _U32, _VP, _VP, _VP, _UP]),
    "blk_query_solid": (ctypes.c_int, [_VP, _VP, _U32, _VP, _UP]),
    "blk_snapshot_overrides": (ctypes.c_int, [_VP, _U32, _VP, _U32, _VP, _UP]),
    "blk_render_params_at": (None, [ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                    _U32, _VP]),
    "blk_render_frames": (ctypes.c_int, [_VP, _VP, _U32, _U32, _VP, _UP]),
    "blk_generate_envs": (ctypes.c_int, [_VP, _VP, _U32, _VP, _VP, _VP, _U32, _UP]),
    "blk_render_observations": (ctypes.c_int, [_VP, _VP, _U32, _U32, _VP, _VP, _UP]),
    "blk_set_generation_path": (ctypes.c_int, [_VP, ctypes.c_int]),
    "blk_generation_fallback_tiles": (ctypes.c_int, [_VP, _VP]),
}


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python blocklab_b200/build.py` (nvcc, sm_100a). "
            "There is no CPU fallback for the world-state path.")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = load()


def last_error() -> str:
    msg = lib.blk_last_error()
    return msg.decode() if msg else ""


def check(status: int) -> None:
    if status != BLK_OK:
        raise BlkError(status, last_error())
