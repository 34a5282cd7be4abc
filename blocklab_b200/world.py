"""Host-side mirror of the reference's world-state interface over the C ABI.

``WorldBatch`` plays the role of the reference's ``WorldGenerator``
(src/world/WorldGenerator.h:69-89) for a whole batch of environments on one
GPU: it owns the resident block-id / light / height-map arrays and enqueues
generation, edits with incremental relight, the render voxel list and the
day/night effective light on the caller's CUDA stream. ``World``-level edit
semantics (src/world/World.cpp:239-287) are applied on the device by
``apply_edits``.

Device arrays are exposed zero-copy as torch tensors:
    ids, light   (num_envs, D, W, H) uint8   — column-major, y fastest
    height_map   (num_envs, D, W)    int16   — world y of the top solid block
    origins      (num_envs, 4)       int32   — x, y, z of each env's region
                                               corner (world coordinates), 0
``light`` packs sky << 4 | block. Every env has its own region origin, set by
``generate`` / ``generate_envs`` (the reference centres the region on the
agent on every generation, src/world/WorldGenerator.cpp:13-21).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _native as N
from ._native import check

OVERRIDE_DTYPE = np.dtype([("x", "<i4"), ("y", "<i4"), ("z", "<i4"), ("env", "<u2"), ("block", "u1"),
                           ("kind", "u1")])
assert OVERRIDE_DTYPE.itemsize == 16


@dataclass(frozen=True)
class WorldConfig:
    num_envs: int
    width: int
    height: int
    depth: int
    origin: tuple[int, int, int] = (0, 0, 0)
    terrain: int = N.TERRAIN_FBM
    base: int = 40
    amplitude: float = 50.0
    max_overrides: int = 1 << 20
    max_edits: int = 1 << 16

    def to_c(self) -> N.WorldConfigC:
        return N.WorldConfigC(self.num_envs, self.width, self.height, self.depth, self.origin[0], self.origin[1],
                              self.origin[2], self.terrain, self.base, float(self.amplitude), self.max_overrides,
                              self.max_edits)

    @property
    def voxels_per_env(self) -> int:
        return self.width * self.height * self.depth


def make_overrides(xyz, block, env=0, kind=0) -> np.ndarray:
    """Packs override / edit records (world coordinates) into the C layout."""
    xyz = np.asarray(xyz, np.int32).reshape(-1, 3)
    out = np.zeros(len(xyz), OVERRIDE_DTYPE)
    out["x"], out["y"], out["z"] = xyz[:, 0], xyz[:, 1], xyz[:, 2]
    out["env"] = np.broadcast_to(np.asarray(env, np.uint16), len(xyz))
    out["block"] = np.broadcast_to(np.asarray(block, np.uint8), len(xyz))
    out["kind"] = np.broadcast_to(np.asarray(kind, np.uint8), len(xyz))
    return out


class _CudaArray:
    """__cuda_array_interface__ over memory owned by a WorldBatch."""

    def __init__(self, owner, ptr: int, shape, typestr: str) -> None:
        self._owner = owner
        self.__cuda_array_interface__ = {"data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
                                         "strides": None, "version": 3, "stream": None}


def _stream_handle(stream: Optional[torch.cuda.Stream], device: int) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return int(s.cuda_stream)


def _origins_ptr(origins, n: int):
    """(pointer, keep-alive) of an (n, 3) int32 origin list, or (None, None)."""
    if origins is None:
        return None, None
    if isinstance(origins, torch.Tensor):
        if origins.dtype != torch.int32 or origins.shape != (n, 3):
            raise ValueError(f"origins must be an ({n}, 3) int32 tensor")
        return _ptr(origins)
    arr = np.ascontiguousarray(np.asarray(origins, np.int64).reshape(-1, 3), np.int32)
    if arr.shape != (n, 3):
        raise ValueError(f"origins must be ({n}, 3)")
    return _ptr(arr)


def _ptr(obj) -> tuple[int, object]:
    """Pointer + keep-alive for a numpy array or torch tensor (host or device)."""
    if isinstance(obj, torch.Tensor):
        if not obj.is_contiguous():
            obj = obj.contiguous()
        return obj.data_ptr(), obj
    arr = np.ascontiguousarray(obj)
    return arr.ctypes.data, arr


class WorldBatch:
    """A batch of resident worlds on one GPU (one blk_ctx)."""

    def __init__(self, config: WorldConfig, device: int = 0) -> None:
        if not torch.cuda.is_available():
            raise RuntimeError("WorldBatch needs a CUDA device; the world-state path has no CPU implementation")
        self.config = config
        self.device = device
        handle = ctypes.c_void_p()
        c = config.to_c()
        check(N.lib.blk_ctx_create(device, ctypes.byref(c), ctypes.byref(handle)))
        self._ctx = handle
        v = N.WorldViewsC()
        check(N.lib.blk_views(self._ctx, ctypes.byref(v)))
        dev = torch.device("cuda", device)
        E, D, W, H = config.num_envs, config.depth, config.width, config.height
        self.ids = torch.as_tensor(_CudaArray(self, v.ids, (E, D, W, H), "|u1"), device=dev)
        self.light = torch.as_tensor(_CudaArray(self, v.light, (E, D, W, H), "|u1"), device=dev)
        self.height_map = torch.as_tensor(_CudaArray(self, v.height_map, (E, D, W), "<i2"), device=dev)
        self.origins = torch.as_tensor(_CudaArray(self, v.env_origins, (E, 4), "<i4"), device=dev)

    # -- lifetime -------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_ctx", None):
            N.lib.blk_ctx_destroy(self._ctx)
            self._ctx = None

    def __del__(self) -> None:  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    # -- the hot path -----------------------------------------------------------
    def generate(self, env_seeds, overrides=None, origins=None, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Full generation + light of every env (reference WorldGenerator::generate).
        ``origins`` (num_envs, 3) int32 world coordinates of each env's region
        corner; None keeps the current ones."""
        seeds_p, keep1 = _ptr(np.asarray(env_seeds, np.uint32) if not isinstance(env_seeds, torch.Tensor)
                              else env_seeds)
        org_p, keep_o = _origins_ptr(origins, self.config.num_envs)
        if overrides is None:
            ovr_p, n, keep2 = 0, 0, None
        elif isinstance(overrides, torch.Tensor):
            ovr_p, keep2 = _ptr(overrides)
            n = overrides.numel() * overrides.element_size() // 16
        else:
            arr = np.ascontiguousarray(overrides, OVERRIDE_DTYPE)
            ovr_p, keep2 = _ptr(arr)
            n = len(arr)
        check(N.lib.blk_generate(self._ctx, seeds_p, org_p, ovr_p, n, _stream_handle(stream, self.device)))
        del keep1, keep2, keep_o

    def generate_envs(self, env_ids, env_seeds, overrides=None, origins=None,
                      stream: Optional[torch.cuda.Stream] = None) -> None:
        """Regenerates only the listed envs (distinct indices) with their seeds,
        overrides and, when given, new region origins (len(env_ids), 3); the
        other envs keep their state."""
        ids_p, keep1 = _ptr(np.asarray(env_ids, np.uint32) if not isinstance(env_ids, torch.Tensor) else env_ids)
        seeds_p, keep2 = _ptr(np.asarray(env_seeds, np.uint32) if not isinstance(env_seeds, torch.Tensor)
                              else env_seeds)
        n_envs = len(env_ids)
        if len(env_seeds) != n_envs:
            raise ValueError("one seed per listed env")
        org_p, keep_o = _origins_ptr(origins, n_envs)
        if overrides is None:
            ovr_p, n, keep3 = 0, 0, None
        elif isinstance(overrides, torch.Tensor):
            ovr_p, keep3 = _ptr(overrides)
            n = overrides.numel() * overrides.element_size() // 16
        else:
            arr = np.ascontiguousarray(overrides, OVERRIDE_DTYPE)
            ovr_p, keep3 = _ptr(arr)
            n = len(arr)
        check(N.lib.blk_generate_envs(self._ctx, ids_p, n_envs, seeds_p, org_p, ovr_p, n,
                                      _stream_handle(stream, self.device)))
        del keep1, keep2, keep3, keep_o

    def place_torches(self, env_seeds, per_env: int, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Device override list of `per_env` torches per env on the terrain surface."""
        n = self.config.num_envs * per_env
        out = torch.empty(max(n, 1) * 16, dtype=torch.uint8, device=torch.device("cuda", self.device))
        cnt = torch.zeros(1, dtype=torch.int32, device=out.device)
        seeds_p, keep = _ptr(np.asarray(env_seeds, np.uint32) if not isinstance(env_seeds, torch.Tensor)
                             else env_seeds)
        check(N.lib.blk_place_torches(self._ctx, seeds_p, per_env, out.data_ptr(), cnt.data_ptr(),
                                      _stream_handle(stream, self.device)))
        del keep
        return out[: n * 16]

    def apply_edits(self, edits, stream: Optional[torch.cuda.Stream] = None) -> None:
        """World::setBlock semantics per env in list order + exact incremental relight."""
        if isinstance(edits, torch.Tensor):
            p, keep = _ptr(edits)
            n = edits.numel() * edits.element_size() // 16
        else:
            arr = np.ascontiguousarray(edits, OVERRIDE_DTYPE)
            p, keep = _ptr(arr)
            n = len(arr)
        check(N.lib.blk_apply_edits(self._ctx, p, n, _stream_handle(stream, self.device)))
        del keep

    def render_voxels(self, env: int, max_voxels: Optional[int] = None,
                      stream: Optional[torch.cuda.Stream] = None) -> tuple[torch.Tensor, int, tuple[int, int, int]]:
        """Reference 12-byte Voxel list of one env, ascending (z, y, x) order."""
        cap = self.config.voxels_per_env if max_voxels is None else max_voxels
        dev = torch.device("cuda", self.device)
        vox = torch.empty((max(cap, 1), 3), dtype=torch.int32, device=dev)
        cnt = torch.zeros(1, dtype=torch.int32, device=dev)
        hdr = torch.zeros(3, dtype=torch.int32, device=dev)
        check(N.lib.blk_build_render_voxels(self._ctx, env, vox.data_ptr(), cap, cnt.data_ptr(), hdr.data_ptr(),
                                            _stream_handle(stream, self.device)))
        n = int(cnt.item())
        return vox[: min(n, cap)], n, tuple(int(v) for v in hdr.tolist())

    def query_cells(self, xyz, env=0, stream: Optional[torch.cuda.Stream] = None):
        """Block id (255 outside the region), light byte and column height (world
        y, INT32_MIN outside) of world cells xyz (N, 3); env scalar or (N,)."""
        q = _queries(CELL_QUERY_DTYPE, xyz, env, ("x", "y", "z"))
        dev = torch.device("cuda", self.device)
        qd = torch.from_numpy(q.view(np.uint8)).to(dev)
        n = len(q)
        block = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
        light = torch.empty(max(n, 1), dtype=torch.uint8, device=dev)
        height = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
        check(N.lib.blk_query_cells(self._ctx, qd.data_ptr(), n, block.data_ptr(), light.data_ptr(), height.data_ptr(),
                                    _stream_handle(stream, self.device)))
        return block[:n], light[:n], height[:n]

    def query_solid(self, box_min, box_max, env=0, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """1 where the inclusive world box [box_min, box_max] (N, 3), clipped to
        the region, holds a solid block (World::hasSolidBlockInArea)."""
        box_min, box_max = np.asarray(box_min, np.int64).reshape(-1, 3), np.asarray(box_max, np.int64).reshape(-1, 3)
        q = np.zeros(len(box_min), BOX_QUERY_DTYPE)
        for k, name in enumerate(("x", "y", "z")):
            q["min_" + name] = box_min[:, k]
            q["max_" + name] = box_max[:, k]
        q["env"] = env
        dev = torch.device("cuda", self.device)
        qd = torch.from_numpy(q.view(np.uint8)).to(dev)
        out = torch.empty(max(len(q), 1), dtype=torch.uint8, device=dev)
        check(N.lib.blk_query_solid(self._ctx, qd.data_ptr(), len(q), out.data_ptr(),
                                    _stream_handle(stream, self.device)))
        return out[: len(q)]

    def render(self, params, width: int, height: int, out: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """RGBA8 sRGB frames (num_envs, height, width, 4) of every env from
        per-env render parameters (RENDER_PARAMS_DTYPE records)."""
        params = np.ascontiguousarray(params, RENDER_PARAMS_DTYPE).reshape(-1)
        if len(params) != self.config.num_envs:
            raise ValueError("one render parameter record per env")
        if out is None:
            out = torch.empty((self.config.num_envs, height, width, 4), dtype=torch.uint8,
                              device=torch.device("cuda", self.device))
        check(N.lib.blk_render_frames(self._ctx, params.ctypes.data, width, height, out.data_ptr(),
                                      _stream_handle(stream, self.device)))
        return out

    def render_observations(self, params, width: int, height: int, out: Optional[torch.Tensor] = None,
                            stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """Rendered frames written straight into a float32 (num_envs, 3, height,
        width) observation tensor (equal to converting the RGBA8 frames)."""
        params = np.ascontiguousarray(params, RENDER_PARAMS_DTYPE).reshape(-1)
        if len(params) != self.config.num_envs:
            raise ValueError("one render parameter record per env")
        if out is None:
            out = torch.empty((self.config.num_envs, 3, height, width), dtype=torch.float32,
                              device=torch.device("cuda", self.device))
        check(N.lib.blk_render_observations(self._ctx, params.ctypes.data, width, height, out.data_ptr(), None,
                                            _stream_handle(stream, self.device)))
        return out

    def snapshot(self, env: int, stream: Optional[torch.cuda.Stream] = None) -> np.ndarray:
        """Overlay of one env: the cells that differ from its terrain, as
        override records in (z, x, y) order; generate(seed, snapshot) rebuilds it."""
        dev = torch.device("cuda", self.device)
        cnt = torch.zeros(1, dtype=torch.int32, device=dev)
        cap = 1 << 16
        while True:
            out = torch.empty(cap * 16, dtype=torch.uint8, device=dev)
            check(N.lib.blk_snapshot_overrides(self._ctx, env, out.data_ptr(), cap, cnt.data_ptr(),
                                               _stream_handle(stream, self.device)))
            n = int(cnt.item())
            if n <= cap:
                return out[: n * 16].cpu().numpy().view(OVERRIDE_DTYPE).copy()
            cap = n

    def effective_light(self, dimming, out: Optional[torch.Tensor] = None,
                        stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        """(sky - min(sky, dimming[env])) << 4 | block for every cell."""
        if out is None:
            out = torch.empty_like(self.light)
        p, keep = _ptr(np.asarray(dimming, np.uint8) if not isinstance(dimming, torch.Tensor) else dimming)
        check(N.lib.blk_effective_light(self._ctx, p, out.data_ptr(), _stream_handle(stream, self.device)))
        del keep
        return out

    def set_generation_path(self, path: str) -> None:
        """'surface': the surface kernel, one light word per column, with the
        tile kernel for the tiles it cannot prove exact; 'tiles': the tile
        kernel for every tile; 'auto' (default): 'tiles' for steep fBm terrain
        (amplitude above 80), else 'surface'. All give the same worlds."""
        code = {"surface": 0, "tiles": 1, "auto": 2}[path]
        check(N.lib.blk_set_generation_path(self._ctx, code))

    def generation_fallback_tiles(self) -> int:
        """Tiles of the last generation left to the tile kernel (waits for the device)."""
        n = ctypes.c_uint32()
        check(N.lib.blk_generation_fallback_tiles(self._ctx, ctypes.byref(n)))
        return int(n.value)

    def profile(self, enable: bool) -> None:
        """Turns per-phase CUDA-event timing on or off (events on the call's stream)."""
        check(N.lib.blk_profile_enable(self._ctx, 1 if enable else 0))

    def profile_read(self, reset: bool = True) -> dict:
        p = N.ProfileC()
        check(N.lib.blk_profile_read(self._ctx, ctypes.byref(p), 1 if reset else 0))
        return {name: getattr(p, name) for name, _ in N.ProfileC._fields_}

    def sync(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Waits for the stream and raises if a kernel flagged an internal limit."""
        check(N.lib.blk_sync(self._ctx, _stream_handle(stream, self.device)))

    def readback(self, env_begin: int = 0, n_envs: Optional[int] = None, ids=True, light=True, height_map=True,
                 stream: Optional[torch.cuda.Stream] = None):
        """Copies env range to pinned host tensors (same layout as the device arrays)."""
        n = self.config.num_envs - env_begin if n_envs is None else n_envs
        c = self.config
        shp = (n, c.depth, c.width, c.height)
        out_ids = torch.empty(shp, dtype=torch.uint8, pin_memory=True) if ids else None
        out_light = torch.empty(shp, dtype=torch.uint8, pin_memory=True) if light else None
        out_hm = torch.empty((n, c.depth, c.width), dtype=torch.int16, pin_memory=True) if height_map else None
        check(N.lib.blk_readback(self._ctx, env_begin, n, out_ids.data_ptr() if ids else None,
                                 out_light.data_ptr() if light else None, out_hm.data_ptr() if height_map else None,
                                 _stream_handle(stream, self.device)))
        return out_ids, out_light, out_hm


CELL_QUERY_DTYPE = np.dtype([("x", "<i4"), ("y", "<i4"), ("z", "<i4"), ("env", "<u4")])
BOX_QUERY_DTYPE = np.dtype([("min_x", "<i4"), ("min_y", "<i4"), ("min_z", "<i4"), ("max_x", "<i4"), ("max_y", "<i4"),
                            ("max_z", "<i4"), ("env", "<u4"), ("reserved", "<u4")])


RENDER_PARAMS_DTYPE = np.dtype([("origin", "<f4", 3), ("forward", "<f4", 3), ("right", "<f4", 3), ("up", "<f4", 3),
                                ("far_plane", "<f4"), ("fov_radians", "<f4"), ("fog_start", "<f4"), ("fog_end", "<f4"),
                                ("sky_color", "<f4", 3), ("sky_light_dimming", "<u4"),
                                ("sky_light_direction", "<f4", 3), ("reserved", "<u4")])


def render_params_at(position, yaw: float, pitch: float, tick: int) -> np.ndarray:
    """blk_render_params of an agent with feet at `position` looking along
    yaw / pitch at day tick `tick` (Renderer::buildRenderParams)."""
    out = np.zeros(1, RENDER_PARAMS_DTYPE)
    x, y, z = (float(v) for v in position)
    N.lib.blk_render_params_at(x, y, z, float(yaw), float(pitch), int(tick) % 24000, out.ctypes.data)
    return out[0]


def _queries(dtype, xyz, env, names):
    xyz = np.asarray(xyz, np.int64).reshape(-1, 3)
    q = np.zeros(len(xyz), dtype)
    for k, name in enumerate(names):
        q[name] = xyz[:, k]
    q["env"] = env
    return q


def save_snapshot(path: str, seeds, overrides, tick: int = 0, config: Optional[WorldConfig] = None) -> None:
    """Writes a batch snapshot: per-env seeds, the overlay records of every env
    (WorldBatch.snapshot), the day tick and the region."""
    meta = {} if config is None else {k: getattr(config, k) for k in ("width", "height", "depth", "terrain", "base",
                                                                      "amplitude")}
    np.savez(path, seeds=np.asarray(seeds, np.uint32), overrides=np.asarray(overrides, OVERRIDE_DTYPE),
             tick=np.int64(tick), meta=np.array(repr(meta)))


def load_snapshot(path: str):
    """(seeds, overrides, tick) of a snapshot written by save_snapshot."""
    with np.load(path) as z:
        return z["seeds"], z["overrides"].view(OVERRIDE_DTYPE), int(z["tick"])


def sky_light_at_time(tick: int) -> int:
    """Integer sky level [4..15] at a day tick (src/world/Lighting.cpp:21-49)."""
    return int(N.lib.blk_sky_light_at_time(tick))


def sky_light_dimming(tick: int) -> int:
    """Renderer dimming uniform 15 - skyLightAtTime(t) (src/graphics/Renderer.cpp:803)."""
    return 15 - sky_light_at_time(tick)


def torch_key(seed: int) -> int:
    """Key of the torch-placement permutation for an env seed."""
    a, b = seed & 0xFFFFFFFF, 0x7F4A7C15
    a ^= (b + 0x9E3779B9 + ((a << 6) & 0xFFFFFFFF) + (a >> 2)) & 0xFFFFFFFF
    return a & 0xFFFFFFFF
