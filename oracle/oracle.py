"""ctypes front end of the test oracle.

ORACLE — TEST INFRASTRUCTURE ONLY. Only tests/, ``__graft_entry__.smoke()``
and the CPU-baseline leg of ``bench.py`` import this module, and only as the
checker or the timed CPU baseline. The product package never imports it.

Two libraries sit behind it:

* ``oracle/liboracle.so`` — the plain C++ restatement (``blk_oracle.cpp``);
* ``oracle/_ref/libref_cpu.so`` / ``libref_cuda.so`` — the reference's own
  ``src/world/WorldGenerator.cu`` and ``src/environment/CudaObservation.cu``
  compiled from the reference sources by ``oracle/Makefile`` (CPU-fallback and
  sm_100a builds). They exist only where the reference was present at build
  time; callers check ``ref_available()``.

Arrays returned here use the reference layout: volumes ``(D, H, W)`` indexed
``[z, y, x]`` (src/world/WorldGenerator.cu:183), height maps ``(D, W)``.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_P = ctypes.c_void_p

AIR, GRASS, DIRT, STONE, TORCH = 0, 1, 2, 3, 4
TERRAIN_REFERENCE, TERRAIN_FBM, TERRAIN_FLAT = 0, 1, 2


class _Params(ctypes.Structure):
    _fields_ = [
        ("seed", ctypes.c_uint32),
        ("origin_x", ctypes.c_int32),
        ("origin_y", ctypes.c_int32),
        ("origin_z", ctypes.c_int32),
        ("width", ctypes.c_uint32),
        ("height", ctypes.c_uint32),
        ("depth", ctypes.c_uint32),
        ("terrain_mode", ctypes.c_int32),
        ("fbm_base", ctypes.c_int32),
        ("fbm_amplitude", ctypes.c_float),
    ]


@dataclass(frozen=True)
class WorldSpec:
    """One region: seed, origin (world coords of local 0,0,0), size, terrain."""

    seed: int
    width: int
    height: int
    depth: int
    origin: tuple[int, int, int] = (0, 0, 0)
    terrain: int = TERRAIN_FBM
    base: int = 40
    amplitude: float = 50.0

    def params(self) -> _Params:
        return _Params(self.seed & 0xFFFFFFFF, self.origin[0], self.origin[1], self.origin[2], self.width,
                       self.height, self.depth, self.terrain, self.base, self.amplitude)


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_P)


def _lib_path(name: str) -> str:
    return os.path.join(HERE, name)


def _load(path: str) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built; run `make -C oracle`")
    return ctypes.CDLL(path)


class Oracle:
    """The C++ restatement (liboracle.so)."""

    def __init__(self) -> None:
        self.lib = _load(_lib_path("liboracle.so"))
        L = self.lib
        L.orc_hash_combine2.restype = ctypes.c_uint32
        L.orc_hash_combine2.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.orc_hash_combine3.restype = ctypes.c_uint32
        L.orc_hash_combine3.argtypes = [ctypes.c_uint32] * 3
        L.orc_hash.restype = ctypes.c_uint32
        L.orc_hash.argtypes = [ctypes.c_uint32]
        L.orc_seed_offset.restype = ctypes.c_int32
        L.orc_seed_offset.argtypes = [ctypes.c_uint32, ctypes.c_uint32]
        L.orc_terrain_height.restype = ctypes.c_int32
        L.orc_terrain_height.argtypes = [ctypes.POINTER(_Params), ctypes.c_int32, ctypes.c_int32]
        L.orc_sky_light_at_time.restype = ctypes.c_uint8
        L.orc_sky_light_at_time.argtypes = [ctypes.c_uint32]
        L.orc_permute.restype = ctypes.c_uint32
        L.orc_permute.argtypes = [ctypes.c_uint32] * 3
        L.orc_place_torches.restype = ctypes.c_uint32
        L.orc_render_voxels.restype = ctypes.c_uint32
        L.orc_apply_edits.restype = ctypes.c_uint32

    # -- hashing / terrain --------------------------------------------------
    def hash_combine(self, *v: int) -> int:
        if len(v) == 2:
            return self.lib.orc_hash_combine2(v[0] & 0xFFFFFFFF, v[1] & 0xFFFFFFFF)
        if len(v) == 3:
            return self.lib.orc_hash_combine3(*(x & 0xFFFFFFFF for x in v))
        raise ValueError("2 or 3 values")

    def hash(self, v: int) -> int:
        return self.lib.orc_hash(v & 0xFFFFFFFF)

    def seed_offset(self, seed: int, salt: int) -> int:
        return self.lib.orc_seed_offset(seed & 0xFFFFFFFF, salt & 0xFFFFFFFF)

    def terrain_height(self, spec: WorldSpec, x: int, z: int) -> int:
        p = spec.params()
        return self.lib.orc_terrain_height(ctypes.byref(p), x, z)

    def permute(self, i: int, n: int, key: int) -> int:
        return self.lib.orc_permute(i, n, key & 0xFFFFFFFF)

    def place_torches(self, spec: WorldSpec, count: int, key: int) -> np.ndarray:
        out = np.zeros((max(count, 1), 3), np.int32)
        p = spec.params()
        n = self.lib.orc_place_torches(ctypes.byref(p), ctypes.c_uint32(count), ctypes.c_uint32(key & 0xFFFFFFFF),
                                       _ptr(out))
        return out[:n].copy()

    # -- world construction --------------------------------------------------
    def build_blocks(self, spec: WorldSpec, ovr_xyz=None, ovr_block=None):
        W, H, D = spec.width, spec.height, spec.depth
        xyz = np.ascontiguousarray(np.zeros((0, 3), np.int32) if ovr_xyz is None else ovr_xyz, dtype=np.int32)
        blk = np.ascontiguousarray(np.zeros(0, np.uint8) if ovr_block is None else ovr_block, dtype=np.uint8)
        blocks = np.zeros((D, H, W), np.uint8)
        hm = np.zeros((D, W), np.int16)
        p = spec.params()
        self.lib.orc_build_blocks(ctypes.byref(p), _ptr(xyz), _ptr(blk), ctypes.c_uint32(len(blk)), _ptr(blocks),
                                  _ptr(hm))
        return blocks, hm

    def light(self, blocks: np.ndarray, hm: np.ndarray, origin_y: int = 0, method: str = "per_source"):
        D, H, W = blocks.shape
        blocks = np.ascontiguousarray(blocks, np.uint8)
        hm = np.ascontiguousarray(hm, np.int16)
        bl = np.zeros_like(blocks)
        sl = np.zeros_like(blocks)
        fn = self.lib.orc_light_per_source if method == "per_source" else self.lib.orc_light_multi_source
        fn(ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_uint32(D), ctypes.c_int32(origin_y), _ptr(blocks), _ptr(hm),
           _ptr(bl), _ptr(sl))
        return bl, sl

    def render_voxels(self, blocks, block_light, sky_light, max_voxels=None) -> np.ndarray:
        D, H, W = blocks.shape
        cap = blocks.size if max_voxels is None else max_voxels
        out = np.zeros((max(cap, 1), 3), np.uint32)
        n = self.lib.orc_render_voxels(ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_uint32(D),
                                       _ptr(np.ascontiguousarray(blocks)), _ptr(np.ascontiguousarray(block_light)),
                                       _ptr(np.ascontiguousarray(sky_light)), _ptr(out), ctypes.c_uint32(cap))
        return out[:min(n, cap)].copy()

    def convert_rgba8(self, rgba: np.ndarray) -> np.ndarray:
        n, h, w, c = rgba.shape
        assert c == 4
        out = np.zeros((n, 3, h, w), np.float32)
        self.lib.orc_convert_rgba8(_ptr(np.ascontiguousarray(rgba, np.uint8)), _ptr(out), ctypes.c_uint32(n),
                                   ctypes.c_uint32(w), ctypes.c_uint32(h))
        return out

    def sky_light_at_time(self, tick: int) -> int:
        return self.lib.orc_sky_light_at_time(tick)

    def apply_edits(self, blocks: np.ndarray, hm: np.ndarray, edit_xyz, edit_kind, edit_block, origin_y: int = 0):
        """Applies edits in place (local coords); returns the number of changed cells."""
        D, H, W = blocks.shape
        assert blocks.flags.c_contiguous and hm.flags.c_contiguous
        xyz = np.ascontiguousarray(edit_xyz, np.int32)
        kind = np.ascontiguousarray(edit_kind, np.uint8)
        blk = np.ascontiguousarray(edit_block, np.uint8)
        return self.lib.orc_apply_edits(ctypes.c_uint32(W), ctypes.c_uint32(H), ctypes.c_uint32(D),
                                        ctypes.c_int32(origin_y), _ptr(blocks), _ptr(hm), _ptr(xyz), _ptr(kind),
                                        _ptr(blk), ctypes.c_uint32(len(kind)))

    # -- whole pipeline -------------------------------------------------------
    def render_frame(self, spec: WorldSpec, blocks, block_light, sky_light, params, width: int, height: int):
        """RGBA8 frame (height, width, 4) of one region (reference-layout
        volumes) for a blk_render_params record given as 96 raw bytes."""
        raw = np.frombuffer(bytes(params), np.uint8)
        assert raw.size == 96
        out = np.zeros((height, width, 4), np.uint8)
        self.lib.orc_render_frame(ctypes.c_uint32(spec.width), ctypes.c_uint32(spec.height), ctypes.c_uint32(spec.depth),
                                  ctypes.c_int32(spec.origin[0]), ctypes.c_int32(spec.origin[1]),
                                  ctypes.c_int32(spec.origin[2]), _ptr(np.ascontiguousarray(blocks, np.uint8)),
                                  _ptr(np.ascontiguousarray(block_light, np.uint8)),
                                  _ptr(np.ascontiguousarray(sky_light, np.uint8)), _ptr(raw.copy()),
                                  ctypes.c_uint32(width), ctypes.c_uint32(height), _ptr(out))
        return out

    def generate(self, spec: WorldSpec, ovr_xyz=None, ovr_block=None, method: str = "per_source"):
        blocks, hm = self.build_blocks(spec, ovr_xyz, ovr_block)
        bl, sl = self.light(blocks, hm, spec.origin[1], method)
        return blocks, bl, sl, hm


@contextlib.contextmanager
def _stdout_to_stderr():
    """The reference CPU launcher prints its thread count on load; keep stdout clean."""
    fd = os.dup(1)
    try:
        os.dup2(2, 1)
        yield
    finally:
        os.dup2(fd, 1)
        os.close(fd)


def ref_available(kind: str = "cpu") -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", f"libref_{kind}.so"))


class Reference:
    """The reference's own generator, built from its sources (oracle/_ref)."""

    def __init__(self, kind: str = "cpu") -> None:
        with _stdout_to_stderr():
            self.lib = _load(os.path.join(HERE, "_ref", f"libref_{kind}.so"))
        self.kind = kind

    def generate(self, seed: int, origin, size, ovr_xyz=None, ovr_block=None, runs: int = 2, max_voxels: int = 0,
                 timing: Optional[list] = None):
        W, H, D = size
        xyz = np.ascontiguousarray(np.zeros((0, 3), np.int32) if ovr_xyz is None else ovr_xyz, np.int32)
        blk = np.ascontiguousarray(np.zeros(0, np.uint8) if ovr_block is None else ovr_block, np.uint8)
        vol = W * H * D
        b = np.zeros(vol, np.uint8)
        bl = np.zeros(vol, np.uint8)
        sl = np.zeros(vol, np.uint8)
        hm = np.zeros(W * D, np.int8)
        vox = np.zeros(max(max_voxels, 1) * 3, np.uint32)
        cnt = np.zeros(1, np.uint32)
        hdr = np.zeros(3, np.int32)
        run_ms = np.zeros(max(runs, 1), np.float64)
        rc = self.lib.ref_generate(ctypes.c_uint32(seed & 0xFFFFFFFF), ctypes.c_int32(origin[0]),
                                   ctypes.c_int32(origin[1]), ctypes.c_int32(origin[2]), ctypes.c_uint32(W),
                                   ctypes.c_uint32(H), ctypes.c_uint32(D), _ptr(xyz), _ptr(blk),
                                   ctypes.c_uint32(len(blk)), ctypes.c_int32(runs), _ptr(b), _ptr(bl), _ptr(sl),
                                   _ptr(hm), _ptr(vox), ctypes.c_uint32(max_voxels), _ptr(cnt), _ptr(hdr),
                                   _ptr(run_ms))
        if rc != 0:
            raise RuntimeError(f"reference generate failed: {rc}")
        if timing is not None:  # wall time of every generation, ms
            timing.extend(float(v) for v in run_ms)
        sh = (D, H, W)
        n = int(min(cnt[0], max_voxels))
        return dict(blocks=b.reshape(sh), block_light=bl.reshape(sh), sky_light=sl.reshape(sh),
                    height_map=hm.reshape(D, W).astype(np.int16), voxel_count=int(cnt[0]),
                    voxels=vox.reshape(-1, 3)[:n].copy(), header=tuple(int(v) for v in hdr))

    @staticmethod
    def dense_overrides(blocks: np.ndarray, origin=(0, 0, 0)):
        """Every cell of a block volume (D, H, W) as override records (xyz, ids)."""
        D, H, W = blocks.shape
        z, y, x = np.meshgrid(np.arange(D, dtype=np.int32), np.arange(H, dtype=np.int32),
                              np.arange(W, dtype=np.int32), indexing="ij")
        xyz = np.stack([x.ravel() + origin[0], y.ravel() + origin[1], z.ravel() + origin[2]], 1)
        return xyz, np.ascontiguousarray(blocks.ravel(), np.uint8)

    def kernel_time(self, blocks: np.ndarray, origin=(0, 0, 0), runs: int = 2, reps: int = 5):
        """(kernel ms, wall ms) of the reference's generator on a block volume
        given as dense overrides: device time of its own kernels per generation
        (CUDA events around a graph of the kernels of one captured generation,
        without its host work and copies), and the wall time of one ordinary
        generation. CUDA build only."""
        D, H, W = blocks.shape
        xyz, blk = self.dense_overrides(blocks, origin)
        k_ms, w_ms = ctypes.c_double(0.0), ctypes.c_double(0.0)
        rc = self.lib.ref_kernel_time(ctypes.c_uint32(0), ctypes.c_int32(origin[0]), ctypes.c_int32(origin[1]),
                                      ctypes.c_int32(origin[2]), ctypes.c_uint32(W), ctypes.c_uint32(H),
                                      ctypes.c_uint32(D), _ptr(xyz), _ptr(blk), ctypes.c_uint32(len(blk)),
                                      ctypes.c_int32(runs), ctypes.c_int32(reps), ctypes.byref(k_ms),
                                      ctypes.byref(w_ms))
        if rc != 0:
            raise RuntimeError(f"reference kernel timing failed: {rc}")
        return k_ms.value, w_ms.value

    def light_blocks(self, blocks: np.ndarray, origin=(0, 0, 0), runs: int = 2, timing: Optional[list] = None):
        """The reference's generator run over a given block volume (D, H, W):
        every cell is passed as an override, so its terrain formula is bypassed
        and its block cache, height map and light are computed on these blocks
        (src/world/WorldGenerator.cu:142-219, :364-588). Needs W, D <= 256 and
        H <= 128 (uchar3 light-source coordinates, int8 height map); the render
        voxel list is skipped (its packing needs W, D <= 64)."""
        D, H, W = blocks.shape
        xyz, blk = self.dense_overrides(blocks, origin)
        return self.generate(0, origin, (W, H, D), xyz, blk, runs=runs, max_voxels=0, timing=timing)

    def convert_rgba8(self, rgba: np.ndarray) -> np.ndarray:
        n, h, w, _ = rgba.shape
        out = np.zeros((n, 3, h, w), np.float32)
        rc = self.lib.ref_convert_rgba8(_ptr(np.ascontiguousarray(rgba, np.uint8)), _ptr(out), ctypes.c_uint32(n),
                                        ctypes.c_uint32(w), ctypes.c_uint32(h))
        if rc != 0:
            raise RuntimeError(f"reference conversion failed: {rc}")
        return out


class ReferenceLighting:
    """The reference's sky functions (src/world/Lighting.cpp) built from its
    sources into oracle/_ref/libref_lighting.so."""

    def __init__(self):
        self.lib = ctypes.CDLL(os.path.join(HERE, "_ref", "libref_lighting.so"))
        self.lib.ref_sky_light_at.restype = ctypes.c_uint8
        self.lib.ref_sky_light_at.argtypes = [ctypes.c_uint32]
        for name in ("ref_sky_color_at", "ref_sky_direction_at"):
            getattr(self.lib, name).restype = None
            getattr(self.lib, name).argtypes = [ctypes.c_uint32, ctypes.c_void_p]

    def sky_light(self, t: int) -> int:
        return int(self.lib.ref_sky_light_at(t))

    def sky_color(self, t: int) -> np.ndarray:
        out = np.zeros(3, np.float32)
        self.lib.ref_sky_color_at(t, out.ctypes.data)
        return out

    def sky_direction(self, t: int) -> np.ndarray:
        out = np.zeros(3, np.float32)
        self.lib.ref_sky_direction_at(t, out.ctypes.data)
        return out
