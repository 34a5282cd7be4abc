"""World-state environment batch: the reset / step surface of the reference's
BlockLabEnv (python/blocklab/env.py:155-194) restricted to the world-state
path. The agent and rewards are not part of this library: `step` takes the
caller's edits (dig / place / torch) and, optionally, rendered RGBA8 frames,
and returns the float32 NCHW observation; `render` produces the observation
from the library's own ray-cast frames of the worlds.

Observations are double-buffered device tensors, valid until the next call
after the following one (the reference's renderer double-buffers them the
same way, src/graphics/Renderer.cpp:605-613); they export through DLPack
(`torch.utils.dlpack.to_dlpack` or the tensor's `__dlpack__`).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .observation import convert_rgba8_to_float_nchw
from .sharding import env_seeds, shard_envs
from .world import WorldBatch, WorldConfig


class WorldEnv:
    def __init__(self, *, num_envs: int = 1, width: int = 160, height: int = 90, device=None,
                 world_size: tuple[int, int, int] = (64, 32, 64), origin: tuple[int, int, int] = (-32, 0, -32),
                 terrain: int = 0, seed_policy: str = "reference", rank: int = 0, ranks: int = 1,
                 max_overrides: int = 1 << 16, max_edits: int = 1 << 16, **terrain_kwargs) -> None:
        """num_envs is the global batch; with `ranks` > 1 this process owns the
        contiguous slice shard_envs(num_envs, ranks, rank). `terrain` is a
        blk_terrain_mode (0: the reference's formula)."""
        dev = torch.device(device) if device is not None else torch.device("cuda")
        self.device = dev
        self.num_envs = num_envs
        self.env_begin, self.local_envs = shard_envs(num_envs, ranks, rank)
        self.width, self.height = width, height
        self.seed_policy = seed_policy
        W, H, D = world_size
        self.config = WorldConfig(num_envs=max(self.local_envs, 1), width=W, height=H, depth=D, origin=origin,
                                  terrain=terrain, max_overrides=max_overrides, max_edits=max_edits,
                                  **terrain_kwargs)
        self.world = WorldBatch(self.config, device=dev.index if dev.index is not None else 0)
        n = self.config.num_envs
        self._obs = [torch.zeros((n, 3, height, width), dtype=torch.float32, device=dev) for _ in range(2)]
        self._flip = 0
        self._version = 0
        self._reset_done = False

    def _next_obs(self, frames: Optional[torch.Tensor]) -> torch.Tensor:
        out = self._obs[self._flip]
        self._flip ^= 1
        if frames is not None:
            if frames.shape != (self.config.num_envs, self.height, self.width, 4):
                raise ValueError(f"frames must be ({self.config.num_envs}, {self.height}, {self.width}, 4) uint8")
            convert_rgba8_to_float_nchw(frames, out=out)
        self._version += 1
        return out

    def reset(self, *, seed: int = 1, overrides=None, frames: Optional[torch.Tensor] = None, origins=None):
        """Regenerates and fully relights every owned world. World i (global
        index) gets the seed of `seed_policy`; overrides are blk_override
        records with env indices local to this process; `origins` (local envs,
        3) places each world's region (None keeps the current ones)."""
        seeds = env_seeds(seed, self.env_begin, self.config.num_envs, self.seed_policy)
        self.world.generate(seeds, overrides, origins=origins)
        self._reset_done = True
        obs = self._next_obs(frames)
        return obs, {"observation_version": self._version, "env_begin": self.env_begin}

    def reset_envs(self, env_ids, *, seed: int = 1, overrides=None, origins=None):
        """Regenerates only the listed worlds (indices local to this process);
        world i gets the seed of its global index, as in reset(), and, when
        given, the region origin origins[k] of its list position k."""
        ids = np.asarray(env_ids, np.int64)
        seeds = np.array([env_seeds(seed, self.env_begin + int(i), 1, self.seed_policy)[0] for i in ids], np.uint32)
        self.world.generate_envs(ids.astype(np.uint32), seeds, overrides, origins=origins)

    def render(self, params) -> torch.Tensor:
        """Observation rendered by the library itself: ray-cast RGBA8 frames of
        every owned world from per-env render parameters (render_params_at),
        converted to float32 NCHW."""
        out = self._obs[self._flip]
        self._flip ^= 1
        self.world.render_observations(params, self.width, self.height, out=out)
        self._version += 1
        return out

    def step(self, edits=None, frames: Optional[torch.Tensor] = None):
        """Applies edits (World::setBlock semantics, exact relight) and converts
        the rendered frames."""
        if not self._reset_done:
            raise RuntimeError("Environment is not reset. Call reset() before step().")
        if edits is not None and (not hasattr(edits, "__len__") or len(edits) > 0):
            self.world.apply_edits(edits)
        obs = self._next_obs(frames)
        return obs, {"observation_version": self._version}

    def close(self) -> None:
        self.world.close()


def make(**kwargs) -> WorldEnv:
    return WorldEnv(**kwargs)
