"""World-state environment batch: the reset / step surface of the reference's
BlockLabEnv (python/blocklab/env.py:155-194) restricted to the world-state
path. The agent and rewards are not part of this library: `step` takes the
caller's edits (dig / place / torch) and, optionally, rendered RGBA8 frames,
and returns the float32 NCHW observation; `render` produces the observation
from the library's own ray-cast frames of the worlds.

Observations are double-buffered device tensors, valid until the next call
after the following one (the reference's renderer double-buffers them the
same way, src/graphics/Renderer.cpp:605-613). reset / step / render return a
WorldObservation: a DLPack producer whose consumer stream waits for the
observation's write, as the reference's BlockLabObservation does
(python/blocklab/env.py:29-62, src/python/Bindings.cpp:138-183).
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .observation import convert_rgba8_to_float_nchw
from .sharding import env_seeds, shard_envs
from .world import WorldBatch, WorldConfig


class WorldObservation:
    """One observation: the float32 (envs, 3, height, width) tensor written on
    the env's stream and a CUDA event recorded after that write. Importing it
    through DLPack (torch.from_dlpack(obs), or obs.to_tensor()) makes the
    consumer's stream wait for the event first, so a consumer on any stream
    sees the finished observation; the data stays valid until the env's next
    call after the following one."""

    def __init__(self, tensor: torch.Tensor, event: torch.cuda.Event, version: int) -> None:
        self._tensor = tensor
        self._event = event
        self.version = version
        self.shape = tuple(tensor.shape)
        self.dtype = tensor.dtype
        self.device = tensor.device

    def __dlpack_device__(self) -> tuple[int, int]:
        return (2, self.device.index if self.device.index is not None else 0)  # kDLCUDA

    def __dlpack__(self, stream: Optional[int] = None, **_kwargs):
        """DLPack capsule of the tensor after making `stream` wait for the
        observation: None waits on the current stream, 1 is the legacy default
        stream, 2 the per-thread default stream, any other value a stream
        handle (the DLPack stream convention for CUDA)."""
        if stream is None:
            consumer = torch.cuda.current_stream(self.device)
        else:
            handle = 0 if stream == 1 else stream  # 0 addresses the legacy default stream
            consumer = torch.cuda.ExternalStream(handle, device=self.device)
        consumer.wait_event(self._event)
        return torch.utils.dlpack.to_dlpack(self._tensor)

    def to_tensor(self) -> torch.Tensor:
        return torch.from_dlpack(self)

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Makes `stream` (default: the current one) wait for the observation."""
        (stream or torch.cuda.current_stream(self.device)).wait_event(self._event)


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

    def _published(self, out: torch.Tensor) -> WorldObservation:
        """Records the observation's ready event on the current stream."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self._version += 1
        return WorldObservation(out, ev, self._version)

    def _next_obs(self, frames: Optional[torch.Tensor]) -> WorldObservation:
        out = self._obs[self._flip]
        self._flip ^= 1
        if frames is not None:
            if frames.shape != (self.config.num_envs, self.height, self.width, 4):
                raise ValueError(f"frames must be ({self.config.num_envs}, {self.height}, {self.width}, 4) uint8")
            convert_rgba8_to_float_nchw(frames, out=out)
        return self._published(out)

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

    def render(self, params) -> WorldObservation:
        """Observation rendered by the library itself: ray-cast RGBA8 frames of
        every owned world from per-env render parameters (render_params_at),
        converted to float32 NCHW."""
        out = self._obs[self._flip]
        self._flip ^= 1
        self.world.render_observations(params, self.width, self.height, out=out)
        return self._published(out)

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
