"""Env sharding across GPUs: one process per GPU, each owning a contiguous
slice of the global env batch, and the optional observation gather.

Envs are independent, so the world-state path has no data-path collective:
rank r generates, edits and relights only its own envs, and results do not
depend on the number of ranks because every env's seed is a function of its
global index. The only exchange is the optional gather of per-rank
observations to one rank (NCCL over NVLink on GPUs, gloo on CPU).
"""
from __future__ import annotations

from typing import Optional

import numpy as np


def shard_envs(num_envs: int, world_size: int, rank: int) -> tuple[int, int]:
    """(first global env, env count) of `rank`: contiguous, sizes differ by at most one."""
    if world_size <= 0 or not 0 <= rank < world_size or num_envs < 0:
        raise ValueError("invalid shard request")
    base, extra = divmod(num_envs, world_size)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def hash32(v: np.ndarray) -> np.ndarray:
    """The reference's integer hash (src/utility/Hash.h:26-34), vectorised."""
    v = np.asarray(v, dtype=np.uint32).copy()
    with np.errstate(over="ignore"):
        v ^= v >> np.uint32(16)
        v *= np.uint32(0x7FEB352D)
        v ^= v >> np.uint32(15)
        v *= np.uint32(0x846CA68B)
        v ^= v >> np.uint32(16)
    return v


def env_seeds(seed: int, begin: int, count: int, policy: str = "reference") -> np.ndarray:
    """World seeds of global envs begin .. begin + count - 1.

    policy "reference": hash(seed + i), as Environment::reset seeds each
    world (src/environment/Environment.cpp:37-42); "offset": seed + i, the
    benchmark configurations' per-env seed."""
    i = np.arange(begin, begin + count, dtype=np.uint64)
    raw = ((np.uint64(seed) + i) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    if policy == "reference":
        return hash32(raw)
    if policy == "offset":
        return raw
    raise ValueError(f"unknown seed policy {policy!r}")


def gather_observations(obs, dst: int = 0, group=None) -> Optional[list]:
    """Gathers every rank's observation tensor (same shape on every rank) to
    rank `dst`; returns the list of tensors in rank order there, None elsewhere.
    Every rank must call it, in the same order relative to other collectives."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return [obs]
    rank = dist.get_rank(group)
    out = [torch.empty_like(obs) for _ in range(dist.get_world_size(group))] if rank == dst else None
    dist.gather(obs, out, dst=dst, group=group)
    return out
