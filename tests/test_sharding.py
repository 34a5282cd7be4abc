"""Env sharding host logic: shard coverage, seed policies, and the observation
gather over a world-size-2 gloo process group on CPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from blocklab_b200.sharding import env_seeds, gather_observations, hash32, shard_envs


@pytest.mark.parametrize("n,world", [(8192, 8), (8192, 3), (7, 4), (3, 8), (0, 2), (1024, 1)])
def test_shards_cover_every_env_once(n, world):
    seen = []
    for r in range(world):
        b, c = shard_envs(n, world, r)
        assert c >= 0
        seen.extend(range(b, b + c))
    assert seen == list(range(n))
    sizes = [shard_envs(n, world, r)[1] for r in range(world)]
    assert max(sizes) - min(sizes) <= 1


def test_invalid_shard_requests():
    for args in [(8, 0, 0), (8, 2, 2), (8, 2, -1), (-1, 2, 0)]:
        with pytest.raises(ValueError):
            shard_envs(*args)


def test_seed_policies_match_reference_hash(oracle):
    # Environment::reset seeds world i with hash(seed + i) (src/environment/Environment.cpp:37-42).
    s = env_seeds(1, 0, 64, "reference")
    assert [int(v) for v in s] == [oracle.hash(1 + i) for i in range(64)]
    assert list(env_seeds(1, 5, 3, "offset")) == [6, 7, 8]
    assert int(hash32(np.array([0xFFFFFFFF], np.uint32))[0]) == oracle.hash(0xFFFFFFFF)
    # wrap-around of seed + i stays in 32 bits
    assert list(env_seeds(0xFFFFFFFF, 0, 2, "offset")) == [0xFFFFFFFF, 0]
    with pytest.raises(ValueError):
        env_seeds(1, 0, 1, "nope")


def test_seeds_independent_of_rank_count():
    whole = env_seeds(77, 0, 100, "reference")
    for world in (2, 3, 8):
        parts = [env_seeds(77, *shard_envs(100, world, r), "reference") for r in range(world)]
        assert np.array_equal(np.concatenate(parts), whole)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, world, port, n_envs, result_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        begin, count = shard_envs(n_envs, world, rank)
        seeds = env_seeds(5, begin, count, "reference")
        # a per-rank "observation": the env seeds of the shard, padded to equal shapes
        size = shard_envs(n_envs, world, 0)[1]
        obs = torch.full((size,), -1, dtype=torch.int64)
        obs[:count] = torch.from_numpy(seeds.astype(np.int64))
        got = gather_observations(obs, dst=0)
        if rank == 0:
            flat = torch.cat([g[g >= 0] for g in got]).numpy()
            np.save(os.path.join(result_dir, "gathered.npy"), flat)
        else:
            assert got is None
    finally:
        dist.destroy_process_group()


def test_gather_two_ranks_gloo(tmp_path):
    world, n_envs = 2, 9
    mp.start_processes(_gather_worker, args=(world, _free_port(), n_envs, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    flat = np.load(tmp_path / "gathered.npy")
    assert np.array_equal(flat, env_seeds(5, 0, n_envs, "reference").astype(np.int64))


def test_gather_single_process_is_identity():
    x = torch.arange(4)
    assert gather_observations(x)[0] is x
