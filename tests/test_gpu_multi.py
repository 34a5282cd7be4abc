"""The sharded WorldEnv on two or more GPUs, one process per GPU: every rank's
shard equals the same envs of a single-process batch (the env-index split has
no data-path collective), and the observation gather to rank 0 over NCCL.

Runs only where at least two CUDA devices are visible (`-m gpu` on a multi-GPU
box); the rank processes are children started with `spawn`."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

W, H, D = 48, 64, 40


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, num_envs, out_dir):
    import datetime

    import torch.distributed as dist

    import blocklab_b200 as B
    from blocklab_b200.env import WorldEnv
    from blocklab_b200.sharding import gather_observations

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    env = WorldEnv(num_envs=num_envs, width=32, height=24, device=f"cuda:{rank}", world_size=(W, H, D),
                   origin=(-24, 0, -20), terrain=B.TERRAIN_FBM, base=30, amplitude=20.0, rank=rank, ranks=world)
    gen = torch.Generator().manual_seed(5)
    frames_all = torch.randint(0, 256, (num_envs, 24, 32, 4), dtype=torch.uint8, generator=gen)
    frames = frames_all[env.env_begin:env.env_begin + env.local_envs].to(f"cuda:{rank}")
    obs, _ = env.reset(seed=3, frames=frames)
    # One step of edits on every local env (world coordinates, local env indices).
    hm = env.world.height_map.cpu().numpy()
    xs = np.arange(env.local_envs) % W
    edits = B.make_overrides(np.stack([xs - 24, hm[np.arange(env.local_envs), 5, xs] + 1, np.full_like(xs, 5 - 20)], 1),
                             B.TORCH, env=np.arange(env.local_envs))
    obs, _ = env.step(edits=edits, frames=frames)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), env.world.ids.cpu().numpy())
    np.save(os.path.join(out_dir, f"light{rank}.npy"), env.world.light.cpu().numpy())
    gathered = gather_observations(obs.to_tensor(), dst=0)
    if rank == 0:
        np.save(os.path.join(out_dir, "gathered.npy"), torch.cat(gathered).cpu().numpy())
    env.close()
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_env_on_two_gpus_equals_single_process(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    import torch.multiprocessing as mp

    import blocklab_b200 as B
    from blocklab_b200.env import WorldEnv

    world, num_envs = 2, 6  # equal shards: the gather needs one shape on every rank
    mp.start_processes(_rank_main, args=(world, _free_port(), num_envs, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    # The same envs in one process on one GPU.
    env = WorldEnv(num_envs=num_envs, width=32, height=24, device="cuda:0", world_size=(W, H, D),
                   origin=(-24, 0, -20), terrain=B.TERRAIN_FBM, base=30, amplitude=20.0)
    gen = torch.Generator().manual_seed(5)
    frames = torch.randint(0, 256, (num_envs, 24, 32, 4), dtype=torch.uint8, generator=gen).cuda()
    env.reset(seed=3, frames=frames)
    hm = env.world.height_map.cpu().numpy()
    ids_parts = [np.load(tmp_path / f"ids{r}.npy") for r in range(world)]
    light_parts = [np.load(tmp_path / f"light{r}.npy") for r in range(world)]
    begins = [0, ids_parts[0].shape[0]]
    edits = []
    for r in range(world):
        n = ids_parts[r].shape[0]
        xs = np.arange(n) % W
        e = np.arange(n) + begins[r]
        edits.append(B.make_overrides(np.stack([xs - 24, hm[e, 5, xs] + 1, np.full_like(xs, 5 - 20)], 1), B.TORCH,
                                      env=e))
    obs, _ = env.step(edits=np.concatenate(edits), frames=frames)
    torch.cuda.synchronize()
    assert np.array_equal(np.concatenate(ids_parts), env.world.ids.cpu().numpy())
    assert np.array_equal(np.concatenate(light_parts), env.world.light.cpu().numpy())
    assert np.array_equal(np.load(tmp_path / "gathered.npy"), obs.to_tensor().cpu().numpy())
    env.close()
