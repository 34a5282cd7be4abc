"""WorldEnv (reset / step over the world-state path) on the GPU: parity with
the oracle, shard consistency across rank counts, observation buffers."""
import numpy as np
import pytest
import torch

from oracle.oracle import TERRAIN_FBM, WorldSpec

pytestmark = pytest.mark.gpu

W, H, D = 48, 64, 40
ORIGIN = (-24, 0, -20)


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


def _env(B, **kw):
    from blocklab_b200.env import WorldEnv

    args = dict(num_envs=3, width=32, height=24, world_size=(W, H, D), origin=ORIGIN, terrain=TERRAIN_FBM, base=30,
                amplitude=20.0)
    args.update(kw)
    return WorldEnv(**args)


def _world(env, e):
    ids = env.world.ids[e].cpu().numpy().transpose(0, 2, 1)
    light = env.world.light[e].cpu().numpy().transpose(0, 2, 1)
    return ids, light & 15, light >> 4, env.world.height_map[e].cpu().numpy()


def test_reset_and_step_match_oracle(B, oracle):
    from blocklab_b200.sharding import env_seeds

    env = _env(B)
    rng = np.random.default_rng(3)
    frames = torch.randint(0, 256, (3, 24, 32, 4), dtype=torch.uint8, device="cuda")
    obs, info = env.reset(seed=11, frames=frames)
    seeds = env_seeds(11, 0, 3, "reference")
    state = []
    for e in range(3):
        spec = WorldSpec(int(seeds[e]), W, H, D, origin=ORIGIN, terrain=TERRAIN_FBM, base=30, amplitude=20.0)
        blocks, hm = oracle.build_blocks(spec)
        bl, sl = oracle.light(blocks, hm, ORIGIN[1], "multi")
        got = _world(env, e)
        assert np.array_equal(got[0], blocks) and np.array_equal(got[3], hm)
        assert np.array_equal(got[1], bl) and np.array_equal(got[2], sl)
        state.append((blocks, hm))
    want_obs = oracle.convert_rgba8(frames.cpu().numpy())
    assert np.array_equal(obs.cpu().numpy().view(np.uint32), want_obs.view(np.uint32))
    for step in range(3):
        lists, local = [], []
        for e in range(3):
            n = 40
            x, z = rng.integers(0, W, n), rng.integers(0, D, n)
            y = state[e][1][z, x] + rng.integers(-6, 7, n)
            blk = rng.choice([0, 3, 4], n, p=[0.45, 0.45, 0.1]).astype(np.uint8)
            kind = np.zeros(n, np.uint8)
            xyz = np.stack([x, y, z], 1)
            local.append((xyz, kind, blk))
            lists.append(B.make_overrides(xyz + np.array(ORIGIN), blk, env=e, kind=kind))
        obs2, info2 = env.step(np.concatenate(lists))
        assert info2["observation_version"] == info["observation_version"] + step + 1
        env.world.sync()
        for e in range(3):
            xyz, kind, blk = local[e]
            oracle.apply_edits(state[e][0], state[e][1], xyz, kind, blk, origin_y=ORIGIN[1])
            bl, sl = oracle.light(state[e][0], state[e][1], ORIGIN[1], "multi")
            got = _world(env, e)
            assert np.array_equal(got[0], state[e][0]), (step, e)
            assert np.array_equal(got[1], bl) and np.array_equal(got[2], sl), (step, e)
    env.close()


def test_shards_equal_single_process_batch(B):
    whole = _env(B, num_envs=5)
    parts = [_env(B, num_envs=5, ranks=2, rank=r) for r in range(2)]
    whole.reset(seed=9)
    for p in parts:
        p.reset(seed=9)
    torch.cuda.synchronize()
    assert (parts[0].env_begin, parts[0].local_envs) == (0, 3)
    assert (parts[1].env_begin, parts[1].local_envs) == (3, 2)
    assert torch.equal(whole.world.ids[:3], parts[0].world.ids)
    assert torch.equal(whole.world.ids[3:], parts[1].world.ids)
    assert torch.equal(whole.world.light[:3], parts[0].world.light)
    assert torch.equal(whole.world.light[3:], parts[1].world.light)
    for e in (whole, *parts):
        e.close()


def test_observation_buffers_and_dlpack(B):
    env = _env(B)
    with pytest.raises(RuntimeError):
        env.step()
    f1 = torch.randint(0, 256, (3, 24, 32, 4), dtype=torch.uint8, device="cuda")
    f2 = torch.randint(0, 256, (3, 24, 32, 4), dtype=torch.uint8, device="cuda")
    o1, _ = env.reset(seed=1, frames=f1)
    keep = o1.clone()
    o2, _ = env.step(frames=f2)
    assert o1.data_ptr() != o2.data_ptr()
    assert torch.equal(o1, keep)  # the previous observation stays valid for one more call
    cap = torch.utils.dlpack.to_dlpack(o2)
    back = torch.utils.dlpack.from_dlpack(cap)
    assert back.data_ptr() == o2.data_ptr() and back.shape == (3, 3, 24, 32)
    with pytest.raises(ValueError):
        env.step(frames=torch.zeros((3, 24, 31, 4), dtype=torch.uint8, device="cuda"))
    env.close()
