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


def _batch_world(wb, e):
    """(ids, block light, sky light, height map) of env e in the oracle's layout."""
    ids = wb.ids[e].cpu().numpy().transpose(0, 2, 1)
    light = wb.light[e].cpu().numpy().transpose(0, 2, 1)
    return ids, light & 15, light >> 4, wb.height_map[e].cpu().numpy()


def _world(env, e):
    return _batch_world(env.world, e)


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
    assert np.array_equal(obs.to_tensor().cpu().numpy().view(np.uint32), want_obs.view(np.uint32))
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
    t1 = o1.to_tensor()
    keep = t1.clone()
    o2, _ = env.step(frames=f2)
    t2 = torch.from_dlpack(o2)
    assert t1.data_ptr() != t2.data_ptr() and o2.version == o1.version + 1
    assert torch.equal(t1, keep)  # the previous observation stays valid for one more call
    assert o2.__dlpack_device__() == (2, 0) and o2.shape == (3, 3, 24, 32)
    back = torch.utils.dlpack.from_dlpack(o2.__dlpack__(stream=1))  # legacy default stream
    assert back.data_ptr() == t2.data_ptr() and back.shape == (3, 3, 24, 32)
    with pytest.raises(ValueError):
        env.step(frames=torch.zeros((3, 24, 31, 4), dtype=torch.uint8, device="cuda"))
    env.close()


def test_partial_reset_matches_full_generation(B):
    W2, H2, D2, E2 = 70, 64, 50, 4
    cfg = B.WorldConfig(num_envs=E2, width=W2, height=H2, depth=D2, origin=(3, 0, -9), terrain=TERRAIN_FBM, base=25,
                        amplitude=15.0)
    rng = np.random.default_rng(9)
    seeds = np.array([11, 12, 13, 14], np.uint32)
    new = np.array([101, 103], np.uint32)

    def overrides(envs):
        out = []
        for e in envs:
            cells = rng.choice(W2 * H2 * D2, 300, replace=False)
            xyz = np.stack([cells % W2, (cells // W2) % H2, cells // (W2 * H2)], 1) + np.array([3, 0, -9])
            out.append(B.make_overrides(xyz, rng.choice([0, 3, 4], 300).astype(np.uint8), env=e))
        return np.concatenate(out)

    first = overrides(range(E2))
    partial = overrides([0, 1, 3])  # env 0's records must be ignored
    wb = B.WorldBatch(cfg)
    wb.generate(seeds, first)
    before = (wb.ids.clone(), wb.light.clone(), wb.height_map.clone())
    wb.generate_envs([1, 3], new, partial)
    wb.sync()
    # reference: a full generation with the new seeds and the partial overrides for envs 1, 3
    full_seeds = seeds.copy()
    full_seeds[[1, 3]] = new
    keep = partial[partial["env"] != 0]
    ref = B.WorldBatch(cfg)
    ref.generate(full_seeds, np.concatenate([first[np.isin(first["env"], [0, 2])], keep]))
    ref.sync()
    for e in (1, 3):
        assert torch.equal(wb.ids[e], ref.ids[e]) and torch.equal(wb.light[e], ref.light[e])
        assert torch.equal(wb.height_map[e], ref.height_map[e])
    for e in (0, 2):
        assert torch.equal(wb.ids[e], before[0][e]) and torch.equal(wb.light[e], before[1][e])
        assert torch.equal(wb.height_map[e], before[2][e])
    # edits and relight still work after a partial reset
    hm = wb.height_map.cpu().numpy()
    ed = B.make_overrides([[3 + 5, int(hm[1, 4, 5]), -9 + 4]], B.AIR, env=1)
    wb.apply_edits(ed)
    ref.apply_edits(ed)
    wb.sync()
    ref.sync()
    assert torch.equal(wb.light, torch.cat([before[1][0:1], ref.light[1:2], before[1][2:3], ref.light[3:4]]))
    # an env index out of range is reported by sync
    wb.generate_envs([1, 9], [5, 6])
    with pytest.raises(B.BlkError):
        wb.sync()
    wb.close()
    ref.close()


def test_env_renders_its_observations(B):
    env = _env(B)
    env.reset(seed=4)
    params = np.array([B.render_params_at((-10 + 3 * e, 45, -5), 0.5 * e, -0.4, 3000) for e in range(3)],
                      B.RENDER_PARAMS_DTYPE)
    obs = env.render(params).to_tensor()
    frames = env.world.render(params, 32, 24)
    torch.cuda.synchronize()
    assert obs.shape == (3, 3, 24, 32)
    assert torch.equal(obs[:, 1], frames[..., 1].float() * np.float32(1.0 / 255.0))
    env.close()


def test_partial_reset_matches_oracle_with_new_origins(B, oracle):
    """blk_generate_envs against the oracle: a ragged, unordered env list with
    new seeds and new region origins per listed env, overrides of listed and
    unlisted envs (the unlisted ones are ignored), then an empty list and a
    list holding an out-of-range id (its valid entries are still reset)."""
    W2, H2, D2, E2 = 45, 96, 38, 5
    base = dict(terrain=TERRAIN_FBM, base=40, amplitude=30.0)
    cfg = B.WorldConfig(num_envs=E2, width=W2, height=H2, depth=D2, origin=(0, 0, 0), **base)
    rng = np.random.default_rng(21)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(31, 31 + E2, dtype=np.uint32)
    wb.generate(seeds)

    def random_overrides(e, origin, n=400):
        cells = rng.choice(W2 * H2 * D2, n, replace=False)
        xyz = np.stack([cells % W2, (cells // W2) % H2, cells // (W2 * H2)], 1) + np.array(origin)
        blk = rng.choice([0, 3, 4, 1, 2], n, p=[0.45, 0.3, 0.15, 0.05, 0.05]).astype(np.uint8)
        return xyz, blk

    listed = [4, 0, 2]
    new_seeds = np.array([501, 502, 503], np.uint32)
    new_origins = np.array([[-100, -8, 7], [3, 5, -2000], [64, 0, 64]], np.int32)
    per, lists = {}, []
    for k, e in enumerate(listed):
        per[e] = random_overrides(e, new_origins[k])
        lists.append(B.make_overrides(*per[e], env=e))
    for e in (1, 3):  # records of envs that are not reset
        lists.append(B.make_overrides(*random_overrides(e, (0, 0, 0)), env=e))
    ovr = np.concatenate(lists)
    rng.shuffle(ovr)
    before = (wb.ids[[1, 3]].clone(), wb.light[[1, 3]].clone(), wb.height_map[[1, 3]].clone())
    wb.generate_envs(listed, new_seeds, ovr, origins=new_origins)
    wb.sync()
    for k, e in enumerate(listed):
        spec = WorldSpec(int(new_seeds[k]), W2, H2, D2, origin=tuple(int(v) for v in new_origins[k]), **base)
        blocks, bl, sl, hm = oracle.generate(spec, *per[e], method="multi")
        got = _batch_world(wb, e)
        assert np.array_equal(got[0], blocks) and np.array_equal(got[3], hm), e
        assert np.array_equal(got[1], bl) and np.array_equal(got[2], sl), e
        assert wb.origins[e, :3].tolist() == new_origins[k].tolist()
    assert torch.equal(wb.ids[[1, 3]], before[0]) and torch.equal(wb.light[[1, 3]], before[1])
    assert torch.equal(wb.height_map[[1, 3]], before[2])
    wb.generate_envs([], [])
    wb.sync()
    wb.generate_envs([7, 1], [900, 901])
    with pytest.raises(B.BlkError):
        wb.sync()
    spec = WorldSpec(901, W2, H2, D2, origin=(0, 0, 0), **base)
    blocks, bl, sl, hm = oracle.generate(spec, method="multi")
    got = _batch_world(wb, 1)
    assert np.array_equal(got[0], blocks) and np.array_equal(got[1], bl) and np.array_equal(got[2], sl)
    wb.close()


def test_observation_consumed_on_another_stream(B, oracle):
    """The consumer of an observation runs on its own stream while the
    producer's stream is still busy (a ~25 ms spin queued before the
    conversion): importing it through DLPack makes the consumer stream wait
    for the write, as the reference's observation_dlpack does with
    enqueueReadyWait (src/python/Bindings.cpp:150-151)."""
    env = _env(B)
    env.reset(seed=2)
    rng = np.random.default_rng(12)
    frames_np = rng.integers(0, 256, (3, 24, 32, 4), dtype=np.uint8)
    frames = torch.from_numpy(frames_np).cuda()
    want = torch.from_numpy(oracle.convert_rgba8(frames_np)).cuda()
    consumer = torch.cuda.Stream()
    for trial in range(3):
        torch.cuda.synchronize()
        torch.cuda._sleep(50_000_000)  # the producer stream stays busy before the conversion
        obs, _ = env.step(frames=frames)
        with torch.cuda.stream(consumer):
            t = torch.from_dlpack(obs)  # the consumer stream waits for the observation's event
            total = (t == want).all()
        consumer.synchronize()
        assert bool(total.item()), f"trial {trial}: the consumer read the observation before it was written"
        frames = torch.flip(frames, dims=[0]).contiguous()
        frames_np = frames_np[::-1].copy()
        want = torch.from_numpy(oracle.convert_rgba8(frames_np)).cuda()
    env.close()
