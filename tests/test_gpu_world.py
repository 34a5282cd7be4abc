"""GPU parity tests of the world-state path through the C ABI.

Every comparison is bit-exact (integer block ids and 4-bit light levels; the
observation conversion is compared as float bit patterns). The oracle is the
C++ restatement pinned to the reference (tests/test_oracle.py); the committed
golden fixture holds the reference's own output for its lighting tests.
At full benchmark size the light field is checked through the fixed-point
equations it uniquely satisfies (see _fixed_point_ok).
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle.oracle import TERRAIN_FBM, TERRAIN_FLAT, TERRAIN_REFERENCE, WorldSpec

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import scenarios as S  # noqa: E402

GOLDEN = os.path.join(HERE, "golden", "lighting_scenarios.npz")


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


def _dev_world(wb, env):
    """Device arrays of one env in the reference layout (D, H, W)."""
    ids = wb.ids[env].cpu().numpy().transpose(0, 2, 1)
    light = wb.light[env].cpu().numpy().transpose(0, 2, 1)
    return ids, light & 15, light >> 4, wb.height_map[env].cpu().numpy()


def _assert_world(wb, env, blocks, bl, sl, hm, label=""):
    ids, gbl, gsl, ghm = _dev_world(wb, env)
    assert np.array_equal(ids, blocks), f"{label} ids differ at {np.argwhere(ids != blocks)[:5].tolist()}"
    assert np.array_equal(ghm, hm), f"{label} height map differs"
    assert np.array_equal(gbl, bl), f"{label} block light differs at {np.argwhere(gbl != bl)[:5].tolist()}"
    assert np.array_equal(gsl, sl), f"{label} sky light differs at {np.argwhere(gsl != sl)[:5].tolist()}"


def _xyz(ovr):
    return np.stack([ovr["x"], ovr["y"], ovr["z"]], 1)


# ------------------------------------------------------------ conversion --
@pytest.mark.parametrize("shape", [(128, 90, 160), (7, 84, 84), (3, 9, 13), (1, 1, 1), (2, 90, 160)])
def test_convert_bit_exact(B, oracle, shape):
    n, h, w = shape
    rng = np.random.default_rng(n * 1000 + h)
    rgba = rng.integers(0, 256, (n, h, w, 4), dtype=np.uint8)
    out = B.convert_rgba8_to_float_nchw(torch.from_numpy(rgba).cuda()).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), oracle.convert_rgba8(rgba).view(np.uint32))


def test_convert_every_byte_and_unaligned(B, oracle):
    rgba = np.tile(np.arange(256, dtype=np.uint8)[None, None, :, None], (1, 3, 1, 4)).copy()
    rgba[..., 1] = 255 - rgba[..., 1]
    dev = torch.from_numpy(rgba).cuda()
    out = B.convert_rgba8_to_float_nchw(dev).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), oracle.convert_rgba8(rgba).view(np.uint32))
    # unaligned source (offset by one pixel) takes the scalar path
    big = torch.from_numpy(np.concatenate([rgba.reshape(-1, 4)[:1], rgba.reshape(-1, 4)])).cuda()
    view = big[1:].reshape(1, 3, 256, 4)
    out2 = torch.empty((1, 3, 3, 256), dtype=torch.float32, device="cuda")
    from blocklab_b200 import _native as N

    N.check(N.lib.blk_convert_rgba8_to_float_nchw(view.data_ptr(), out2.data_ptr(), 1, 256, 3, 0))
    torch.cuda.synchronize()
    assert np.array_equal(out2.cpu().numpy().view(np.uint32), oracle.convert_rgba8(rgba).view(np.uint32))


# ------------------------------------------------------------ generation --
def test_config0_fbm_with_torches_matches_oracle(B, oracle):
    """Config 0: 64 x 64 x 128, fBm seed 1, 200 surface torches (per-source oracle)."""
    cfg = B.WorldConfig(num_envs=1, width=64, height=128, depth=64)
    wb = B.WorldBatch(cfg)
    spec = WorldSpec(1, 64, 128, 64)
    t = oracle.place_torches(spec, 200, B.torch_key(1))
    assert len(t) == 200
    wb.generate([1], B.make_overrides(t, B.TORCH))
    wb.sync()
    blocks, bl, sl, hm = oracle.generate(spec, t, np.full(len(t), 4, np.uint8), method="per_source")
    _assert_world(wb, 0, blocks, bl, sl, hm, "config0")
    assert (bl > 0).sum() > 10000
    wb.close()


def test_device_torch_placement_matches_oracle(B, oracle):
    cfg = B.WorldConfig(num_envs=3, width=96, height=128, depth=80)
    wb = B.WorldBatch(cfg)
    seeds = np.array([1, 2, 99], np.uint32)
    dev = wb.place_torches(seeds, 300).cpu().numpy().view(B.OVERRIDE_DTYPE)
    assert len(dev) == 900
    for e, s in enumerate(seeds):
        spec = WorldSpec(int(s), 96, 128, 80)
        want = oracle.place_torches(spec, 300, B.torch_key(int(s)))
        got = dev[(dev["env"] == e) & (dev["y"] > -(1 << 30))]
        assert np.array_equal(_xyz(got), want)
    wb.close()


@pytest.mark.parametrize("terrain,base,amp", [(TERRAIN_FBM, 40, 50.0), (TERRAIN_FLAT, 20, 0.0),
                                             (TERRAIN_FBM, 60, 120.0)])
def test_random_overrides_match_oracle(B, oracle, terrain, base, amp):
    """Caves, floating stone, torches everywhere; ragged tile edges (W, D not multiples of 32)."""
    W, H, D, E = 77, 128, 45, 3
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=(-10, 0, 5), terrain=terrain, base=base,
                        amplitude=amp)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(base)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    lists, per = [], []
    for e in range(E):
        n = 6000
        cells = rng.choice(W * H * D, n, replace=False)
        xyz = np.stack([cells % W - 10, (cells // W) % H, cells // (W * H) + 5], 1)
        blk = rng.choice([0, 3, 4, 1, 2], n, p=[0.5, 0.3, 0.1, 0.05, 0.05]).astype(np.uint8)
        per.append((xyz, blk))
        lists.append(B.make_overrides(xyz, blk, env=e))
    wb.generate(seeds, np.concatenate(lists))
    wb.sync()
    for e in range(E):
        spec = WorldSpec(int(seeds[e]), W, H, D, origin=(-10, 0, 5), terrain=terrain, base=base, amplitude=amp)
        blocks, bl, sl, hm = oracle.generate(spec, *per[e], method="multi")
        _assert_world(wb, e, blocks, bl, sl, hm, f"env{e}")
    wb.close()


@pytest.mark.parametrize("W,H,D,terrain,base,amp", [(70, 256, 40, TERRAIN_FBM, 40, 50.0),
                                                     (45, 160, 33, TERRAIN_FLAT, 150, 0.0),
                                                     (64, 224, 64, TERRAIN_FBM, 120, 100.0)])
def test_tall_worlds_match_oracle(B, oracle, W, H, D, terrain, base, amp):
    """Heights above 128: the layer rule over the upper rows, and tiles whose
    torch rows are far apart, so their light is computed in several row windows."""
    E = 2
    origin = (3, 0, -7)
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=origin, terrain=terrain, base=base,
                        amplitude=amp)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(H + base)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    lists, per = [], []
    for e in range(E):
        n = 4000
        cells = rng.choice(W * H * D, n, replace=False)
        xyz = np.stack([cells % W, (cells // W) % H, cells // (W * H)], 1) + np.array(origin)
        blk = rng.choice([0, 3, 4, 1, 2], n, p=[0.5, 0.3, 0.1, 0.05, 0.05]).astype(np.uint8)
        # torch columns spanning the whole height inside one tile
        ty = np.arange(2, H - 1, 23)
        txyz = np.stack([np.full_like(ty, 5), ty, np.full_like(ty, 6)], 1) + np.array(origin)
        xyz = np.concatenate([xyz, txyz])
        blk = np.concatenate([blk, np.full(len(ty), 4, np.uint8)])
        per.append((xyz, blk))
        lists.append(B.make_overrides(xyz, blk, env=e))
    wb.generate(seeds, np.concatenate(lists))
    wb.sync()
    for e in range(E):
        spec = WorldSpec(int(seeds[e]), W, H, D, origin=origin, terrain=terrain, base=base, amplitude=amp)
        blocks, bl, sl, hm = oracle.generate(spec, *per[e], method="multi")
        _assert_world(wb, e, blocks, bl, sl, hm, f"env{e}")
    wb.close()


def test_duplicates_outside_and_invalid_overrides(B, oracle):
    """Latest duplicate wins; overrides outside the region or with unknown ids are ignored."""
    cfg = B.WorldConfig(num_envs=2, width=40, height=64, depth=33, terrain=TERRAIN_FLAT, base=20)
    wb = B.WorldBatch(cfg)
    o = B.make_overrides([[5, 21, 5], [5, 21, 5], [5, 21, 5], [-1, 21, 5], [5, 64, 5], [5, 25, 40], [6, 21, 6],
                          [7, 21, 7], [1, 21, 1]],
                         [3, 0, 4, 4, 4, 4, 9, 3, 4], env=[0, 0, 0, 0, 0, 0, 0, 5, 1])
    wb.generate([3, 4], o)
    wb.sync()
    spec = WorldSpec(3, 40, 64, 33, terrain=TERRAIN_FLAT, base=20)
    blocks, bl, sl, hm = oracle.generate(spec, [[5, 21, 5]], [4], method="multi")
    _assert_world(wb, 0, blocks, bl, sl, hm, "env0")
    spec = WorldSpec(4, 40, 64, 33, terrain=TERRAIN_FLAT, base=20)
    blocks, bl, sl, hm = oracle.generate(spec, [[1, 21, 1]], [4], method="multi")
    _assert_world(wb, 1, blocks, bl, sl, hm, "env1")
    wb.close()


def test_dense_column_overrides_deterministic(B, oracle):
    """Many overrides per column, duplicates included (latest wins), several
    runs: the per-column sort must be race-free and the result deterministic."""
    W, H, D = 40, 64, 40
    cfg = B.WorldConfig(num_envs=2, width=W, height=H, depth=D, terrain=TERRAIN_FBM, base=30, amplitude=10.0)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(99)
    n = 20000
    cols = rng.integers(0, 400, n)
    x, z = (cols % 20) * 2, (cols // 20) * 2
    y = rng.integers(0, H, n)
    blk = rng.choice([0, 3, 4, 2], n).astype(np.uint8)
    env = rng.integers(0, 2, n).astype(np.uint16)
    xyz = np.stack([x, y, z], 1)
    o = B.make_overrides(xyz, blk, env=env)
    want = []
    for e in range(2):
        sel = env == e
        spec = WorldSpec(e + 1, W, H, D, terrain=TERRAIN_FBM, base=30, amplitude=10.0)
        want.append(oracle.generate(spec, xyz[sel], blk[sel], method="multi"))
    for run in range(3):
        wb.generate([1, 2], o)
        wb.sync()
        for e in range(2):
            _assert_world(wb, e, *want[e], f"run{run} env{e}")
    wb.close()


@pytest.mark.parametrize("base", [-5, 200, 31])
def test_empty_and_full_worlds(B, oracle, base):
    cfg = B.WorldConfig(num_envs=1, width=33, height=32, depth=31, terrain=TERRAIN_FLAT, base=base)
    wb = B.WorldBatch(cfg)
    wb.generate([1], B.make_overrides([[0, 0, 0], [32, 31, 30]], B.TORCH))
    wb.sync()
    spec = WorldSpec(1, 33, 32, 31, terrain=TERRAIN_FLAT, base=base)
    blocks, bl, sl, hm = oracle.generate(spec, [[0, 0, 0], [32, 31, 30]], [4, 4], method="per_source")
    _assert_world(wb, 0, blocks, bl, sl, hm, f"base{base}")
    wb.close()


def test_tiny_world(B, oracle):
    cfg = B.WorldConfig(num_envs=2, width=1, height=32, depth=1, terrain=TERRAIN_FLAT, base=3)
    wb = B.WorldBatch(cfg)
    wb.generate([1, 2], B.make_overrides([[0, 10, 0], [0, 2, 0]], [4, 0], env=[0, 1]))
    wb.sync()
    for e, (xyz, blk) in enumerate([([[0, 10, 0]], [4]), ([[0, 2, 0]], [0])]):
        spec = WorldSpec(e + 1, 1, 32, 1, terrain=TERRAIN_FLAT, base=3)
        _assert_world(wb, e, *oracle.generate(spec, xyz, blk, method="per_source"), f"env{e}")
    wb.close()


# ------------------------------------------------ reference golden fixture --
def test_reference_lighting_scenarios(B):
    """The 13 generations of the reference's lighting tests, against the
    reference's own output (fixture made by tests/golden/make_golden.py)."""
    if not os.path.exists(GOLDEN):
        pytest.skip("golden fixture missing")
    g = np.load(GOLDEN)
    names = sorted({k[: -len("_xyz")] for k in g.files if k.endswith("_xyz")})
    cfg = B.WorldConfig(num_envs=len(names), width=64, height=32, depth=64, origin=S.ORIGIN,
                        terrain=B.TERRAIN_REFERENCE)
    wb = B.WorldBatch(cfg)
    lists = [B.make_overrides(g[n + "_xyz"], g[n + "_blk"], env=i) for i, n in enumerate(names)]
    wb.generate(np.full(len(names), 23, np.uint32), np.concatenate(lists))
    wb.sync()
    for i, n in enumerate(names):
        _assert_world(wb, i, g[n + "_blocks"], g[n + "_block_light"], g[n + "_sky_light"], g[n + "_height_map"], n)
        vox, cnt, hdr = wb.render_voxels(i)
        v = vox.cpu().numpy().view(np.uint32)
        assert hdr == S.ORIGIN
        assert np.array_equal(v[np.lexsort((v[:, 2], v[:, 1], v[:, 0]))], g[n + "_voxels"]), n
    wb.close()


def test_reference_terrain_matches_reference_cuda_build(B):
    """Reference-terrain mode (fast __sinf/__cosf) against the reference's own sm_100a build."""
    from oracle.oracle import Reference, ref_available

    if not ref_available("cuda"):
        pytest.skip("reference CUDA build not present")
    R = Reference("cuda")
    seeds = [1, 17, 23, 4242, 99991]
    cfg = B.WorldConfig(num_envs=len(seeds), width=64, height=32, depth=64, origin=(-32, 0, -32),
                        terrain=B.TERRAIN_REFERENCE)
    wb = B.WorldBatch(cfg)
    wb.generate(np.array(seeds, np.uint32))
    wb.sync()
    for e, s in enumerate(seeds):
        r = R.generate(s, (-32, 0, -32), (64, 32, 64), max_voxels=64 * 32 * 64)
        _assert_world(wb, e, r["blocks"], r["block_light"], r["sky_light"], r["height_map"], f"seed{s}")
    wb.close()


def test_reference_terrain_with_torches_per_env_origins(B, oracle):
    """Config 0's region (64 x 128 x 64) in reference-terrain mode with 200
    surface torches, one batch whose envs each sit at their own origin (as the
    reference centres each env's region on its agent,
    src/world/WorldGenerator.cpp:13-21), against the reference's own sm_100a
    build per env: ids, height map, both lights and the render voxel list
    (src/world/WorldGenerator.cu:171-588, :221-303)."""
    from oracle.oracle import Reference, ref_available

    if not ref_available("cuda"):
        pytest.skip("reference CUDA build not present")
    R = Reference("cuda")
    W, H, D = 64, 128, 64
    seeds = [1, 23, 4242, 77]
    origins = np.array([[-32, 0, -32], [1000, -6, -77], [-4083, 3, 2048], [37, -20, 91]], np.int32)
    cfg = B.WorldConfig(num_envs=len(seeds), width=W, height=H, depth=D, terrain=B.TERRAIN_REFERENCE,
                        max_overrides=4096)
    wb = B.WorldBatch(cfg)
    torches = [oracle.place_torches(WorldSpec(s, W, H, D, origin=tuple(o), terrain=TERRAIN_REFERENCE), 200,
                                    B.torch_key(s)) for s, o in zip(seeds, origins)]
    assert all(len(t) == 200 for t in torches)
    ovr = np.concatenate([B.make_overrides(t, B.TORCH, env=e) for e, t in enumerate(torches)])
    wb.generate(np.array(seeds, np.uint32), ovr, origins=origins)
    wb.sync()
    assert np.array_equal(wb.origins.cpu().numpy()[:, :3], origins)
    for e, s in enumerate(seeds):
        r = R.generate(s, tuple(origins[e]), (W, H, D), torches[e], np.full(200, 4, np.uint8), runs=2,
                       max_voxels=W * H * D)
        _assert_world(wb, e, r["blocks"], r["block_light"], r["sky_light"], r["height_map"], f"env{e}")
        assert (r["block_light"] > 0).sum() > 10000
        vox, n, hdr = wb.render_voxels(e)
        assert hdr == tuple(int(v) for v in origins[e]) == r["header"]
        v = vox.cpu().numpy().view(np.uint32)
        key = lambda a: a[np.lexsort((a[:, 2], a[:, 1], a[:, 0]))]
        assert n == r["voxel_count"] and np.array_equal(key(v), key(r["voxels"]))
    # Moving two envs' regions (their agents walked off): the other envs keep
    # their worlds, the moved ones match the reference at the new origins.
    moved = np.array([[-28, 0, -40], [995, -6, -60]], np.int32)
    before = wb.ids[[0, 3]].clone()
    t_new = [oracle.place_torches(WorldSpec(seeds[e], W, H, D, origin=tuple(o), terrain=TERRAIN_REFERENCE), 200,
                                  B.torch_key(seeds[e])) for e, o in zip((1, 2), moved)]
    wb.generate_envs([1, 2], [seeds[1], seeds[2]], np.concatenate(
        [B.make_overrides(t, B.TORCH, env=e) for e, t in zip((1, 2), t_new)]), origins=moved)
    wb.sync()
    assert torch.equal(wb.ids[[0, 3]], before)
    for k, e in enumerate((1, 2)):
        r = R.generate(seeds[e], tuple(moved[k]), (W, H, D), t_new[k], np.full(200, 4, np.uint8), runs=2)
        _assert_world(wb, e, r["blocks"], r["block_light"], r["sky_light"], r["height_map"], f"moved env{e}")
    wb.close()


# ------------------------------------------------------ edits and relight --
def _edit_batch(rng, E, W, H, D, n, origin, hm_list):
    lists, local = [], []
    for e in range(E):
        x = rng.integers(0, W, n)
        z = rng.integers(0, D, n)
        y = np.clip(hm_list[e][z, x] - origin[1] + rng.integers(-8, 9, n), -2, H + 1)
        kind = (rng.random(n) < 0.05).astype(np.uint8)
        blk = rng.choice([0, 3, 4], n, p=[0.47, 0.47, 0.06]).astype(np.uint8)
        xyz = np.stack([x, y, z], 1)
        local.append((xyz, kind, blk))
        lists.append(B_make(xyz + np.array(origin), blk, e, kind))
    return np.concatenate(lists), local


def B_make(xyz, blk, env, kind):
    import blocklab_b200 as B

    return B.make_overrides(xyz, blk, env=env, kind=kind)


@pytest.mark.parametrize("W,H,D", [(64, 32, 64), (96, 128, 70), (50, 256, 40)])
def test_edit_sequences_relight_exactly(B, oracle, W, H, D):
    """Dig / place / torch add / remove-torch edits near the surface, several
    steps, World::setBlock semantics incl. torch support; relit light must equal
    a full relight of the edited world."""
    E = 3
    origin = (-5, 0, 9)
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=origin, terrain=TERRAIN_FBM, base=H // 3,
                        amplitude=H / 4)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(W + H)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    specs = [WorldSpec(int(s), W, H, D, origin=origin, terrain=TERRAIN_FBM, base=H // 3, amplitude=H / 4)
             for s in seeds]
    torches = [oracle.place_torches(sp, 40, B.torch_key(int(s))) for sp, s in zip(specs, seeds)]
    wb.generate(seeds, np.concatenate([B.make_overrides(t, B.TORCH, env=e) for e, t in enumerate(torches)]))
    state = []
    for e in range(E):
        blocks, hm = oracle.build_blocks(specs[e], torches[e], np.full(len(torches[e]), 4, np.uint8))
        state.append([blocks, hm])
    for step in range(4):
        edits, local = _edit_batch(rng, E, W, H, D, 60, origin, [s[1] for s in state])
        wb.apply_edits(edits)
        wb.sync()
        for e in range(E):
            xyz, kind, blk = local[e]
            oracle.apply_edits(state[e][0], state[e][1], xyz, kind, blk, origin_y=origin[1])
            bl, sl = oracle.light(state[e][0], state[e][1], origin[1], "multi")
            _assert_world(wb, e, state[e][0], bl, sl, state[e][1], f"step{step} env{e}")
    wb.close()


@pytest.mark.parametrize("W,H,D,per_env", [(128, 64, 96, 2), (45, 96, 70, 1), (200, 128, 33, 3)])
def test_sparse_edits_relight_exactly(B, oracle, W, H, D, per_env):
    """A few edits per env (each relit through a box around the change rather
    than whole dirty tiles), including changes at region borders and torch
    support removal; several steps, compared with a full relight."""
    E = 4
    origin = (7, -3, -11)
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=origin, terrain=TERRAIN_FBM, base=H // 3,
                        amplitude=H / 5)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(W * H + per_env)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    specs = [WorldSpec(int(s), W, H, D, origin=origin, terrain=TERRAIN_FBM, base=H // 3, amplitude=H / 5)
             for s in seeds]
    torches = [oracle.place_torches(sp, 30, B.torch_key(int(s))) for sp, s in zip(specs, seeds)]
    wb.generate(seeds, np.concatenate([B.make_overrides(t, B.TORCH, env=e) for e, t in enumerate(torches)]))
    state = []
    for e in range(E):
        blocks, hm = oracle.build_blocks(specs[e], torches[e], np.full(len(torches[e]), 4, np.uint8))
        state.append([blocks, hm])
    for step in range(5):
        lists, local = [], []
        for e in range(E):
            n = per_env
            x = rng.integers(0, W, n)
            z = rng.integers(0, D, n)
            if step == 1:  # region borders and corners
                x[0], z[0] = [(0, 0), (W - 1, D - 1), (0, D - 1), (W - 1, 0)][e % 4]
            hm_l = state[e][1] - origin[1]
            y = np.clip(hm_l[z, x] + rng.integers(-3, 4, n), 0, H - 1)
            if step == 3:  # dig a torch's support
                t = torches[e][e % len(torches[e])] - np.array(origin)
                x[0], y[0], z[0] = t[0], t[1] - 1, t[2]
            blk = rng.choice([0, 3, 4], n, p=[0.5, 0.35, 0.15]).astype(np.uint8)
            if step == 3:
                blk[0] = 0
            kind = np.zeros(n, np.uint8)
            xyz = np.stack([x, y, z], 1)
            local.append((xyz, kind, blk))
            lists.append(B.make_overrides(xyz + np.array(origin), blk, env=e, kind=kind))
        wb.apply_edits(np.concatenate(lists))
        wb.sync()
        for e in range(E):
            xyz, kind, blk = local[e]
            oracle.apply_edits(state[e][0], state[e][1], xyz, kind, blk, origin_y=origin[1])
            bl, sl = oracle.light(state[e][0], state[e][1], origin[1], "multi")
            _assert_world(wb, e, state[e][0], bl, sl, state[e][1], f"step{step} env{e}")
    wb.close()


def test_edits_support_removal_and_heightmap(B, oracle):
    """Digging the block under a torch removes the torch; digging the top block
    lowers the height map (cells below become lit); placing above raises it."""
    cfg = B.WorldConfig(num_envs=1, width=40, height=32, depth=40, terrain=TERRAIN_FLAT, base=10)
    wb = B.WorldBatch(cfg)
    wb.generate([1], B.make_overrides([[20, 11, 20]], B.TORCH))
    blocks, hm = oracle.build_blocks(WorldSpec(1, 40, 32, 40, terrain=TERRAIN_FLAT, base=10), [[20, 11, 20]], [4])
    steps = [
        ([[20, 10, 20]], [0], [0]),                      # dig the support: torch goes too
        ([[5, 10, 5], [5, 9, 5], [5, 8, 5]], [0, 0, 0], [0, 0, 0]),  # shaft, lowers the top
        ([[30, 25, 30]], [3], [0]),                      # floating stone raises the top
        ([[30, 25, 30], [31, 12, 31]], [0, 4], [1, 0]),  # remove-torch on stone is a no-op; new torch
        ([[31, 12, 31]], [0], [1]),                      # remove the torch
    ]
    for xyz, blk, kind in steps:
        xyz = np.array(xyz)
        wb.apply_edits(B.make_overrides(xyz, np.array(blk, np.uint8), env=0, kind=np.array(kind, np.uint8)))
        wb.sync()
        oracle.apply_edits(blocks, hm, xyz, np.array(kind, np.uint8), np.array(blk, np.uint8))
        bl, sl = oracle.light(blocks, hm, 0, "per_source")
        _assert_world(wb, 0, blocks, bl, sl, hm, str(xyz.tolist()))
    wb.close()


def test_shaft_filled_bottom_up_in_one_step(B, oracle):
    """A 1-wide shaft open to the sky (26 deep, opaque walls) is filled with
    stone from the bottom up in one step. Each filled cell ends the step
    enclosed, but each one raised its column's top when it was placed, so all
    of them must be relit: the lit shaft cells go dark. A second env fills a
    sealed cave pocket, whose changes need no relight, beside an open one."""
    W, H, D = 40, 64, 40
    cfg = B.WorldConfig(num_envs=2, width=W, height=H, depth=D, terrain=TERRAIN_FLAT, base=40)
    wb = B.WorldBatch(cfg)
    wb.generate([1, 2])
    state = [list(oracle.build_blocks(WorldSpec(s, W, H, D, terrain=TERRAIN_FLAT, base=40))) for s in (1, 2)]
    shaft = np.array([[20, y, 20] for y in range(15, 41)])
    pocket = np.array([[x, 20, 10] for x in range(8, 12)] + [[30, 25, 30], [30, 26, 30]])
    steps = [
        [(shaft[::-1], 0), (pocket, 0)],  # dig the shaft top-down; dig a pocket and a 2-cell void
        [(shaft, 3), (pocket[::-1], 3)],  # fill both bottom-up / in reverse, one step
    ]
    for k, per_env in enumerate(steps):
        lists = []
        for e, (xyz, blk) in enumerate(per_env):
            lists.append(B.make_overrides(xyz, np.full(len(xyz), blk, np.uint8), env=e))
            oracle.apply_edits(state[e][0], state[e][1], xyz, np.zeros(len(xyz), np.uint8),
                               np.full(len(xyz), blk, np.uint8))
        wb.apply_edits(np.concatenate(lists))
        wb.sync()
        for e in range(2):
            bl, sl = oracle.light(state[e][0], state[e][1], 0, "multi")
            _assert_world(wb, e, state[e][0], bl, sl, state[e][1], f"step{k} env{e}")
    wb.close()


@pytest.mark.parametrize("axis", [0, 1, 2])
def test_relight_regions_at_merge_distance(B, oracle, axis):
    """Changes whose dirty cubes (L-inf 14 around each) are 28 .. 31 cells
    apart along one axis: at 29 and closer the cubes touch and their regions
    merge; at 30 and 31 they stay apart and share (30) or neighbour (31) a
    boundary layer whose light no change can reach. Torches and digs in open
    air and under ground, at the world's edges too, over three steps."""
    W, H, D = 100, 96, 100
    cfg = B.WorldConfig(num_envs=4, width=W, height=H, depth=D, terrain=TERRAIN_FLAT, base=40)
    wb = B.WorldBatch(cfg)
    wb.generate([1, 2, 3, 4])
    state = [list(oracle.build_blocks(WorldSpec(s, W, H, D, terrain=TERRAIN_FLAT, base=40))) for s in (1, 2, 3, 4)]
    for step, (y_a, blk) in enumerate([(48, 4), (40, 0), (48, 0)]):  # torches in air, dig the top, remove
        lists, local = [], []
        for e, gap in enumerate((28, 29, 30, 31)):
            xyz = np.array([[20, y_a, 20], [20, y_a, 20], [0, y_a, 99]])
            xyz[1, axis] += gap if axis != 1 else -gap  # vertical pairs go down, staying in the world
            b = np.full(len(xyz), blk, np.uint8)
            local.append((xyz, b))
            lists.append(B.make_overrides(xyz, b, env=e))
            oracle.apply_edits(state[e][0], state[e][1], xyz, np.zeros(len(xyz), np.uint8), b)
        wb.apply_edits(np.concatenate(lists))
        wb.sync()
        for e in range(4):
            bl, sl = oracle.light(state[e][0], state[e][1], 0, "multi")
            _assert_world(wb, e, state[e][0], bl, sl, state[e][1], f"axis{axis} step{step} env{e}")
    wb.close()


def test_apply_edits_requires_generate_and_capacity(B):
    cfg = B.WorldConfig(num_envs=1, width=32, height=32, depth=32, max_overrides=4, max_edits=2)
    wb = B.WorldBatch(cfg)
    with pytest.raises(B.BlkError) as ei:
        wb.apply_edits(B.make_overrides([[1, 1, 1]], 0))
    assert ei.value.status == 6
    with pytest.raises(B.BlkError) as ei:
        wb.generate([1], B.make_overrides(np.zeros((5, 3), np.int32), 0))
    assert ei.value.status == 4
    wb.generate([1], B.make_overrides(np.zeros((4, 3), np.int32), 0))
    with pytest.raises(B.BlkError) as ei:
        wb.apply_edits(B.make_overrides(np.zeros((3, 3), np.int32), 0))
    assert ei.value.status == 4
    wb.sync()
    wb.close()


# ------------------------------------------------ voxels and day/night --
def test_render_voxels_match_oracle(B, oracle):
    cfg = B.WorldConfig(num_envs=2, width=64, height=64, depth=48, terrain=TERRAIN_FBM, base=25, amplitude=15.0)
    wb = B.WorldBatch(cfg)
    rng = np.random.default_rng(11)
    lists, per = [], []
    for e in range(2):
        n = 800
        cells = rng.choice(64 * 64 * 48, n, replace=False)
        xyz = np.stack([cells % 64, (cells // 64) % 64, cells // (64 * 64)], 1)
        blk = rng.choice([0, 3, 4], n).astype(np.uint8)
        per.append((xyz, blk))
        lists.append(B.make_overrides(xyz, blk, env=e))
    wb.generate([5, 6], np.concatenate(lists))
    for e in range(2):
        spec = WorldSpec(5 + e, 64, 64, 48, terrain=TERRAIN_FBM, base=25, amplitude=15.0)
        blocks, bl, sl, hm = oracle.generate(spec, *per[e], method="multi")
        want = oracle.render_voxels(blocks, bl, sl)
        got, n, hdr = wb.render_voxels(e)
        assert n == len(want) and hdr == (0, 0, 0)
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want)
        # a too-small buffer reports the full count and writes a prefix
        got2, n2, _ = wb.render_voxels(e, max_voxels=100)
        assert n2 == n and np.array_equal(got2.cpu().numpy().view(np.uint32), want[:100])
    wb.close()


def test_effective_light(B):
    cfg = B.WorldConfig(num_envs=12, width=32, height=64, depth=32)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(12, dtype=np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, 20))
    ticks = np.linspace(11000, 24000, 12).astype(int)
    dim = np.array([B.sky_light_dimming(int(t)) for t in ticks], np.uint8)
    out = wb.effective_light(dim).cpu().numpy()
    light = wb.light.cpu().numpy()
    sky = light >> 4
    want = ((sky - np.minimum(sky, dim[:, None, None, None])) << 4) | (light & 15)
    assert np.array_equal(out, want.astype(np.uint8))
    assert set(dim.tolist()) >= {0, 11}
    wb.close()


# --------------------------------------------------- full benchmark size --
def _fixed_point_ok(ids, light, hmap, origin_y=0):
    """Light satisfies L = opaque ? 0 : max(src, max_N6 L - 1, 0) at every cell
    (cells outside the region count as opaque). This equation has exactly one
    solution: any positive level needs a neighbour one higher, so it is
    supported by a chain to a source and cannot exceed 15 - distance, and the
    equation forces at least 15 - distance. ids/light are (D, W, H) tensors."""
    opaque = (ids != 0) & (ids != 4)

    def nmax(L):
        P = F.pad(L, (1, 1, 1, 1, 1, 1))
        return torch.stack([P[:-2, 1:-1, 1:-1], P[2:, 1:-1, 1:-1], P[1:-1, :-2, 1:-1], P[1:-1, 2:, 1:-1],
                            P[1:-1, 1:-1, :-2], P[1:-1, 1:-1, 2:]]).amax(0)

    bl = (light & 15).to(torch.int16)
    sl = (light >> 4).to(torch.int16)
    zero = torch.zeros_like(bl)
    src_b = (ids == 4).to(torch.int16) * 15
    exp_b = torch.where(opaque, zero, torch.maximum(src_b, (nmax(bl) - 1).clamp(min=0)))
    y = torch.arange(ids.shape[2], device=ids.device, dtype=torch.int16) + origin_y
    lit = (y[None, None, :] > hmap[:, :, None]).to(torch.int16) * 15
    exp_s = torch.where(opaque, zero, torch.maximum(lit, (nmax(sl) - 1).clamp(min=0)))
    top = torch.where(opaque, y[None, None, :].expand_as(bl), torch.full_like(bl, -1)).amax(2)
    return bool((exp_b == bl).all()) and bool((exp_s == sl).all()) and bool((top.clamp(min=-1) == hmap).all())


def test_full_size_config1(B, oracle):
    """Benchmark size: 128 envs of 256 x 256 x 128 with 1000 torches each.
    Every env satisfies the light fixed point; two envs are compared
    cell-for-cell with the oracle."""
    cfg = B.WorldConfig(num_envs=128, width=256, height=128, depth=256, max_overrides=128 * 1000)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(1, 129, dtype=np.uint32)
    t = wb.place_torches(seeds, 1000)
    wb.generate(seeds, t)
    wb.sync()
    for e in range(128):
        assert _fixed_point_ok(wb.ids[e], wb.light[e], wb.height_map[e]), f"env {e}"
    assert int((wb.ids == 4).sum()) == 128 * 1000
    tn = t.cpu().numpy().view(B.OVERRIDE_DTYPE)
    for e in (0, 77):
        sel = tn[(tn["env"] == e) & (tn["y"] > -(1 << 30))]
        spec = WorldSpec(int(seeds[e]), 256, 128, 256)
        blocks, bl, sl, hm = oracle.generate(spec, _xyz(sel), sel["block"], method="multi")
        _assert_world(wb, e, blocks, bl, sl, hm, f"env{e}")
    wb.close()


def test_daynight_shape_cell_for_cell(B, oracle):
    """The day/night workload's worlds (128 x 96 x 128 with 300 surface torches),
    six envs of the benchmark's seeds, cell for cell against the oracle."""
    E, W, H, D = 6, 128, 96, 128
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * 300)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(1, 1 + E, dtype=np.uint32)
    t = wb.place_torches(seeds, 300)
    wb.generate(seeds, t)
    wb.sync()
    tn = t.cpu().numpy().view(B.OVERRIDE_DTYPE)
    for e in range(E):
        sel = tn[(tn["env"] == e) & (tn["y"] > -(1 << 30))]
        assert len(sel) == 300
        blocks, bl, sl, hm = oracle.generate(WorldSpec(int(seeds[e]), W, H, D), _xyz(sel), sel["block"],
                                             method="multi")
        _assert_world(wb, e, blocks, bl, sl, hm, f"env{e}")
    wb.close()


def test_relight_shape_edit_steps_cell_for_cell(B, oracle):
    """The relight workload's worlds (128^3, 200 surface torches) through six
    steps of its edit mix (45 % dig, 45 % stone, 5 % torch, 5 % removal of an
    existing torch, within 8 of the surface): four steps at its density (about
    ten edits per env: relight boxes) and two dense ones (whole dirty tiles),
    every env cell for cell against the oracle's full relight."""
    E, W, H, D = 5, 128, 128, 128
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * 200, max_edits=E * 400)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(1, 1 + E, dtype=np.uint32)
    t = wb.place_torches(seeds, 200)
    wb.generate(seeds, t)
    tn = t.cpu().numpy().view(B.OVERRIDE_DTYPE)
    state, torches = [], []
    for e in range(E):
        sel = tn[(tn["env"] == e) & (tn["y"] > -(1 << 30))]
        torches.append(_xyz(sel))
        state.append(list(oracle.build_blocks(WorldSpec(int(seeds[e]), W, H, D), _xyz(sel), sel["block"])))
    rng = np.random.default_rng(17)
    for step, per_env in enumerate([10, 10, 10, 10, 400, 400]):
        lists, local = [], []
        for e in range(E):
            x, z = rng.integers(0, W, per_env), rng.integers(0, D, per_env)
            y = state[e][1][z, x].astype(np.int64) + rng.integers(-8, 9, per_env)
            r = rng.random(per_env)
            blk = np.where(r < 0.45, 0, np.where(r < 0.9, 3, 4)).astype(np.uint8)
            kind = np.zeros(per_env, np.uint8)
            rm = r >= 0.95
            pick = torches[e][rng.integers(0, len(torches[e]), int(rm.sum()))]
            x[rm], y[rm], z[rm] = pick[:, 0], pick[:, 1], pick[:, 2]
            blk[rm], kind[rm] = 0, 1
            xyz = np.stack([x, y, z], 1)
            local.append((xyz, kind, blk))
            lists.append(B.make_overrides(xyz, blk, env=e, kind=kind))
        ovr = np.concatenate(lists)
        # Envs interleaved at random, each env's edits kept in their order.
        slots = ovr["env"][rng.permutation(len(ovr))]
        mixed = np.empty_like(ovr)
        for e in range(E):
            mixed[slots == e] = ovr[ovr["env"] == e]
        wb.apply_edits(mixed)
        wb.sync()
        for e in range(E):
            xyz, kind, blk = local[e]
            oracle.apply_edits(state[e][0], state[e][1], xyz, kind, blk)
            bl, sl = oracle.light(state[e][0], state[e][1], 0, "multi")
            _assert_world(wb, e, state[e][0], bl, sl, state[e][1], f"step{step} env{e}")
    wb.close()


def test_full_size_incremental_steps_fixed_point(B):
    """Config-2 shaped incremental steps (128^3 worlds, ~10 edits per env per
    step) keep the light field at its fixed point."""
    E = 64
    cfg = B.WorldConfig(num_envs=E, width=128, height=128, depth=128, max_edits=1 << 14)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(E, dtype=np.uint32) + 7
    wb.generate(seeds, wb.place_torches(seeds, 200))
    rng = np.random.default_rng(2)
    hm = wb.height_map.cpu().numpy()
    for step in range(5):
        n = 10 * E
        env = rng.integers(0, E, n)
        x, z = rng.integers(0, 128, n), rng.integers(0, 128, n)
        y = hm[env, z, x] + rng.integers(-8, 9, n)
        r = rng.random(n)
        blk = np.where(r < 0.45, 0, np.where(r < 0.9, 3, 4)).astype(np.uint8)
        kind = (r >= 0.95).astype(np.uint8)
        order = np.argsort(env, kind="stable")
        wb.apply_edits(B.make_overrides(np.stack([x, y, z], 1)[order], blk[order], env=env[order],
                                        kind=kind[order]))
    wb.sync()
    for e in range(E):
        assert _fixed_point_ok(wb.ids[e], wb.light[e], wb.height_map[e]), f"env {e}"
    wb.close()


def test_full_size_tall_worlds_fixed_point(B, oracle):
    """Scale-out shaped worlds: 256 x 256 x 256 with terrain amplitude 120 and
    2000 torches each (a slice of the env batch). Every env satisfies the light
    fixed point, one env matches the oracle cell for cell, then a step of
    edits keeps the fixed point."""
    E = 8
    cfg = B.WorldConfig(num_envs=E, width=256, height=256, depth=256, amplitude=120.0, max_overrides=E * 2000,
                        max_edits=E * 5000)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(100, 100 + E, dtype=np.uint32)
    t = wb.place_torches(seeds, 2000)
    wb.generate(seeds, t)
    wb.sync()
    for e in range(E):
        assert _fixed_point_ok(wb.ids[e], wb.light[e], wb.height_map[e]), f"env {e}"
    tn = t.cpu().numpy().view(B.OVERRIDE_DTYPE)
    sel = tn[(tn["env"] == 3) & (tn["y"] > -(1 << 30))]
    spec = WorldSpec(int(seeds[3]), 256, 256, 256, amplitude=120.0)
    blocks, bl, sl, hm = oracle.generate(spec, _xyz(sel), sel["block"], method="multi")
    _assert_world(wb, 3, blocks, bl, sl, hm, "env3")
    rng = np.random.default_rng(4)
    hmn = wb.height_map.cpu().numpy()
    n = 5000 * E
    env = np.repeat(np.arange(E), 5000)
    x, z = rng.integers(0, 256, n), rng.integers(0, 256, n)
    y = hmn[env, z, x] + rng.integers(-8, 9, n)
    r = rng.random(n)
    blk = np.where(r < 0.45, 0, np.where(r < 0.9, 3, 4)).astype(np.uint8)
    kind = (r >= 0.95).astype(np.uint8)
    wb.apply_edits(B.make_overrides(np.stack([x, y, z], 1), blk, env=env, kind=kind))
    wb.sync()
    for e in range(E):
        assert _fixed_point_ok(wb.ids[e], wb.light[e], wb.height_map[e]), f"env {e} after edits"
    wb.close()
