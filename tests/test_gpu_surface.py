"""GPU tests of the generation paths: the surface kernel (one light word per
column, based at the column's first open row) and the tile kernel it hands the
tiles it cannot prove exact to. Every comparison is bit-exact: the two paths
against each other on the benchmark's world shapes, and the surface path
against the oracle on worlds built to sit at each edge of its conditions
(steps between neighbouring columns of 16 and 17 rows, torches 15 and 16 rows
above the surface, light running past the top of a column's word, caves)."""
import numpy as np
import pytest
import torch

from oracle.oracle import TERRAIN_FLAT, TERRAIN_REFERENCE, WorldSpec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


def _state(wb):
    return wb.ids.clone(), wb.light.clone(), wb.height_map.clone()


def _both_paths(B, cfg, seeds, make_overrides):
    """Generates the same batch on both paths; returns both states and the
    surface path's fallback tile count."""
    wb = B.WorldBatch(cfg)
    ovr = make_overrides(wb)
    wb.set_generation_path("surface")
    wb.generate(seeds, ovr)
    wb.sync()
    fallback = wb.generation_fallback_tiles()
    surface = _state(wb)
    wb.set_generation_path("tiles")
    wb.generate(seeds, ovr)
    wb.sync()
    assert wb.generation_fallback_tiles() == 0
    tiles = _state(wb)
    wb.close()
    return surface, tiles, fallback


def _assert_same(a, b, label):
    for name, x, y in zip(("ids", "light", "height map"), a, b):
        if not torch.equal(x, y):
            bad = (x != y).nonzero()[:5].tolist()
            raise AssertionError(f"{label}: {name} differ between the paths at {bad}")


@pytest.mark.parametrize("envs,W,H,D,base,amp,torches", [
    (3, 256, 128, 256, 40, 50.0, 1000),   # reset workload worlds
    (2, 256, 256, 256, 40, 120.0, 2000),  # scale-out worlds (steep terrain: some tiles fall back)
    (6, 128, 96, 128, 40, 50.0, 300),     # day/night worlds
    (6, 128, 128, 128, 40, 50.0, 200),    # relight workload worlds
    (4, 64, 128, 64, 40, 50.0, 200),      # config 0
    (4, 70, 32, 45, 20, 40.0, 100),       # surface above the region top in places, ragged tiles
])
def test_paths_agree_on_benchmark_worlds(B, envs, W, H, D, base, amp, torches):
    cfg = B.WorldConfig(num_envs=envs, width=W, height=H, depth=D, base=base, amplitude=amp,
                        max_overrides=envs * torches)
    seeds = np.arange(1, envs + 1, dtype=np.uint32)
    surface, tiles, fallback = _both_paths(B, cfg, seeds, lambda wb: wb.place_torches(seeds, torches))
    _assert_same(surface, tiles, f"{W}x{H}x{D}")
    n_tiles = envs * ((W + 31) // 32) * ((D + 31) // 32)
    if (W, H, D) == (256, 128, 256):
        assert fallback <= n_tiles // 20, f"{fallback} of {n_tiles} reset tiles left to the tile kernel"


def test_paths_agree_with_caves_and_reference_terrain(B):
    """Random caves, floating blocks and torches (most tiles fall back), and the
    reference's terrain formula with surface torches."""
    W, H, D, E = 96, 128, 80, 3
    rng = np.random.default_rng(5)

    def caves(wb):
        lists = []
        for e in range(E):
            cells = rng.choice(W * H * D, 3000, replace=False)
            xyz = np.stack([cells % W, (cells // W) % H, cells // (W * H)], 1)
            blk = rng.choice([0, 3, 4], len(cells), p=[0.6, 0.3, 0.1]).astype(np.uint8)
            lists.append(B.make_overrides(xyz, blk, env=e))
        return np.concatenate(lists)

    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * 3000)
    surface, tiles, fallback = _both_paths(B, cfg, [3, 4, 5], caves)
    _assert_same(surface, tiles, "caves")
    assert fallback > 0
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, terrain=TERRAIN_REFERENCE, max_overrides=E * 200)
    seeds = np.array([7, 8, 9], np.uint32)
    surface, tiles, _ = _both_paths(B, cfg, seeds, lambda wb: wb.place_torches(seeds, 200))
    _assert_same(surface, tiles, "reference terrain")


def _pillar_world(B, oracle, W, H, D, base, pillars, torches):
    """Flat terrain at `base` with stone pillars (x, z, height above the
    surface) and torches (x, y, z); generated on the surface path and checked
    cell for cell against the oracle. Returns the fallback tile count."""
    xyz, blk = [], []
    for x, z, h in pillars:
        for y in range(base + 1, base + 1 + h):
            xyz.append((x, y, z))
            blk.append(3)
    for t in torches:
        xyz.append(t)
        blk.append(4)
    xyz = np.array(xyz, np.int32).reshape(-1, 3)
    blk = np.array(blk, np.uint8)
    cfg = B.WorldConfig(num_envs=1, width=W, height=H, depth=D, terrain=TERRAIN_FLAT, base=base,
                        max_overrides=max(len(blk), 1))
    wb = B.WorldBatch(cfg)
    wb.set_generation_path("surface")
    wb.generate([1], B.make_overrides(xyz, blk))
    wb.sync()
    fallback = wb.generation_fallback_tiles()
    spec = WorldSpec(1, W, H, D, terrain=TERRAIN_FLAT, base=base)
    blocks, bl, sl, hm = oracle.generate(spec, xyz, blk, method="multi")
    ids = wb.ids[0].cpu().numpy().transpose(0, 2, 1)
    light = wb.light[0].cpu().numpy().transpose(0, 2, 1)
    assert np.array_equal(ids, blocks)
    assert np.array_equal(wb.height_map[0].cpu().numpy(), hm)
    assert np.array_equal(light & 15, bl), f"block light differs at {np.argwhere((light & 15) != bl)[:5].tolist()}"
    assert np.array_equal(light >> 4, sl)
    wb.close()
    return fallback


def test_steps_between_columns(B, oracle):
    """Pillars 16 rows tall (the largest step the surface path aligns) stay on
    it, with torches on and around them; 17 rows sends their tiles to the tile
    kernel. Light runs over the pillars and down their sides."""
    W, H, D, base = 64, 128, 64, 40
    torches = [(20, 41, 20), (22, base + 17, 22), (40, 41, 41), (12, 41, 50)]
    assert _pillar_world(B, oracle, W, H, D, base, [(21, 20, 16), (22, 22, 16), (41, 41, 16)], torches) == 0
    assert _pillar_world(B, oracle, W, H, D, base, [(21, 20, 17), (22, 22, 16), (41, 41, 3)], torches) > 0


def test_torch_height_above_surface(B, oracle):
    """Torches up to 15 rows above their column's first open row stay on the
    surface path (in a flat world their light ends inside the word); a torch
    16 rows up is left to the tile kernel from the start. On a 10-row pillar,
    light from a torch 9 rows above the pillar's top reaches the rows just
    above the neighbouring low columns' words at level 2, which the exactness
    test catches; from 8 rows up it reaches them at level 1 only, which
    spreads no further, and the tile stays on the surface path."""
    W, H, D, base = 64, 64, 64, 20
    assert _pillar_world(B, oracle, W, H, D, base, [], [(10, 21, 10), (30, 28, 30), (40, 36, 40)]) == 0
    assert _pillar_world(B, oracle, W, H, D, base, [], [(30, 37, 30)]) > 0
    assert _pillar_world(B, oracle, W, H, D, base, [(30, 30, 10)], [(30, 40, 30)]) > 0
    assert _pillar_world(B, oracle, W, H, D, base, [(30, 30, 10)], [(30, 39, 30)]) == 0


def test_light_into_pits(B, oracle):
    """A pit one step (16 rows) below a ledge: light from a torch on the ledge
    falls into the pit inside the pit columns' words (surface path). A pit two
    steps of 16 below an outer ledge: light from the outer ledge would reach
    rows above the pit bottom's words, and the exactness test hands the tile
    over. Both match the oracle."""
    W, H, D, base = 64, 128, 64, 40
    ring = [(x, z, 16) for x in range(24, 40) for z in range(24, 40) if not (30 <= x < 34 and 30 <= z < 34)]
    assert _pillar_world(B, oracle, W, H, D, base, ring, [(28, base + 17, 28), (33, base + 17, 29)]) == 0
    # Steps of 16 everywhere: pit, ring, outer ledge (32), rim (16), plain.
    outer = [(x, z, 32) for x in range(18, 46) for z in range(18, 46) if not (24 <= x < 40 and 24 <= z < 40)]
    rim = [(x, z, 16) for x in range(12, 52) for z in range(12, 52) if not (18 <= x < 46 and 18 <= z < 46)]
    assert _pillar_world(B, oracle, W, H, D, base, ring + outer + rim, [(23, base + 33, 31)]) > 0


def test_automatic_path_choice(B):
    """The default path takes the tile kernel for steep fBm terrain (no tile is
    reported as handed over) and the surface kernel otherwise."""
    seeds = np.arange(1, 3, dtype=np.uint32)
    for amp, steep in ((50.0, False), (120.0, True)):
        cfg = B.WorldConfig(num_envs=2, width=128, height=256, depth=128, amplitude=amp, max_overrides=2 * 300)
        wb = B.WorldBatch(cfg)
        wb.generate(seeds, wb.place_torches(seeds, 300))
        wb.sync()
        auto = _state(wb)
        n_auto = wb.generation_fallback_tiles()
        wb.set_generation_path("surface")
        wb.generate(seeds, wb.place_torches(seeds, 300))
        wb.sync()
        _assert_same(auto, _state(wb), f"amplitude {amp}")
        if steep:
            assert n_auto == 0 and wb.generation_fallback_tiles() > 0
        else:
            assert n_auto == wb.generation_fallback_tiles()
        wb.close()
