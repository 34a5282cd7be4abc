"""The reference's world-overlay tests restated on this library's API.

reference tests/SmokeTest.cpp:
- 293-320 "World collision queries respect air and solid override masks";
- 322-333 "World can remove a solid block at the top height";
- 434-462 "World collects only overrides inside a requested region".

The reference worlds: its terrain formula, World::resetSeed(seed) as the env
seed, a 64 x 32 x 64 region (World::s_height = 32, src/world/World.h:30) centred
on the queried column as its agent-centred cache is (src/graphics/Renderer.cpp:45).
Each case also checks that the incrementally relit world equals a full
regeneration with the same edits given as overrides.
"""
import numpy as np
import pytest
import torch

from oracle.oracle import TERRAIN_REFERENCE

pytestmark = pytest.mark.gpu

AIR, STONE = 0, 3
MAX_Y = 31  # World::s_maxY of a 32-high world


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


def _world(B, seed, center):
    origin = (center[0] - 32, 0, center[2] - 32)
    cfg = B.WorldConfig(num_envs=1, width=64, height=32, depth=64, origin=origin, terrain=TERRAIN_REFERENCE)
    wb = B.WorldBatch(cfg)
    wb.generate(np.array([seed], np.uint32))
    wb.sync()
    return wb, cfg


def _cell(wb, xyz):
    block, light, height = wb.query_cells(np.array([xyz]))
    return int(block[0]), int(light[0]), int(height[0])


def _solid(wb, a, b):
    return int(wb.query_solid(np.array([a]), np.array([b]))[0])


def _set(B, wb, xyz, block):
    wb.apply_edits(B.make_overrides(np.array([xyz]), np.array([block], np.uint8), env=0))
    wb.sync()


def _assert_equals_regeneration(B, wb, cfg, seed, edits):
    """The relit world equals one generated from scratch with the edits as overrides."""
    ref = B.WorldBatch(cfg)
    xyz = np.array([e[0] for e in edits])
    blk = np.array([e[1] for e in edits], np.uint8)
    ref.generate(np.array([seed], np.uint32), B.make_overrides(xyz, blk, env=0))
    ref.sync()
    assert torch.equal(wb.ids, ref.ids)
    assert torch.equal(wb.height_map, ref.height_map)
    assert torch.equal(wb.light, ref.light)
    ref.close()


def test_collision_queries_respect_air_and_solid_overrides(B):
    seed, x, z = 17, 5, -3
    wb, cfg = _world(B, seed, (x, 0, z))
    ground_y = _cell(wb, (x, 0, z))[2]  # the column's height (World::terrainHeight here: no overrides yet)
    ground = (x, ground_y, z)
    assert _cell(wb, ground)[0] != AIR
    assert _solid(wb, ground, ground) == 1

    _set(B, wb, ground, AIR)
    assert _solid(wb, ground, ground) == 0
    assert _cell(wb, ground)[0] == AIR

    top = (x, MAX_Y, z)
    assert _cell(wb, top)[0] == AIR
    assert _solid(wb, top, top) == 0
    _set(B, wb, top, STONE)
    assert _solid(wb, top, top) == 1
    assert _cell(wb, top)[0] == STONE
    _assert_equals_regeneration(B, wb, cfg, seed, [(ground, AIR), (top, STONE)])
    wb.close()


def test_remove_solid_block_at_top_height(B):
    seed = 17
    top = (5, MAX_Y, -3)
    wb, cfg = _world(B, seed, (top[0], 0, top[2]))
    terrain_top = _cell(wb, top)[2]
    _set(B, wb, top, STONE)
    block, _, height = _cell(wb, top)
    assert block == STONE and height == MAX_Y
    _set(B, wb, top, AIR)
    block, light, height = _cell(wb, top)
    assert block == AIR
    assert height == terrain_top  # the height map falls back to the terrain
    assert light >> 4 == 15  # open sky again
    _assert_equals_regeneration(B, wb, cfg, seed, [])
    wb.close()


def test_overlay_holds_only_overrides_inside_a_requested_region(B):
    seed = 13
    wb, cfg = _world(B, seed, (32, 0, 32))  # region x, z in [0, 64): holds every edit below
    edits = [((1, 30, 1), STONE), ((9, 30, 1), STONE), ((1, 20, 1), STONE), ((40, 30, 40), STONE)]
    for xyz, blk in edits:
        _set(B, wb, xyz, blk)
    snap = wb.snapshot(0)
    coords = sorted((int(r["x"]), int(r["y"]), int(r["z"])) for r in snap)
    assert coords == sorted(xyz for xyz, _ in edits)
    # World::collectOverridesInRegion({0, 24, 0}, {16, 8, 16}) of the reference.
    inside = [c for c in coords if 0 <= c[0] < 16 and 24 <= c[1] < 32 and 0 <= c[2] < 16]
    assert inside == [(1, 30, 1), (9, 30, 1)]
    _assert_equals_regeneration(B, wb, cfg, seed, edits)
    wb.close()


def test_enclosed_dig_opened_later_in_the_same_step_is_relit(B):
    """An edit step digs a cell deep in the ground (enclosed when dug) and then
    the cells that connect it to the surface: judged by the step's final cells,
    it is no longer enclosed, so its light (now reached from the sky) must be
    relit. A second deep dig that stays enclosed changes no light. Both against
    a full regeneration with the same edits as overrides."""
    seed, x, z = 17, 5, -3
    wb, cfg = _world(B, seed, (x, 0, z))
    top = _cell(wb, (x, 0, z))[2]
    assert top >= 4
    shaft = [((x, y, z), AIR) for y in range(top - 3, top + 1)]  # deepest first: enclosed when dug
    sealed = [((x + 6, top - 3, z + 6), AIR)]                       # stays enclosed
    edits = shaft + sealed
    wb.apply_edits(B.make_overrides(np.array([e[0] for e in edits]), np.array([e[1] for e in edits], np.uint8),
                                    env=0))
    wb.sync()
    light = _cell(wb, (x, top - 3, z))[1]
    assert light >> 4 == 15  # the shaft bottom sees the sky
    _assert_equals_regeneration(B, wb, cfg, seed, edits)
    wb.close()
