"""The library against the reference's OWN generator (its src/world/WorldGenerator.cu
built for sm_100a under oracle/_ref) on the benchmark's worlds.

The reference's terrain formula differs from the benchmark's fBm, so its
generator is given each world as a dense override list (every cell), which
bypasses its terrain and runs its block cache, height map and light
(src/world/WorldGenerator.cu:142-219, :364-588) on exactly our blocks. That
pins the light of the benchmark worlds, floating blocks, caves and edited
worlds included, to the reference itself rather than to the restatement; the
restatement is checked against the same outputs.
"""
import numpy as np
import pytest
import torch

from oracle.oracle import WorldSpec

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


@pytest.fixture(scope="module")
def R():
    from oracle.oracle import Reference, ref_available

    if not ref_available("cuda"):
        pytest.skip("reference CUDA build (oracle/_ref/libref_cuda.so) not present")
    return Reference("cuda")


def _ref_layout(wb, e):
    ids = wb.ids[e].cpu().numpy().transpose(0, 2, 1)  # (D, W, H) -> (D, H, W)
    light = wb.light[e].cpu().numpy().transpose(0, 2, 1)
    return np.ascontiguousarray(ids), light & 15, light >> 4, wb.height_map[e].cpu().numpy()


def _check_against_reference(wb, e, R, oracle, origin_y=0, label=""):
    ids, bl, sl, hm = _ref_layout(wb, e)
    r = R.light_blocks(ids, origin=(0, origin_y, 0))
    assert np.array_equal(r["blocks"], ids), label
    assert np.array_equal(r["height_map"], hm), f"{label} height map differs from the reference"
    assert np.array_equal(r["block_light"], bl), \
        f"{label} block light differs from the reference at {np.argwhere(r['block_light'] != bl)[:5].tolist()}"
    assert np.array_equal(r["sky_light"], sl), \
        f"{label} sky light differs from the reference at {np.argwhere(r['sky_light'] != sl)[:5].tolist()}"
    obl, osl = oracle.light(ids, hm, origin_y, "multi")
    assert np.array_equal(obl, bl) and np.array_equal(osl, sl), f"{label} oracle differs"
    return r


def test_benchmark_reset_world_lit_by_reference(B, R, oracle):
    """One env of the reset benchmark (256 x 128 x 256, fBm, 1000 surface
    torches), plus one of the same shape with caves, floating stone and
    buried torches drawn at random."""
    W, H, D = 256, 128, 256
    cfg = B.WorldConfig(num_envs=2, width=W, height=H, depth=D, max_overrides=2 * 1000 + 20000)
    wb = B.WorldBatch(cfg)
    seeds = np.array([1, 2], np.uint32)
    torches = wb.place_torches(seeds, 1000).cpu().numpy().view(B.OVERRIDE_DTYPE)
    rng = np.random.default_rng(8)
    n = 20000
    cells = rng.choice(W * H * D, n, replace=False)
    xyz = np.stack([cells % W, (cells // W) % H, cells // (W * H)], 1)
    blk = rng.choice([0, 3, 4], n, p=[0.6, 0.3, 0.1]).astype(np.uint8)
    wb.generate(seeds, np.concatenate([torches, B.make_overrides(xyz, blk, env=1)]))
    wb.sync()
    for e in range(2):
        r = _check_against_reference(wb, e, R, oracle, label=f"env{e}")
        assert (r["block_light"] > 0).sum() > 100000


def test_relight_workload_world_after_edits_lit_by_reference(B, R, oracle):
    """Relight benchmark worlds (128^3, 200 torches) after five steps of its
    edit mix, incrementally relit by the library: every env's light equals the
    reference generator's full light of the edited world."""
    E, W, H, D = 4, 128, 128, 128
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, max_overrides=E * 200, max_edits=E * 50)
    wb = B.WorldBatch(cfg)
    seeds = np.arange(1, 1 + E, dtype=np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, 200))
    rng = np.random.default_rng(23)
    for step in range(5):
        hm = wb.height_map.cpu().numpy()
        n = 12 * E
        env = np.repeat(np.arange(E), 12)
        x, z = rng.integers(0, W, n), rng.integers(0, D, n)
        y = hm[env, z, x] + rng.integers(-8, 9, n)
        r = rng.random(n)
        blk = np.where(r < 0.45, 0, np.where(r < 0.9, 3, 4)).astype(np.uint8)
        wb.apply_edits(B.make_overrides(np.stack([x, y, z], 1), blk, env=env))
    wb.sync()
    for e in range(E):
        _check_against_reference(wb, e, R, oracle, label=f"env{e}")


def test_origin_offset_world_lit_by_reference(B, R, oracle):
    """A world whose region starts below y = 0 (origin y = -20): the height map
    holds world y, the light is the same function of the blocks."""
    W, H, D = 96, 128, 80
    cfg = B.WorldConfig(num_envs=1, width=W, height=H, depth=D, origin=(0, -20, 0), amplitude=40.0)
    wb = B.WorldBatch(cfg)
    wb.generate(np.array([9], np.uint32), wb.place_torches(np.array([9], np.uint32), 150))
    wb.sync()
    _check_against_reference(wb, 0, R, oracle, origin_y=-20, label="origin y -20")
