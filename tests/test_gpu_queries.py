"""Sparse world queries (the physics' block / height / solid-box reads) and
overlay snapshots (save, restore by regeneration) on the GPU."""
import numpy as np
import pytest
import torch

from oracle.oracle import TERRAIN_FBM, WorldSpec

pytestmark = pytest.mark.gpu

W, H, D, E = 70, 64, 45, 3
ORIGIN = (-20, 4, 9)


@pytest.fixture(scope="module")
def B():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200

    return blocklab_b200


def _edited_world(B, oracle, rng):
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=ORIGIN, terrain=TERRAIN_FBM, base=30,
                        amplitude=18.0)
    wb = B.WorldBatch(cfg)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    lists = []
    for e in range(E):
        n = 800
        cells = rng.choice(W * H * D, n, replace=False)
        xyz = np.stack([cells % W, (cells // W) % H, cells // (W * H)], 1) + np.array(ORIGIN)
        blk = rng.choice([0, 3, 4, 1, 2], n, p=[0.5, 0.3, 0.1, 0.05, 0.05]).astype(np.uint8)
        lists.append(B.make_overrides(xyz, blk, env=e))
    wb.generate(seeds, np.concatenate(lists))
    hm = wb.height_map.cpu().numpy()
    edits = []
    for e in range(E):
        n = 50
        x, z = rng.integers(0, W, n), rng.integers(0, D, n)
        y = hm[e, z, x] - ORIGIN[1] + rng.integers(-4, 5, n)
        blk = rng.choice([0, 3, 4], n).astype(np.uint8)
        edits.append(B.make_overrides(np.stack([x, y, z], 1) + np.array(ORIGIN), blk, env=e))
    wb.apply_edits(np.concatenate(edits))
    wb.sync()
    return wb, seeds, cfg


def test_query_cells_match_resident_arrays(B, oracle):
    rng = np.random.default_rng(1)
    wb, _, _ = _edited_world(B, oracle, rng)
    ids = wb.ids.cpu().numpy()      # (E, D, W, H)
    light = wb.light.cpu().numpy()
    hm = wb.height_map.cpu().numpy()
    n = 4000
    env = rng.integers(0, E, n)
    lx, ly, lz = rng.integers(-5, W + 5, n), rng.integers(-5, H + 5, n), rng.integers(-5, D + 5, n)
    xyz = np.stack([lx, ly, lz], 1) + np.array(ORIGIN)
    block, lt, height = (t.cpu().numpy() for t in wb.query_cells(xyz, env))
    col = (lx >= 0) & (lx < W) & (lz >= 0) & (lz < D)
    inside = col & (ly >= 0) & (ly < H)
    assert inside.sum() > 1000 and (~inside).sum() > 100
    assert np.array_equal(block[inside], ids[env[inside], lz[inside], lx[inside], ly[inside]])
    assert np.array_equal(lt[inside], light[env[inside], lz[inside], lx[inside], ly[inside]])
    assert (block[~inside] == 255).all() and (lt[~inside] == 0).all()
    assert np.array_equal(height[col], hm[env[col], lz[col], lx[col]].astype(np.int32))
    assert (height[~col] == np.iinfo(np.int32).min).all()
    # an env index past the batch is outside
    b2, _, h2 = (t.cpu().numpy() for t in wb.query_cells([ORIGIN], E + 3))
    assert b2[0] == 255 and h2[0] == np.iinfo(np.int32).min
    wb.close()


def test_query_solid_matches_brute_force(B, oracle):
    rng = np.random.default_rng(2)
    wb, _, _ = _edited_world(B, oracle, rng)
    ids = wb.ids.cpu().numpy()
    solid = (ids != 0) & (ids != 4)
    n = 600
    env = rng.integers(0, E, n)
    lo = np.stack([rng.integers(-8, W + 2, n), rng.integers(-8, H + 2, n), rng.integers(-8, D + 2, n)], 1)
    size = rng.integers(0, 6, (n, 3))
    size[:10] = [[40, 70, 40]] * 10  # large boxes, partly outside
    hi = lo + size
    got = wb.query_solid(lo + np.array(ORIGIN), hi + np.array(ORIGIN), env).cpu().numpy()
    want = np.zeros(n, np.uint8)
    for i in range(n):
        x0, y0, z0 = np.maximum(lo[i], 0)
        x1, y1, z1 = np.minimum(hi[i], [W - 1, H - 1, D - 1])
        if x0 <= x1 and y0 <= y1 and z0 <= z1:
            want[i] = solid[env[i], z0:z1 + 1, x0:x1 + 1, y0:y1 + 1].any()
    assert np.array_equal(got, want)
    assert 0 < want.sum() < n
    wb.close()


def test_snapshot_restores_world(B, oracle, tmp_path):
    rng = np.random.default_rng(3)
    wb, seeds, cfg = _edited_world(B, oracle, rng)
    snaps = [wb.snapshot(e) for e in range(E)]
    for e, s in enumerate(snaps):
        assert len(s) > 0 and (s["env"] == e).all()
        key = (s["z"].astype(np.int64) * W + s["x"]) * H + s["y"]
        assert (np.diff(key) > 0).all()  # ascending (z, x, y), one record per cell
    path = tmp_path / "snap.npz"
    B.save_snapshot(str(path), seeds, np.concatenate(snaps), tick=123, config=cfg)
    seeds2, ovr2, tick = B.load_snapshot(str(path))
    assert tick == 123 and np.array_equal(seeds2, seeds)
    wb2 = B.WorldBatch(cfg)
    wb2.generate(seeds2, ovr2)
    wb2.sync()
    assert torch.equal(wb.ids, wb2.ids)
    assert torch.equal(wb.light, wb2.light)
    assert torch.equal(wb.height_map, wb2.height_map)
    # a snapshot of an untouched world is empty
    wb3 = B.WorldBatch(cfg)
    wb3.generate(seeds)
    assert len(wb3.snapshot(1)) == 0
    # capacity smaller than the overlay: full count, first records written
    dev = torch.device("cuda", 0)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.zeros(16 * 5, dtype=torch.uint8, device=dev)
    from blocklab_b200 import _native as N

    assert N.lib.blk_snapshot_overrides(wb._ctx, 0, out.data_ptr(), 5, cnt.data_ptr(), 0) == 0
    assert int(cnt.item()) == len(snaps[0])
    assert np.array_equal(out.cpu().numpy().view(B.OVERRIDE_DTYPE), snaps[0][:5])
    # host memory is refused for device-only arguments
    host = np.zeros(4, np.uint32)
    assert N.lib.blk_snapshot_overrides(wb._ctx, 0, out.data_ptr(), 5, host.ctypes.data, 0) == 1
    for w in (wb, wb2, wb3):
        w.close()


def test_readback_ranges(B, oracle):
    """blk_readback copies an env range of the resident arrays to host memory
    (the reference copies its whole block cache after every generation,
    src/world/WorldGenerator.cu:798-815): equal to the device arrays and to
    the oracle's world; outputs left out stay untouched; bad ranges fail."""
    rng = np.random.default_rng(5)
    cfg = B.WorldConfig(num_envs=4, width=W, height=H, depth=D, origin=ORIGIN, terrain=TERRAIN_FBM, base=30,
                        amplitude=18.0)
    wb = B.WorldBatch(cfg)
    seeds = rng.integers(1, 1 << 31, 4).astype(np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, 40))
    wb.sync()
    ids, light, hm = wb.readback(1, 2)
    torch.cuda.synchronize()
    assert ids.shape == (2, D, W, H) and hm.shape == (2, D, W)
    assert torch.equal(ids, wb.ids[1:3].cpu()) and torch.equal(light, wb.light[1:3].cpu())
    assert torch.equal(hm, wb.height_map[1:3].cpu())
    tl = wb.place_torches(seeds, 40).cpu().numpy().view(B.OVERRIDE_DTYPE)
    for k, e in enumerate((1, 2)):
        sel = tl[(tl["env"] == e) & (tl["y"] > -(1 << 30))]
        spec = WorldSpec(int(seeds[e]), W, H, D, origin=ORIGIN, terrain=TERRAIN_FBM, base=30, amplitude=18.0)
        blocks, bl, sl, hmap = oracle.generate(spec, np.stack([sel["x"], sel["y"], sel["z"]], 1), sel["block"],
                                               method="multi")
        l = light[k].numpy().transpose(0, 2, 1)
        assert np.array_equal(ids[k].numpy().transpose(0, 2, 1), blocks)
        assert np.array_equal(l & 15, bl) and np.array_equal(l >> 4, sl)
        assert np.array_equal(hm[k].numpy(), hmap)
    _, light_only, _ = wb.readback(3, 1, ids=False, height_map=False)
    torch.cuda.synchronize()
    assert torch.equal(light_only, wb.light[3:4].cpu())
    # device destination through the C ABI
    dst = torch.zeros((1, D, W, H), dtype=torch.uint8, device="cuda")
    from blocklab_b200 import _native as N

    N.check(N.lib.blk_readback(wb._ctx, 0, 1, dst.data_ptr(), None, None, 0))
    torch.cuda.synchronize()
    assert torch.equal(dst, wb.ids[0:1])
    with pytest.raises(B.BlkError):
        wb.readback(3, 2)
    wb.close()
