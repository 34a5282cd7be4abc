"""Headless frames: render parameters pinned to the reference's sky functions
(CPU), and the CUDA ray cast against the CPU restatement of the voxel
pipeline's shading (GPU, within a stated tolerance: pixel colours go through
powf / tanf, whose last bits differ between device and host)."""
import os

import numpy as np
import pytest
import torch

from oracle.oracle import HERE as ORACLE_DIR
from oracle.oracle import TERRAIN_FBM, WorldSpec

LIGHTING_LIB = os.path.join(ORACLE_DIR, "_ref", "libref_lighting.so")


@pytest.mark.skipif(not os.path.exists(LIGHTING_LIB), reason="reference sky functions not built")
def test_render_params_match_reference_sky_and_camera():
    import blocklab_b200 as B
    from oracle.oracle import ReferenceLighting

    ref = ReferenceLighting()
    rng = np.random.default_rng(0)
    for t in list(range(0, 24000, 37)) + [12000, 13702, 22300, 23961, 6000, 18000, 23999]:
        yaw, pitch = float(rng.uniform(-3.2, 3.2)), float(rng.uniform(-1.5, 1.5))
        p = B.render_params_at((1.5, 40.0, -7.25), yaw, pitch, t)
        assert np.allclose(p["sky_color"], ref.sky_color(t), atol=2e-6), t
        assert np.allclose(p["sky_light_direction"], ref.sky_direction(t), atol=2e-6), t
        assert p["sky_light_dimming"] == 15 - ref.sky_light(t)
        # src/graphics/Renderer.cpp:76-80, 773-778
        f = np.array([np.sin(yaw) * np.cos(pitch), np.sin(pitch), np.cos(yaw) * np.cos(pitch)])
        f /= np.linalg.norm(f)
        r = np.array([np.cos(yaw), 0.0, -np.sin(yaw)])
        u = np.cross(f, r)
        u /= np.linalg.norm(u)
        assert np.allclose(p["forward"], f, atol=1e-6) and np.allclose(p["right"], r, atol=1e-6)
        assert np.allclose(p["up"], u, atol=1e-6)
        assert np.allclose(p["origin"], [1.5, 41.62, -7.25])
        assert (p["far_plane"], p["fog_start"], p["fog_end"]) == (48.0, 10.0, 28.0)
        assert np.isclose(p["fov_radians"], np.pi / 2.25)


def _srgb8(c):
    c = np.clip(np.float32(c), 0, 1)
    s = np.where(c <= 0.0031308, 12.92 * c, 1.055 * np.power(c, 1 / 2.4) - 0.055)
    return np.rint(s * 255).astype(np.uint8)


def test_oracle_frame_of_empty_world_is_sky(oracle):
    import blocklab_b200 as B

    spec = WorldSpec(1, 16, 32, 16, terrain=2, base=-5)  # flat terrain below the region: all air
    blocks, hm = oracle.build_blocks(spec)
    bl, sl = oracle.light(blocks, hm, 0, "multi")
    p = B.render_params_at((8, 10, 8), 0.4, 0.2, 13000)
    img = oracle.render_frame(spec, blocks, bl, sl, p.tobytes(), 40, 30)
    assert (img[..., :3] == _srgb8(p["sky_color"])).all() and (img[..., 3] == 255).all()


def _cameras(B, W, H, D, origin, rng, n):
    cams = []
    for k in range(n):
        if k % 4 == 0:   # above the region looking down
            pos = (origin[0] + W / 2, origin[1] + H + 4, origin[2] + D / 2)
            yaw, pitch = rng.uniform(-3, 3), -1.2
        elif k % 4 == 1:  # outside the region looking in
            pos = (origin[0] - 6, origin[1] + H * 0.6, origin[2] + D / 2)
            yaw, pitch = 1.4, -0.3
        else:             # inside, anywhere (possibly inside a block)
            pos = (origin[0] + rng.uniform(0, W), origin[1] + rng.uniform(0, H), origin[2] + rng.uniform(0, D))
            yaw, pitch = rng.uniform(-3.2, 3.2), rng.uniform(-1.0, 1.0)
        cams.append(B.render_params_at(pos, yaw, pitch, int(rng.integers(0, 24000))))
    return np.array(cams, B.RENDER_PARAMS_DTYPE)


@pytest.mark.gpu
def test_frames_match_oracle(oracle):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200 as B

    W, H, D, E = 48, 64, 40, 6
    origin = (-20, 0, 11)
    rng = np.random.default_rng(5)
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=origin, terrain=TERRAIN_FBM, base=28,
                        amplitude=14.0)
    wb = B.WorldBatch(cfg)
    seeds = rng.integers(1, 1 << 31, E).astype(np.uint32)
    lists, per = [], []
    for e in range(E):
        n = 1500
        cells = rng.choice(W * H * D, n, replace=False)
        xyz = np.stack([cells % W, (cells // W) % H, cells // (W * H)], 1) + np.array(origin)
        blk = rng.choice([0, 3, 4, 1, 2], n, p=[0.5, 0.2, 0.2, 0.05, 0.05]).astype(np.uint8)
        per.append((xyz, blk))
        lists.append(B.make_overrides(xyz, blk, env=e))
    wb.generate(seeds, np.concatenate(lists))
    params = _cameras(B, W, H, D, origin, rng, E)
    width, height = 160, 90
    frames = wb.render(params, width, height).cpu().numpy()
    assert frames.shape == (E, height, width, 4)
    total_bad = 0
    for e in range(E):
        spec = WorldSpec(int(seeds[e]), W, H, D, origin=origin, terrain=TERRAIN_FBM, base=28, amplitude=14.0)
        blocks, bl, sl, _ = oracle.generate(spec, *per[e], method="multi")
        want = oracle.render_frame(spec, blocks, bl, sl, params[e].tobytes(), width, height)
        diff = np.abs(frames[e].astype(np.int16) - want.astype(np.int16)).max(axis=2)
        bad = int((diff > 2).sum())
        total_bad += bad
        # tolerance: colours within 2 levels on >= 99.5 % of the pixels (edge pixels where
        # device and host float steps pick different faces account for the rest)
        assert bad <= 0.005 * width * height, (e, bad)
        assert (frames[e][..., 3] == 255).all()
    # the scenes are not trivial: faces, sky and torch light all appear
    assert len(np.unique(frames[..., :3].reshape(-1, 3), axis=0)) > 1000
    wb.close()


@pytest.mark.gpu
def test_render_then_convert_pipeline():
    """Rendered frames feed the observation conversion unchanged."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200 as B

    cfg = B.WorldConfig(num_envs=2, width=64, height=64, depth=64, origin=(-32, 0, -32))
    wb = B.WorldBatch(cfg)
    wb.generate([3, 4], wb.place_torches([3, 4], 50))
    params = np.array([B.render_params_at((0, 45, 0), 0.2 * e, -0.3, 1000) for e in range(2)], B.RENDER_PARAMS_DTYPE)
    frames = wb.render(params, 84, 84)
    obs = B.convert_rgba8_to_float_nchw(frames)
    torch.cuda.synchronize()
    assert obs.shape == (2, 3, 84, 84)
    assert torch.equal(obs[:, 0], frames[..., 0].float() * np.float32(1.0 / 255.0))
    with pytest.raises(ValueError):
        wb.render(params[:1], 84, 84)
    wb.close()


@pytest.mark.gpu
def test_render_observations_equal_converted_frames():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200 as B

    cfg = B.WorldConfig(num_envs=3, width=64, height=64, depth=64, origin=(-32, 0, -32))
    wb = B.WorldBatch(cfg)
    wb.generate([7, 8, 9], wb.place_torches([7, 8, 9], 60))
    params = np.array([B.render_params_at((e - 3.0, 44, 2.0), 1.1 * e, -0.35, 9000 * e) for e in range(3)],
                      B.RENDER_PARAMS_DTYPE)
    frames = wb.render(params, 96, 72)
    want = B.convert_rgba8_to_float_nchw(frames)
    got = wb.render_observations(params, 96, 72)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    wb.close()
