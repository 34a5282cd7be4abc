"""The allocation-free render voxel entry point (blk_build_render_voxels_static)
against the context entry point blk_build_render_voxels on the same worlds.

Collected last on purpose: it must also pass after every other test of the
session has used the device."""
import ctypes

import numpy as np
import pytest
import torch

from blocklab_b200 import _native as N

BLK_ERR_INVALID_ARGUMENT = 1
BLK_ERR_CAPACITY = 4


def _call(ids, light, W, H, D, origin, vox, cap, cnt, hdr, stream=0):
    return N.lib.blk_build_render_voxels_static(ids, light, W, H, D, origin[0], origin[1], origin[2], vox, cap, cnt,
                                                hdr, stream)


def test_static_voxels_rejects_sizes_beyond_scratch():
    """Argument checks come before any device work (no GPU needed)."""
    p = ctypes.c_void_p(16)  # never dereferenced: the call is rejected first
    for W, H, D in [(65, 32, 8), (8, 32, 65), (8, 544, 8), (64, 520, 64)]:
        rc = _call(p, p, W, H, D, (0, 0, 0), p, 1, p, p)
        assert rc == BLK_ERR_CAPACITY, (W, H, D)
        assert "static scratch" in N.last_error()
    assert _call(None, p, 8, 32, 8, (0, 0, 0), p, 1, p, p) == BLK_ERR_INVALID_ARGUMENT
    assert _call(p, p, 0, 32, 8, (0, 0, 0), p, 1, p, p) == BLK_ERR_INVALID_ARGUMENT


@pytest.mark.gpu
def test_static_voxels_match_context_entry_on_consecutive_calls():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import blocklab_b200 as B

    W, H, D, E = 64, 128, 64, 2
    origin = (-7, 3, 11)
    cfg = B.WorldConfig(num_envs=E, width=W, height=H, depth=D, origin=origin, amplitude=60.0)
    wb = B.WorldBatch(cfg)
    seeds = np.array([5, 6], np.uint32)
    wb.generate(seeds, wb.place_torches(seeds, 300))
    wb.sync()
    dev = torch.device("cuda", 0)
    cap = W * H * D
    stream = torch.cuda.current_stream(dev).cuda_stream
    # Two calls in a row (the second reuses the scratch of the first), then
    # the first env again.
    for e in (0, 1, 0):
        want, n_want, hdr_want = wb.render_voxels(e)
        vox = torch.full((cap, 3), -1, dtype=torch.int32, device=dev)
        cnt = torch.full((1,), 0x7FFFFFFF, dtype=torch.int32, device=dev)
        hdr = torch.full((3,), -99, dtype=torch.int32, device=dev)
        rc = _call(wb.ids[e].data_ptr(), wb.light[e].data_ptr(), W, H, D, origin, vox.data_ptr(), cap,
                   cnt.data_ptr(), hdr.data_ptr(), stream)
        assert rc == 0, N.last_error()
        torch.cuda.synchronize(dev)
        n = int(cnt.item())
        assert n == n_want > 0, e
        assert tuple(hdr.tolist()) == hdr_want == origin
        assert torch.equal(vox[:n], want), e
        assert bool((vox[n:] == -1).all())
    # A capacity smaller than the list: the count is the full size, only the
    # first max_voxels entries are written.
    want, n_want, _ = wb.render_voxels(1)
    small = 1000
    vox = torch.full((small, 3), -1, dtype=torch.int32, device=dev)
    cnt = torch.zeros(1, dtype=torch.int32, device=dev)
    hdr = torch.zeros(3, dtype=torch.int32, device=dev)
    assert _call(wb.ids[1].data_ptr(), wb.light[1].data_ptr(), W, H, D, origin, vox.data_ptr(), small,
                 cnt.data_ptr(), hdr.data_ptr(), stream) == 0
    torch.cuda.synchronize(dev)
    assert int(cnt.item()) == n_want
    assert torch.equal(vox, want[:small])
    # A world in host memory is refused before any device work (the scratch
    # belongs to the current device).
    host_ids = wb.ids[1].cpu().numpy()
    assert _call(host_ids.ctypes.data, host_ids.ctypes.data, W, H, D, origin, vox.data_ptr(), small, cnt.data_ptr(),
                 hdr.data_ptr(), stream) == BLK_ERR_INVALID_ARGUMENT
    assert "device memory" in N.last_error()
    wb.close()
