"""CPU tests of the C ABI library: it loads, exports every declared symbol, and
its host-only entry points and argument validation behave (no GPU needed)."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "blk_world.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(blk_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from blocklab_b200 import _native as N

    syms = declared_symbols()
    assert len(syms) >= 15
    lib = ctypes.CDLL(N.LIB_PATH)
    missing = [s for s in syms if not hasattr(lib, s)]
    assert missing == []
    assert set(syms) == set(N.SIGNATURES)


def test_sky_light_at_time_matches_oracle(oracle):
    import blocklab_b200 as B

    for t in range(0, 24000, 7):
        assert B.sky_light_at_time(t) == oracle.sky_light_at_time(t)
    assert B.sky_light_dimming(0) == 0 and B.sky_light_dimming(18000) == 11


def test_invalid_config_rejected_without_device():
    from blocklab_b200 import _native as N

    for bad in [dict(num_envs=0), dict(height=48), dict(height=288), dict(width=0), dict(terrain_mode=7)]:
        c = dict(num_envs=1, width=8, height=32, depth=8, terrain_mode=1)
        c.update(bad)
        cfg = N.WorldConfigC(c["num_envs"], c["width"], c["height"], c["depth"], 0, 0, 0, c["terrain_mode"], 40, 50.0,
                             16, 16)
        h = ctypes.c_void_p()
        rc = N.lib.blk_ctx_create(0, ctypes.byref(cfg), ctypes.byref(h))
        assert rc == 1, bad
        assert "unsupported configuration" in N.last_error()
    assert N.lib.blk_ctx_create(0, None, None) == 1


def test_null_context_errors():
    from blocklab_b200 import _native as N

    assert N.lib.blk_generate(None, None, None, None, 0, 0) == 1
    assert N.lib.blk_sync(None, 0) == 1
    assert N.lib.blk_apply_edits(None, None, 0, 0) == 1
    assert N.lib.blk_ctx_destroy(None) == 0


def test_override_record_layout():
    from blocklab_b200 import OVERRIDE_DTYPE, make_overrides

    o = make_overrides([[1, 2, 3], [-4, 5, -6]], [4, 0], env=[0, 7], kind=[0, 1])
    assert o.dtype == OVERRIDE_DTYPE and o.itemsize == 16
    raw = o.view(np.uint8).reshape(2, 16)
    assert raw[1, 12] == 7 and raw[1, 14] == 0 and raw[1, 15] == 1
    assert np.frombuffer(raw[1, :12].tobytes(), np.int32).tolist() == [-4, 5, -6]
