"""Generates tests/golden/lighting_scenarios.npz from the reference itself.

    python tests/golden/make_golden.py [--reference DIR]   (default: $BLOCKLAB_REFERENCE_DIR or /root/reference)

For every generation of the lighting-test scenarios (tests/golden/scenarios.py)
this runs the reference's own generator (its CUDA CPU-fallback build,
oracle/_ref/libref_cpu.so, compiled from the reference sources by
oracle/Makefile), checks the result against the block-light masks parsed from
the reference's tests/WorldLighting.cpp, and stores the reference's output
(override list, block ids, block light, sky light, height map) so the GPU
tests can compare against it on a machine without the reference.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import scenarios as S  # noqa: E402
from oracle.oracle import Reference  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("BLOCKLAB_REFERENCE_DIR", "/root/reference"))
    args = ap.parse_args()
    masks = S.parse_masks(os.path.join(args.reference, "tests", "WorldLighting.cpp"))
    R = Reference("cpu")
    base = R.generate(23, S.ORIGIN, S.SIZE)["blocks"]
    out = {}
    mask_i = 0
    for name, gen, xyz, blk, checks in S.scenarios(base):
        r = R.generate(23, S.ORIGIN, S.SIZE, xyz, blk, runs=2, max_voxels=64 * 32 * 64)
        for origin, size in checks:
            errs = S.check_mask(r["blocks"], r["block_light"], origin, size, masks[mask_i])
            if errs:
                raise SystemExit(f"{name}/{gen}: reference output disagrees with its own mask: {errs[:5]}")
            mask_i += 1
        key = f"{name}_{gen}"
        out[key + "_xyz"] = xyz
        out[key + "_blk"] = blk
        out[key + "_blocks"] = r["blocks"]
        out[key + "_block_light"] = r["block_light"]
        out[key + "_sky_light"] = r["sky_light"]
        out[key + "_height_map"] = r["height_map"]
        # The reference voxel order is nondeterministic: store it sorted.
        v = r["voxels"]
        out[key + "_voxels"] = v[np.lexsort((v[:, 2], v[:, 1], v[:, 0]))]
        print(f"{key}: {len(xyz)} overrides, {r['voxel_count']} voxels, masks ok")
    if mask_i != len(masks):
        raise SystemExit(f"checked {mask_i} masks of {len(masks)}")
    np.savez_compressed(os.path.join(HERE, "lighting_scenarios.npz"), **out)
    print(f"wrote lighting_scenarios.npz ({mask_i} reference masks verified)")


if __name__ == "__main__":
    main()
