"""World edit scenarios of the reference's lighting tests, as override lists.

The reference's tests/WorldLighting.cpp builds its worlds through
World::setBlock on a seed-23 world and checks block-light masks of a region
centred at 0 (64 x 32 x 64, origin (-32, 0, -32)). This module replays the same
edit sequences with World::setBlock semantics (src/world/World.cpp:239-287) and
yields, per generation, the override list the reference would pass to its
generator (one override per edited cell, the latest value winning).

Each scenario is (name, seed, [generation]), and each generation carries the
check volumes (origin, size) in the order the reference test checks them.
"""
from __future__ import annotations

import numpy as np

ORIGIN = (-32, 0, -32)
SIZE = (64, 32, 64)
AIR, GRASS, DIRT, STONE, TORCH = 0, 1, 2, 3, 4


def _opaque(b: int) -> bool:
    return b not in (AIR, TORCH)


class Overlay:
    """Override map + World::setBlock semantics over a generated base region."""

    def __init__(self, base_blocks: np.ndarray) -> None:
        self.base = base_blocks  # (D, H, W) reference layout, local coords
        self.ovr: dict[tuple[int, int, int], int] = {}

    def block(self, p) -> int:
        if p in self.ovr:
            return self.ovr[p]
        x, y, z = p[0] - ORIGIN[0], p[1] - ORIGIN[1], p[2] - ORIGIN[2]
        if 0 <= x < SIZE[0] and 0 <= y < SIZE[1] and 0 <= z < SIZE[2]:
            return int(self.base[z, y, x])
        return AIR

    def set(self, p, b: int) -> None:
        if not 0 <= p[1] < SIZE[1]:
            return
        old = self.block(p)
        if old == b:
            return
        self.ovr[p] = b
        above = (p[0], p[1] + 1, p[2])
        if _opaque(old) and not _opaque(b) and self.block(above) == TORCH:
            self.set(above, AIR)

    def fill(self, origin, size, b: int) -> None:
        for y in range(size[1]):
            for z in range(size[2]):
                for x in range(size[0]):
                    self.set((origin[0] + x, origin[1] + y, origin[2] + z), b)

    def overrides(self):
        keys = sorted(self.ovr)
        xyz = np.array(keys, np.int32).reshape(-1, 3)
        blk = np.array([self.ovr[k] for k in keys], np.uint8)
        return xyz, blk


def _cave(o: Overlay, origin, size, wall=STONE):
    o.fill(origin, size, wall)
    o.fill((origin[0] + 1, origin[1] + 1, origin[2] + 1), (size[0] - 2, size[1] - 2, size[2] - 2), AIR)


CAVE_ORIGIN, CAVE_SIZE = (-4, 12, -4), (9, 7, 9)


def _cave_with_entrance(o: Overlay):
    _cave(o, CAVE_ORIGIN, CAVE_SIZE)
    for y in range(13, 16):
        for x in range(-1, 2):
            o.set((x, y, -4), AIR)


def _close_entrance(o: Overlay):
    for y in range(13, 16):
        for x in range(-1, 2):
            o.set((x, y, -4), STONE)


def _partially_close_entrance(o: Overlay):
    for y in range(13, 16):
        o.set((0, y, -4), STONE)


def scenarios(base_blocks: np.ndarray):
    """Yields (scenario, generation index, override xyz, override blocks, checks)."""
    # tests/WorldLighting.cpp:42-150
    o = Overlay(base_blocks)
    o.fill((-16, 0, -16), (33, 32, 33), AIR)
    o.set((0, 16, 0), TORCH)
    yield ("explicit_torch_volume", 0, *o.overrides(),
           [((-3, 13, -3), (7, 7, 7)), ((11, 14, 0), (5, 5, 1)), ((-2, 27, 0), (5, 5, 1))])

    # tests/WorldLighting.cpp:152-355
    o = Overlay(base_blocks)
    _cave_with_entrance(o)
    chk = [((-3, 13, -4), (7, 5, 6))]
    yield ("cave_outside_torch", 0, *o.overrides(), chk)
    o.set((0, 19, -3), TORCH)
    yield ("cave_outside_torch", 1, *o.overrides(), chk)
    _partially_close_entrance(o)
    yield ("cave_outside_torch", 2, *o.overrides(), chk)
    _close_entrance(o)
    yield ("cave_outside_torch", 3, *o.overrides(), chk)

    # tests/WorldLighting.cpp:357-511
    o = Overlay(base_blocks)
    _cave_with_entrance(o)
    o.set((0, 13, -2), TORCH)
    chk = [((-3, 13, -8), (7, 5, 6))]
    yield ("cave_inside_torch", 0, *o.overrides(), chk)
    _partially_close_entrance(o)
    yield ("cave_inside_torch", 1, *o.overrides(), chk)
    _close_entrance(o)
    yield ("cave_inside_torch", 2, *o.overrides(), chk)

    # tests/WorldLighting.cpp:513-758
    o = Overlay(base_blocks)
    o.fill((-4, 14, -2), (13, 5, 5), AIR)
    o.set((0, 15, 0), STONE)
    o.set((4, 15, 0), STONE)
    chk = [((-2, 12, -1), (9, 9, 3))]
    yield ("torch_transitions", 0, *o.overrides(), chk)
    o.set((0, 16, 0), TORCH)
    yield ("torch_transitions", 1, *o.overrides(), chk)
    o.set((4, 16, 0), TORCH)
    yield ("torch_transitions", 2, *o.overrides(), chk)
    o.set((4, 16, 0), AIR)
    yield ("torch_transitions", 3, *o.overrides(), chk)
    o.set((0, 15, 0), AIR)  # removes the torch above it
    assert o.block((0, 16, 0)) == AIR
    yield ("torch_transitions", 4, *o.overrides(), chk)


def parse_masks(path: str) -> list[list[str]]:
    """Mask layers of every checkBlockLight call of the reference test file, in order.

    Each call's last argument is a brace list of layers; a layer is one or more
    adjacent string literals (C++ concatenation)."""
    import re

    text = open(path).read()
    calls = []
    pos = 0
    while True:
        i = text.find("checkBlockLight(__LINE__", pos)
        if i < 0:
            break
        j = text.find("{\n", text.find("generated", i))
        depth, k = 0, j
        while True:
            if text[k] == "{":
                depth += 1
            elif text[k] == "}":
                depth -= 1
                if depth == 0:
                    break
            k += 1
        body = text[j + 1:k]
        body = re.sub(r"//[^\n]*", "", body)
        layers = []
        for part in body.split(","):
            lits = re.findall(r'"((?:[^"\\]|\\.)*)"', part)
            if lits:
                layers.append("".join(l.replace("\\n", "\n") for l in lits))
        calls.append(layers)
        pos = k
    return calls


def check_mask(blocks: np.ndarray, block_light: np.ndarray, origin, size, layers) -> list[str]:
    """Mismatches of one mask (reference tests/WorldTestUtils.cpp:192-235 rules)."""
    errors = []
    assert len(layers) == size[1]
    for ly, layer in enumerate(layers):
        rows = layer.split("\n")
        assert len(rows) == size[2], (len(rows), size)
        for lz, row in enumerate(rows):
            assert len(row) == size[0]
            for lx, c in enumerate(row):
                if c == ".":
                    continue
                x = origin[0] + lx - ORIGIN[0]
                y = origin[1] + ly - ORIGIN[1]
                z = origin[2] + lz - ORIGIN[2]
                b, l = int(blocks[z, y, x]), int(block_light[z, y, x])
                if c == "S":
                    if not _opaque(b) or l != 0:
                        errors.append(f"{(x, y, z)} want S got block {b} light {l}")
                else:
                    want = int(c, 16)
                    if _opaque(b) or l != want:
                        errors.append(f"{(x, y, z)} want {want} got block {b} light {l}")
    return errors
