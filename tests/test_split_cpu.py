"""The decode kernel's split of the U * bpu blocks among its CTAs (`Split` in
rotatek_b200/csrc/decode_tc.cu, phantom count chosen in capi.cu's tc_shape),
restated in Python: every real block belongs to exactly one CTA, the ranges are
contiguous and in order, no range is empty under the host's size rule, and the
block -> CTA map that the merge uses to find a unit's first and last CTA agrees
with the ranges."""
import random

import pytest

UNIT_SWITCH_BLOCKS = 12   # capi.cu kUnitSwitchBlocks


def phantom_for(total, grid):
    return UNIT_SWITCH_BLOCKS if total // grid >= 16 * UNIT_SWITCH_BLOCKS else 0


def real_of(v, bpu, ph):
    u = v // (bpu + ph)
    off = v - u * (bpu + ph) - ph
    return u * bpu + max(off, 0)


def ranges(units, bpu, grid, ph):
    vtotal = units * (bpu + ph)
    return [real_of(c * vtotal // grid, bpu, ph) for c in range(grid + 1)]


def cta_of(blk, units, bpu, grid, ph):
    vtotal = units * (bpu + ph)
    u = blk // bpu
    v = u * (bpu + ph) + ph + (blk - u * bpu)
    return ((v + 1) * grid - 1) // vtotal


@pytest.mark.parametrize("units,bpu", [
    (128, 260),     # config 2: B=32 x 4 KV heads, 20 prompt/text + 240 visual blocks
    (64, 528),      # config 5, one rank at 8 GPUs: B=64 x 1 KV head, 32 + 496 blocks
    (32, 258),      # config 3 at batch 1
    (1, 5), (3, 1), (7, 33), (896, 20),
])
def test_split_covers_every_block_once(units, bpu):
    total = units * bpu
    grid = max(1, min(total, 148))
    ph = phantom_for(total, grid)
    lo = ranges(units, bpu, grid, ph)
    assert lo[0] == 0 and lo[-1] == total
    assert all(lo[c] < lo[c + 1] for c in range(grid)), "a CTA without blocks"
    for c in range(grid):
        for b in (lo[c], lo[c + 1] - 1):
            assert cta_of(b, units, bpu, grid, ph) == c


def test_split_random_shapes_and_forced_phantoms():
    rng = random.Random(0)
    for _ in range(300):
        units, bpu = rng.randint(1, 400), rng.randint(1, 700)
        total = units * bpu
        grid = max(1, min(total, 148))
        for ph in {0, phantom_for(total, grid)}:
            lo = ranges(units, bpu, grid, ph)
            assert lo[0] == 0 and lo[-1] == total
            assert all(lo[c] < lo[c + 1] for c in range(grid))
            blocks = rng.sample(range(total), min(total, 50))
            for b in blocks:
                c = cta_of(b, units, bpu, grid, ph)
                assert lo[c] <= b < lo[c + 1]


def test_phantoms_are_what_a_range_gives_up():
    # a CTA's real blocks = its share of the virtual blocks minus the phantom
    # positions (each unit's first 12) that fall in it; at config 2 the ranges
    # that hold no phantom are the longest
    units, bpu, grid, ph = 128, 260, 148, 12
    vtotal = units * (bpu + ph)
    lo = ranges(units, bpu, grid, ph)
    lengths = []
    for c in range(grid):
        v0, v1 = c * vtotal // grid, (c + 1) * vtotal // grid
        phantoms = sum(1 for v in range(v0, v1) if v % (bpu + ph) < ph)
        assert lo[c + 1] - lo[c] == (v1 - v0) - phantoms
        lengths.append((phantoms, lo[c + 1] - lo[c]))
    free = [n for k, n in lengths if k == 0]
    priced = [n for k, n in lengths if k == ph]
    assert free and priced and min(free) > max(priced)
