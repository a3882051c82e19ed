"""The tile loop (`--tile` / `--mem`, src/tile.rs of the reference).

CPU: tile::auto_tile's arithmetic, with the reference's own test cases
(tests/tiling.rs:146-207). GPU: a tile that covers the image is one tile and bit-equal to
the untiled pass; a margin that covers the image reproduces it exactly; and the tiled
pass matches the same tile loop run on the CPU oracle (src/tile.rs:47-105).
"""
import numpy as np
import pytest

import hat_b200
from golden_io import cases, checkpoint_for

WIN = 16


def test_auto_tile_reference_cases():
    per_pixel, constant = 1500, 15_000_000
    assert hat_b200.auto_tile(1024, 1024, WIN, 32 << 20, per_pixel, constant, 0) is None
    for budget in (1 << 30, 2 << 30, 4 << 30):
        t = hat_b200.auto_tile(1024, 1024, WIN, budget, per_pixel, constant, 0)
        assert t % WIN == 0
        assert t * t * per_pixel * 4 + constant * 4 <= budget
        up = t + WIN
        assert up * up > 1024 * 1024 or up * up * per_pixel * 4 + constant * 4 > budget
    assert hat_b200.auto_tile(1024, 1024, WIN, 64 << 30, per_pixel, constant, 0) == 1024
    assert hat_b200.auto_tile(64, 64, WIN, 64 << 30, per_pixel, constant, 0) == 64
    margin = 32
    for budget in (1 << 30, 2 << 30, 4 << 30):
        t = hat_b200.auto_tile(1024, 1024, WIN, budget, per_pixel, constant, margin)
        assert t % WIN == 0
        side = t + 2 * margin
        assert side * side > 1024 * 1024 or side * side * per_pixel * 4 + constant * 4 <= budget
        assert t <= hat_b200.auto_tile(1024, 1024, WIN, budget, per_pixel, constant, 0)
    t0 = hat_b200.auto_tile(1024, 1024, WIN, 1 << 30, per_pixel, constant, 0)
    exact = t0 * t0 * per_pixel * 4 + constant * 4
    assert hat_b200.auto_tile(1024, 1024, WIN, exact, per_pixel, constant, margin) < t0


def oracle_tiled(m, img, tile, margin, win=WIN):
    """src/tile.rs:47-105 over the oracle: cores of `tile`, `margin` of context each side
    (clamped to the image), each sub-image its own forward, cores copied unblended."""
    from oracle import hat_oracle as O
    _, h, w = img.shape
    s = m.scale
    step = max(-(-tile // win) * win, win)
    margin = -(-margin // win) * win
    out = np.zeros((3, h * s, w * s), np.float32)
    for y0 in range(0, h, step):
        for x0 in range(0, w, step):
            y1, x1 = min(y0 + step, h), min(x0 + step, w)
            sy0, sx0, sy1, sx1 = max(y0 - margin, 0), max(x0 - margin, 0), min(y1 + margin, h), min(x1 + margin, w)
            y = O.forward(m, img[:, sy0:sy1, sx0:sx1])
            dy, dx = (y0 - sy0) * s, (x0 - sx0) * s
            out[:, y0 * s:y1 * s, x0 * s:x1 * s] = y[:, dy:dy + (y1 - y0) * s, dx:dx + (x1 - x0) * s]
    return out


@pytest.fixture(scope="module")
def ck(tmp_path_factory):
    case = next(c for c in cases() if c["name"] == "hats_x4_48x48_p")
    return checkpoint_for(case, tmp_path_factory.mktemp("tile"))


@pytest.mark.gpu
def test_one_tile_and_covered_margin_are_exact(ck):
    from hat_b200 import synth
    be = hat_b200.B200(ck, device=0)
    img = synth.image(32, 32, 5)
    whole = be.forward(32, 32, img)
    for tile in (32, 64, 4096):
        got, info = be.forward_tiled(32, 32, img, tile, 0)
        assert info["tiles"] == 1
        assert np.array_equal(got, whole)
    got, info = be.forward_tiled(32, 32, img, WIN, 3 * WIN)
    assert info["tiles"] == 4 and info["largest_h"] == 32
    assert np.array_equal(got, whole)
    be.close()


@pytest.mark.gpu
def test_tiled_matches_oracle_tile_loop(ck):
    from hat_b200 import synth
    from oracle import hat_oracle as O
    m = O.Model.load(ck)
    be = hat_b200.B200(ck, device=0)
    img = synth.image(72, 56, 6)  # ragged: edge tiles of 8 rows / 24 columns
    got, info = be.forward_tiled(72, 56, img, 32, 2 * WIN)
    assert info["tiles"] == 6 and info["margin"] == 32 and info["tile"] == 32
    want = oracle_tiled(m, img, 32, 2 * WIN)
    assert float(np.abs(got - want).max()) <= 1e-4
    # The tiles differ from the untiled pass near their edges: the reference's
    # measurement (tests/tiling.rs:108-143) that margin is not exactness.
    whole = be.forward(72, 56, img)
    assert float(np.abs(got - whole).max()) > 0
    be.close()


@pytest.mark.gpu
def test_gpu_auto_tile_admits_the_whole_small_image(ck):
    be = hat_b200.B200(ck, device=0)
    assert be.gpu_auto_tile(64, 64) >= 64
    be.close()
