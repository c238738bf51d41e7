"""The encoder front end in the oracle (CPU): analysis tiling pinned to the layouts the
reference's own tests assert (src/encoder/tiles.rs, `matches_reference_layout` for 2096x1400
and `small_pictures_are_one_tile`), and `preprocess_rgb` against an independent numpy
restatement of colour.rs (float32 operations one by one, no fused multiply-adds)."""

import numpy as np
import pytest

import oracle as zo


def area(t, pre):
    return (t[pre + "_x"], t[pre + "_y"], t[pre + "_w"], t[pre + "_h"])


def test_analysis_tiles_reference_layout():
    luma = zo.analysis_tiles(0, 1400, 2096, 88, 131)
    assert [area(t, "img") for t in luma] == [
        (0, 0, 1024, 1024), (960, 0, 1024, 1024), (1920, 0, 176, 1024),
        (0, 960, 1024, 440), (960, 960, 1024, 440), (1920, 960, 176, 440)]
    assert area(luma[1], "lat") == (60, 0, 64, 64)
    assert area(luma[5], "lat") == (120, 60, 11, 28)
    assert sum(t["core_w"] * t["core_h"] for t in luma) == 88 * 131
    assert area(luma[0], "core") == (0, 0, 62, 62)
    assert (luma[1]["off_x"], luma[1]["off_y"]) == (2, 0)
    chroma = zo.analysis_tiles(1, 700, 1048, 88, 131)
    assert [area(t, "img") for t in chroma] == [
        (0, 0, 512, 512), (480, 0, 512, 512), (960, 0, 88, 512),
        (0, 480, 512, 220), (480, 480, 512, 220), (960, 480, 88, 220)]
    assert [area(t, "lat") for t in chroma] == [area(t, "lat") for t in luma]


def test_small_pictures_are_one_tile():
    for ccs, d in ((0, 1), (1, 2)):
        t = zo.analysis_tiles(ccs, 888 // d, 560 // d, 56, 35)
        assert len(t) == 1 and area(t[0], "core") == (0, 0, 35, 56)
    # exactly 1 MP (the batched-decode configuration's 1024 x 1024) is not tiled
    assert len(zo.analysis_tiles(0, 1024, 1024, 64, 64)) == 1
    assert len(zo.analysis_tiles(1, 512, 512, 64, 64)) == 1


@pytest.mark.parametrize("h,w", [(6, 10), (7, 9), (32, 48)])
def test_preprocess_rgb(h, w):
    rng = np.random.default_rng(h * w)
    rgb = rng.integers(0, 256, (h, w, 3), dtype=np.uint8)
    luma, chroma = zo.preprocess_rgb(rgb)
    f = np.float32
    r, g, b = (rgb[..., k].astype(f) / f(255) for k in range(3))
    y = (f(0.2126) * r + f(0.7152) * g) + f(0.0722) * b
    u = ((b - y) / f(1.8556) + f(0.5)) * f(255)
    v = ((r - y) / f(1.5748) + f(0.5)) * f(255)
    y = y * f(255)
    assert np.array_equal(luma[0], y)
    ph, pw = h + h % 2, w + w % 2
    for base, p in ((0, y), (4, u), (8, v)):
        pad = np.pad(p, ((0, ph - h), (0, pw - w)), mode="edge")
        for k in range(4):
            dy, dx = k // 2, k % 2
            assert np.array_equal(chroma[base + k], pad[dy::2, dx::2])


def test_analyze_tiled_one_tile_equals_untiled():
    import synthetic as syn
    pa, pauv = syn.analysis_params("bop", 4)
    x = np.floor(syn.uniform(9, "fe/x", (1, 48, 80), 0.0, 256.0)).astype(np.float32)
    ck = zo.Checkpoint(pa)
    assert np.array_equal(zo.analyze_tiled(ck, zo.BOP, 0, x), zo.analysis_primary(ck, zo.BOP, x))
