"""The CPU oracle against the reference's own golden vectors (torch-computed layer cases).

Mirrors `tests/nn_vectors.rs` of the reference: conv geometries (`:100-112`) and transposed
convs (`:114-118`) within max |d| / max(|y|, 1) < 2e-6 (`:55-62`); pixel shuffle bit-exact
(`:120-130`); bicubic align-corners bit-exact (`:163-187`).
"""

import os

import numpy as np
import pytest

import oracle as zo

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "nn_vectors.npz"))


def _close(got, want):
    assert got.shape == want.shape
    worst = float(np.max(np.abs(got - want) / np.maximum(np.abs(want), 1.0)))
    assert worst < 2e-6, worst


@pytest.mark.parametrize("name,stride,pad,groups", [
    ("conv3x3_s1_p1_bias", 1, (1, 1), 1),
    ("conv3x3_s1_p1_g4_nobias", 1, (1, 1), 4),
    ("conv3x3_depthwise", 1, (1, 1), 12),
    ("conv1x1_nobias", 1, (0, 0), 1),
    ("conv3x3_s2_p1_bias", 2, (1, 1), 1),
    ("conv2x2_s1_p0", 1, (0, 0), 1),
    ("conv1x3_p01_bias", 1, (0, 1), 1),
    ("conv3x1_p10_bias", 1, (1, 0), 1),
])
def test_conv2d_golden(name, stride, pad, groups):
    x, w, y = GOLDEN[name + "/x"], GOLDEN[name + "/w"], GOLDEN[name + "/y"]
    b = GOLDEN[name + "/b"] if name + "/b" in GOLDEN.files else None
    _close(zo.conv2d(x, w, b, stride=stride, pad=pad, groups=groups), y)


@pytest.mark.parametrize("name,stride,pad,op", [
    ("convt4x4_s2_p1_bias", 2, 1, 0),
    ("convt3x3_s2_p1_op1_bias", 2, 1, 1),
])
def test_conv_transpose2d_golden(name, stride, pad, op):
    x, w, y = GOLDEN[name + "/x"], GOLDEN[name + "/w"], GOLDEN[name + "/y"]
    b = GOLDEN[name + "/b"]
    _close(zo.conv_transpose2d(x, w, b, stride=stride, pad=pad, out_pad=op), y)


def test_pixel_shuffle_golden():
    x = GOLDEN["pixel_shuffle/x"]
    for r, key in ((2, "y2"), (4, "y4")):
        got = zo.pixel_shuffle(x, r)
        assert np.array_equal(got, GOLDEN["pixel_shuffle/" + key])


def test_bicubic_golden_bit_exact():
    for i in range(6):
        x = GOLDEN["bicubic_align_corners/x%d" % i]
        want = GOLDEN["bicubic_align_corners/y%d" % i]
        got = zo.resize_bicubic(x, want.shape[1], want.shape[2])
        assert got.tobytes() == want.tobytes(), i


def test_conv_threads_bit_identical():
    """Tier/thread bit-identity (fast_vs_reference.rs:31-39): the thread count never changes
    the bits."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((12, 9, 11)).astype(np.float32)
    w = rng.standard_normal((8, 12, 3, 3)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    zo.set_threads(1)
    a = zo.conv2d(x, w, b, pad=(1, 1))
    zo.set_threads(4)
    c = zo.conv2d(x, w, b, pad=(1, 1))
    zo.set_threads(1)
    assert a.tobytes() == c.tobytes()


def test_exp_matches_libm_closely():
    xs = np.linspace(-80, 80, 2001).astype(np.float32)
    got = zo.exp(xs)
    want = np.exp(xs.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 4e-7


def test_conv_against_float64():
    """A larger random conv agrees with an f64 evaluation to f32 rounding."""
    rng = np.random.default_rng(7)
    x = rng.uniform(-1, 1, (16, 20, 24)).astype(np.float32)
    w = (rng.standard_normal((24, 16, 3, 3)) / 12).astype(np.float32)
    b = rng.standard_normal(24).astype(np.float32) * 0.01
    got = zo.conv2d(x, w, b, pad=(1, 1))
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1)))
    want = np.zeros_like(got, dtype=np.float64) + b[:, None, None]
    for ky in range(3):
        for kx in range(3):
            want += np.einsum("oc,chw->ohw", w[:, :, ky, kx].astype(np.float64),
                              xp[:, ky:ky + 20, kx:kx + 24])
    assert np.max(np.abs(got - want)) < 1e-5


def test_layer_norm_and_attention_reference_formulas():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16, 5, 7)).astype(np.float32)
    w = rng.standard_normal(16).astype(np.float32)
    b = rng.standard_normal(16).astype(np.float32)
    got = zo.layer_norm_channels(x, w, b)
    xd = x.astype(np.float64)
    m = xd.mean(0)
    v = ((xd - m) ** 2).mean(0)
    want = (xd - m) / np.sqrt(v + 1e-5) * w[:, None, None] + b[:, None, None]
    assert np.max(np.abs(got - want)) < 1e-5
    qkv = rng.standard_normal((48, 6, 5)).astype(np.float32)
    t = rng.uniform(0.5, 2, 4).astype(np.float32)
    got = zo.channel_attention(qkv, 4, t)
    q, k, vv = qkv[:16].reshape(16, -1), qkv[16:32].reshape(16, -1), qkv[32:].reshape(16, -1)
    q = q / np.linalg.norm(q.astype(np.float64), axis=1, keepdims=True)
    k = k / np.linalg.norm(k.astype(np.float64), axis=1, keepdims=True)
    out = np.zeros((16, 30))
    for hd in range(4):
        s = q[hd * 4:hd * 4 + 4] @ k[hd * 4:hd * 4 + 4].T * t[hd]
        s = np.exp(s - s.max(1, keepdims=True))
        s /= s.sum(1, keepdims=True)
        out[hd * 4:hd * 4 + 4] = s @ vv[hd * 4:hd * 4 + 4]
    assert np.max(np.abs(got.reshape(16, -1) - out)) < 1e-5


def test_tiles_cfg4_grid():
    """4K, 512/16 tiling: 8 x 5 = 40 tiles (tiles.rs:39-119)."""
    t = zo.synthesis_tiles(2160, 3840, 135, 240, 512, 16)
    assert len(t) == 40
    widths = sorted({x["img_w"] for x in t})
    heights = sorted({x["img_h"] for x in t})
    assert widths == [368, 512] and heights == [176, 512]
    # cores tile the picture exactly once
    cover = np.zeros((2160, 3840), np.int32)
    for x in t:
        cover[x["core_y"]:x["core_y"] + x["core_h"], x["core_x"]:x["core_x"] + x["core_w"]] += 1
    assert (cover == 1).all()


@pytest.mark.parametrize("op,secondary", [("bop", False), ("bop", True), ("hop", False)])
def test_analysis_stages_compose(op, secondary):
    """The four analysis stages chained give the whole transform bit for bit (the per-stage
    GPU check runs them one at a time)."""
    import synthetic as syn
    pa, puv = syn.analysis_params(op, 4)
    ck = zo.Checkpoint(puv if secondary else pa)
    h, w = (20, 28) if secondary else (40, 56)
    x = np.floor(syn.uniform(1, "x", (12 if secondary else 1, h, w), 0, 256)).astype(np.float32)
    t = x
    for stage in range(1, 5):
        t = zo.analysis_stage(ck, zo.OPS[op], secondary, stage, t, h, w)
    whole = (zo.analysis_secondary if secondary else zo.analysis_primary)(ck, zo.OPS[op], x)
    assert np.array_equal(t, whole)


def test_lef_reference_unit_cases():
    """src/filters/lef.rs tests: torch's nearest indices for 56 -> 888 rows and 3 -> 3, a flat
    picture kept, a border sample above the range clamped, out-of-range indices rejected."""
    assert [zo.nearest_index(i, 56, 888) for i in (0, 15, 16, 887)] == [0, 0, 1, 55]
    assert [zo.nearest_index(i, 3, 3) for i in range(3)] == [0, 1, 2]
    y = np.full((4, 4), 128.0, np.float32)
    y[0, 0] = 300.0
    s = np.array([[[5000]]], np.int32)
    out = zo.lef(y, s, 0, 0)
    assert out[0, 0] == 255.0 and abs(out[3, 3] - 128.0) < 1e-4
    for bad in ((1, 0), (0, 4)):
        with pytest.raises(ValueError):
            zo.lef(y, s, *bad)


def test_icci_transforms_and_tiling():
    """The two-level Haar transform pair inverts to f32 rounding, and the oracle's filter
    tiling follows src/filters/icci.rs:68-96 (a short last tile takes 176 samples from its
    neighbour; impossible layouts are rejected)."""
    rng = np.random.default_rng(2)
    for _ in range(20):
        b = rng.uniform(0, 1, 16).astype(np.float32)
        assert np.abs(zo.idwt2_block(zo.dwt2_block(b)).reshape(16) - b).max() < 1e-6
    flat = np.full(16, 0.5, np.float32)
    bands = zo.dwt2_block(flat)
    assert bands[0] == 2.0 * 0.5 * 2.0 and np.all(bands[1:] == 0)  # DC only, scaled by 2 per level
    import synthetic as syn
    ck = zo.Checkpoint(syn.icci_params(1))
    y = u = v = np.full((200, 500), 100.0, np.float32)
    with pytest.raises(ValueError):
        zo.icci_filter(ck, ck, 1, 1, y, u, v, tile=64, overlap=8)
    zo.icci_filter(ck, None, 0, 0, y, u, v, tile=256, overlap=32)
