"""Parity of the benchmarked configurations at their real sizes, through the C ABI.

Config 4 runs exactly what `bench.py` times: the 3840x2160 HOP picture (512/16 tiles, 40 of
them) through one zjai_synthesize_tiles_q call with device buffers, which batches the tiles by
shape (28 interior, 7 bottom 512x176, 4 right 368x512, the 368x176 corner) with per-picture
tensor maps and writes the cores as 8-bit samples from the final layers' epilogue. One tile of
each shape class is checked against the oracle (the reference's f32 path restated) at the
north star's gate: 8-bit samples within +-1 on >= 99.9% and PSNR >= 50 dB. Size-independent
properties cover the whole picture: every output sample is written by exactly the tiles' cores
(the result does not depend on the planes' initial contents) and two runs are identical.

Config 3 runs the SOP 1920x1080 4:2:0 picture as one tile (the bench's `sop1080`), whole
picture against the oracle at the same gate.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo


def psnr8(a, b):
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return 99.0 if mse == 0 else 10 * np.log10(255.0 ** 2 / mse)


def gate8(got, want):
    """got, want: 8-bit samples. Fraction within +-1, worst difference, PSNR."""
    d = np.abs(np.asarray(got, np.int32) - np.asarray(want, np.int32))
    return float(np.mean(d <= 1)), int(d.max()), psnr8(got, want)


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=16 << 30)
    yield e
    e.close()


def _oracle_tile(cky, ckuv, op, ly, luv, t, sv=2, sh=2):
    """The oracle's tile t: its luma core (rows, cols, f32) and its chroma core samples on the
    sv x sh grid, assembled like synthesize_luma_into / synthesize_chroma_into
    (reconstruct.rs:379-464)."""
    wy = np.ascontiguousarray(ly[:, t["lat_y"]:t["lat_y"] + t["lat_h"],
                                 t["lat_x"]:t["lat_x"] + t["lat_w"]])
    wuv = np.ascontiguousarray(luv[:, t["lat_y"]:t["lat_y"] + t["lat_h"],
                                   t["lat_x"]:t["lat_x"] + t["lat_w"]])
    py = zo.synthesis_primary(cky, op, wy, t["img_h"], t["img_w"])[0]
    puv = zo.synthesis_secondary(ckuv, op, wy, wuv, t["img_h"], t["img_w"])
    oy, ox, ch, cw = t["off_y"], t["off_x"], t["core_h"], t["core_w"]
    luma = py[oy:oy + ch, ox:ox + cw]
    ys = np.arange(-(-t["core_y"] // sv) * sv, t["core_y"] + ch, sv)
    xs = np.arange(-(-t["core_x"] // sh) * sh, t["core_x"] + cw, sh)
    sub = np.ix_(oy + ys - t["core_y"], ox + xs - t["core_x"])
    return luma, puv[0][sub], puv[1][sub], ys // sv, xs // sh


def test_config4_hop4k_tiled_q():
    import torch

    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder

    H, W, tile, overlap = 2160, 3840, 512, 16
    lh, lw = -(-H // 16), -(-W // 16)
    py, puv = syn.synthesis_params("hop", 3)
    ly = syn.laplace_latent(100, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(100, "luv", (96, lh, lw), 1.5)
    e = zj.Engine(0, arena_bytes=64 << 30)
    dec = Decoder(e, "hop", py, puv)
    try:
        tiles = zj.synthesis_tiles(H, W, lh, lw, tile, overlap)
        assert len(tiles) == 40
        shapes = sorted({(t["img_h"], t["img_w"]) for t in tiles})
        assert shapes == [(176, 368), (176, 512), (512, 368), (512, 512)]
        d_ly, d_luv = torch.from_numpy(ly).cuda(), torch.from_numpy(luv).cuda()
        runs = []
        for fill in (0, 255):  # every sample must come from a core, whatever was there
            planes = dec._planes(d_ly, H, W, 2, 2, 8)
            for p in planes:
                p.fill_(fill)
            dec.synthesize_tiles(d_ly, d_luv, tiles, H, W, out=planes, bit_depth=8)
            e.sync()
            runs.append([p.cpu().numpy() for p in planes])
        for a, b in zip(*runs):
            assert np.array_equal(a, b)
        gy, gu, gv = runs[0]
        cky, ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
        # one tile per shape class: interior (row 1, col 1), right column (row 2), bottom row
        # (col 3), the corner
        for i in (9, 23, 35, 39):
            t = tiles[i]
            luma, u, v, cy, cx = _oracle_tile(cky, ckuv, zo.HOP, ly, luv, t)
            r0, c0 = t["core_y"], t["core_x"]
            got_y = gy[r0:r0 + luma.shape[0], c0:c0 + luma.shape[1]]
            for got, want in ((got_y, luma), (gu[np.ix_(cy, cx)], u), (gv[np.ix_(cy, cx)], v)):
                frac, worst, p = gate8(got, zo.quantize_plane(want))
                assert frac >= 0.999 and p >= 50.0, (i, t["img_h"], t["img_w"], frac, worst, p)
    finally:
        dec.close()
        e.close()


def test_config3_sop1080_one_tile(eng):
    import synthetic as syn
    from zenjpegai_b200.decoder import Decoder

    H, W = 1080, 1920
    lh, lw = -(-H // 16), -(-W // 16)
    py, puv = syn.synthesis_params("sop", 2)
    ly = syn.laplace_latent(100, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(100, "luv", (96, lh, lw), 1.5)
    dec = Decoder(eng, "sop", py, puv)
    try:
        got = dec.synthesize(ly, luv, H, W, bit_depth=8)
        want = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.SOP, ly, luv, H, W)
        assert got[0].shape == (H, W) and got[1].shape == (H // 2, W // 2)
        for g, w in zip(got, want):
            frac, worst, p = gate8(g, zo.quantize_plane(w))
            assert frac >= 0.999 and p >= 50.0, (frac, worst, p)
    finally:
        dec.close()


def test_config2_upsample_stage(eng):
    """conv 3x3 192 -> 512 (bias) + depth-to-space 2, then two residual
    blocks (conv3x3 - LeakyReLU(0.01) - conv3x3 + skip) at 128 channels, on x [192, 68, 120]
    ~ N(0, 1) with He-normal weights (seed 1), through zjai_stage_forward, against the oracle's
    composition of the same layers at the layer tolerance (relative L2 <= 1e-3)."""
    import synthetic as syn
    import zenjpegai_b200 as zj

    prm = syn.upsample_stage_params(1)
    x = syn.normal(1, "x", (192, 68, 120))
    st = zj.Stage(eng, prm, shuffle=2, act=zj.ACT_NONE, res_act=zj.ACT_LEAKY)
    try:
        got = st.forward(x)
    finally:
        st.close()
    y = zo.pixel_shuffle(zo.conv2d(x, prm["conv.weight"], prm["conv.bias"], pad=(1, 1)), 2)
    for i in range(2):
        p = "res.%d." % i
        t = zo.leaky_relu(zo.conv2d(y, prm[p + "conv1.weight"], prm[p + "conv1.bias"],
                                    pad=(1, 1)))
        y = zo.add(zo.conv2d(t, prm[p + "conv2.weight"], prm[p + "conv2.bias"], pad=(1, 1)), y)
    assert got.shape == (128, 136, 240)
    err = float(np.linalg.norm(got.astype(np.float64) - y) / np.linalg.norm(y))
    assert err < 1e-3, err


def test_config1_conv_stage(eng):
    """BASELINE config 1 through the conv-stage entry (one conv, LeakyReLU in its epilogue,
    planar output straight from the epilogue) with device buffers, against the oracle."""
    import torch

    import synthetic as syn
    import zenjpegai_b200 as zj

    prm = syn.conv_layer_params(0)
    x = syn.uniform(0, "x", (128, 128, 128), -1.0, 1.0)
    st = zj.Stage(eng, prm, shuffle=1, act=zj.ACT_LEAKY)
    try:
        got = st.forward(torch.from_numpy(x).cuda())
        eng.sync()
        got = got.cpu().numpy()
    finally:
        st.close()
    want = zo.leaky_relu(zo.conv2d(x, prm["conv.weight"], prm["conv.bias"], pad=(1, 1)))
    err = float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want))
    assert err < 1e-3, err
    assert np.max(np.abs(got - want)) < 1e-2
