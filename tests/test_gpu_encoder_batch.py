"""GPU parity of the encoder front end and of picture batches (BASELINE config 5's path),
through the C ABI, against the CPU oracle (the reference's f32 path restated):

- `preprocess_rgb` (colour.rs) bit-exact;
- the batched RGB analysis (preprocess + both analysis transforms on n pictures as one batch)
  within the analysis gate, and each batch slot equal to a one-picture call;
- analysis tiling above 1 MP (encoder/tiles.rs) against the oracle's tiled analysis;
- batched synthesis of n pictures in one call (4:4:4, 8-bit) within the 8-bit gate, each slot
  equal to a one-picture zjai_synthesize_q;
- one config-5 picture (BOP 1024 x 1024 4:4:4) through both halves.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo

ANA_REL = 5e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def gate8(got, want):
    d = np.abs(np.asarray(got, np.int32) - np.asarray(want, np.int32))
    mse = float(np.mean(d.astype(np.float64) ** 2))
    return float(np.mean(d <= 1)), 99.0 if mse == 0 else 10 * np.log10(255.0 ** 2 / mse)


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=24 << 30)
    yield e
    e.close()


def _rgb(seed, n, h, w):
    import synthetic as syn
    return np.stack([np.floor(syn.uniform(seed + i + 1000, "rgb", (h, w, 3), 0.0, 256.0))
                     .astype(np.uint8) for i in range(n)])


@pytest.mark.parametrize("h,w", [(37, 50), (64, 64), (1, 3)])
def test_preprocess_rgb_bit_exact(eng, h, w):
    from zenjpegai_b200.decoder import preprocess_rgb
    rgb = _rgb(50, 1, h, w)[0]
    gl, gc = preprocess_rgb(eng, rgb)
    wl, wc = zo.preprocess_rgb(rgb)
    assert np.array_equal(gl, wl)
    assert np.array_equal(gc, wc)


def _encoder(eng, op="bop"):
    import synthetic as syn
    from zenjpegai_b200.decoder import Encoder
    pa, pauv = syn.analysis_params(op, 4)
    return Encoder(eng, op, pa, pauv), zo.Checkpoint(pa), zo.Checkpoint(pauv)


def test_analyze_rgb_batch(eng):
    enc, cka, ckc = _encoder(eng)
    try:
        rgb = _rgb(60, 3, 96, 160)
        gy, guv = enc.analyze_rgb(rgb)
        for i in range(3):
            luma, chroma = zo.preprocess_rgb(rgb[i])
            assert rel_l2(gy[i], zo.analysis_primary(cka, zo.BOP, luma)) < ANA_REL
            assert rel_l2(guv[i], zo.analysis_secondary(ckc, zo.BOP, chroma)) < ANA_REL
            # a batch slot equals the picture analysed alone
            sy, suv = enc.analyze_rgb(rgb[i:i + 1])
            assert np.array_equal(sy[0], gy[i]) and np.array_equal(suv[0], guv[i])
    finally:
        enc.close()


def test_analyze_rgb_tiled(eng):
    """1040 x 1024: 1.065 MP luma (tiles of 1024, overlap 64) and a 520 x 512 chroma plane
    above 262,144 samples (tiles of 512, overlap 32): both components are tiled."""
    enc, cka, ckc = _encoder(eng)
    try:
        rgb = _rgb(70, 1, 1040, 1024)
        assert len(zo.analysis_tiles(0, 1040, 1024, 65, 64)) == 2
        assert len(zo.analysis_tiles(1, 520, 512, 65, 64)) == 2
        gy, guv = enc.analyze_rgb(rgb)
        luma, chroma = zo.preprocess_rgb(rgb[0])
        zo.set_fast(True)
        zo.set_threads(16)
        try:
            wy = zo.analyze_tiled(cka, zo.BOP, 0, luma)
            wuv = zo.analyze_tiled(ckc, zo.BOP, 1, chroma)
        finally:
            zo.set_fast(False)
        assert gy.shape[1:] == wy.shape and guv.shape[1:] == wuv.shape
        assert rel_l2(gy[0], wy) < ANA_REL
        assert rel_l2(guv[0], wuv) < ANA_REL
    finally:
        enc.close()


def test_synthesize_batch(eng):
    import synthetic as syn
    from zenjpegai_b200.decoder import Decoder
    py, puv = syn.synthesis_params("bop", 4)
    dec = Decoder(eng, "bop", py, puv)
    try:
        H, W, n = 128, 192, 3
        ly = np.stack([syn.laplace_latent(100 + i, "ly", (160, H // 16, W // 16), 2.0)
                       for i in range(n)])
        luv = np.stack([syn.laplace_latent(100 + i, "luv", (96, H // 16, W // 16), 2.0)
                        for i in range(n)])
        gy, gu, gv = dec.synthesize_batch(ly, luv, H, W, sv=1, sh=1, bit_depth=8)
        cky, ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
        for i in range(n):
            want = zo.synthesize(cky, ckuv, zo.BOP, ly[i], luv[i], H, W, sv=1, sh=1)
            for got, w in zip((gy[i], gu[i], gv[i]), want):
                frac, p = gate8(got, zo.quantize_plane(w))
                assert frac >= 0.999 and p >= 50.0, (i, frac, p)
            one = dec.synthesize(ly[i], luv[i], H, W, sv=1, sh=1, bit_depth=8)
            for a, b in zip(one, (gy[i], gu[i], gv[i])):
                assert np.array_equal(a, b)
    finally:
        dec.close()


def test_config5_one_picture(eng):
    """BASELINE config 5's picture: BOP 1024 x 1024 4:4:4, latents Laplace(2.0) seed 100,
    weights seed 4; synthesis (one tile, 8-bit) and the RGB analysis against the oracle."""
    import synthetic as syn
    from zenjpegai_b200.decoder import Decoder
    py, puv = syn.synthesis_params("bop", 4)
    dec = Decoder(eng, "bop", py, puv)
    enc, cka, ckc = _encoder(eng)
    try:
        ly = syn.laplace_latent(100, "ly", (160, 64, 64), 2.0)[None]
        luv = syn.laplace_latent(100, "luv", (96, 64, 64), 2.0)[None]
        gy, gu, gv = dec.synthesize_batch(ly, luv, 1024, 1024, sv=1, sh=1, bit_depth=8)
        zo.set_fast(True)
        zo.set_threads(16)
        try:
            want = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.BOP, ly[0], luv[0],
                                 1024, 1024, sv=1, sh=1)
            rgb = _rgb(100, 1, 1024, 1024)
            luma, chroma = zo.preprocess_rgb(rgb[0])
            wy = zo.analysis_primary(cka, zo.BOP, luma)
            wuv = zo.analysis_secondary(ckc, zo.BOP, chroma)
        finally:
            zo.set_fast(False)
        for got, w in zip((gy[0], gu[0], gv[0]), want):
            frac, p = gate8(got, zo.quantize_plane(w))
            assert frac >= 0.999 and p >= 50.0, (frac, p)
        ay, auv = enc.analyze_rgb(rgb)
        assert rel_l2(ay[0], wy) < ANA_REL
        assert rel_l2(auv[0], wuv) < ANA_REL
    finally:
        dec.close()
        enc.close()
