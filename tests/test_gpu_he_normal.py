"""The networks under the weight law BASELINE prescribes: He-normal, N(0, 2 / fan_in) with
PyTorch's fan_in, for every conv and transposed conv. Under it the activations grow through
the ResAU gates to about 2.4e4 (the 4K picture's tiles; f16 holds up to 65504) and almost every
output sample clamps to 0 or 255, so the networks' values are compared before the clamp
(zjai_ctx_set_output_clamp(0), the oracle's zo_set_output_clamp(0)) at the layer tolerance, and
the 8-bit outputs at the usual gate. Each layer stays within the per-layer 1e-3 (f16's relative
precision does not depend on the weights' scale); before the clamp, the whole network's planes
carry that error compounded through about twenty layers whose ResAU gates x * (1 + m) amplify it
where 1 + m is small, so they are gated at 2e-2 (measured 1.1e-3 .. 1.03e-2). The same
amplification puts the raw planes near 1e5 while the visible window is [0, 255]: the few
samples that land inside it need about 5e-6 relative precision, f32's, not f16 storage's, so
the 8-bit agreement under this law is gated at 98.5% within one step (measured 98.9 .. 99.7%;
the role-scaled law of the other tests meets the 99.9% gate). An input that pushes a residual /
gate output beyond the f16 range is reported as ZJAI_LIMIT_EXCEEDED, and the context stays
usable."""

NETWORK_PRECLAMP = 2e-2

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=8 << 30)
    yield e
    e.close()


def _run(eng, op, seed, h, w, lat_seed=7):
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder
    py, puv = syn.synthesis_params_he(op, seed)
    lh, lw = -(-h // 16), -(-w // 16)
    ly = syn.laplace_latent(lat_seed, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(lat_seed, "luv", (96, lh, lw), 1.5)
    dec = Decoder(eng, op, py, puv)
    try:
        eng.set_output_clamp(False)
        raw = dec.synthesize(ly, luv, h, w, sv=1, sh=1)
        eng.set_output_clamp(True)
        q = dec.synthesize(ly, luv, h, w, sv=1, sh=1, bit_depth=8)
    finally:
        eng.set_output_clamp(True)
        dec.close()
    zo.set_fast(True)
    zo.set_threads(16)
    try:
        zo.set_output_clamp(False)
        want_raw = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.OPS[op], ly, luv,
                                 h, w, sv=1, sh=1)
        zo.set_output_clamp(True)
        want = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.OPS[op], ly, luv, h, w,
                             sv=1, sh=1)
    finally:
        zo.set_output_clamp(True)
        zo.set_fast(False)
    return raw, q, want_raw, want


@pytest.mark.parametrize("op,seed,h,w", [("sop", 2, 128, 192), ("bop", 4, 128, 192),
                                         ("hop", 3, 128, 192), ("hop", 3, 512, 512),
                                         ("sop", 2, 1080, 1920)])
def test_he_normal_prescribed_law(eng, op, seed, h, w):
    raw, q, want_raw, want = _run(eng, op, seed, h, w)
    for g, wr in zip(raw, want_raw):
        assert np.isfinite(g).all()
        print("%s %dx%d pre-clamp relative L2 %.2e" % (op, h, w, rel_l2(g, wr)))
        assert rel_l2(g, wr) < NETWORK_PRECLAMP, (op, rel_l2(g, wr))
    for g, wq in zip(q, want):
        d = np.abs(g.astype(np.int32) - zo.quantize_plane(wq).astype(np.int32))
        print("%s %dx%d 8-bit within one step %.5f" % (op, h, w, float(np.mean(d <= 1))))
        assert float(np.mean(d <= 1)) >= 0.985


def test_activation_range_reported(eng):
    """A mask conv scaled far beyond any trained weight makes the ResAU gate x * (1 + m)
    overflow f16: the call returns ZJAI_LIMIT_EXCEEDED (not silent inf / NaN planes), and the
    same context then decodes the unscaled network."""
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder
    py, puv = syn.synthesis_params_he("sop", 2)
    big = dict(py)
    big["iact3.conv2.weight"] = big["iact3.conv2.weight"] * np.float32(2.0 ** 12)
    ly = syn.laplace_latent(7, "ly", (160, 8, 12), 1.5)
    luv = syn.laplace_latent(7, "luv", (96, 8, 12), 1.5)
    dec = Decoder(eng, "sop", big, puv)
    try:
        with pytest.raises(zj.ZjaiError) as err:
            dec.synthesize(ly, luv, 128, 192)
        assert err.value.status == 3 and "f16 range" in str(err.value)
    finally:
        dec.close()
    dec = Decoder(eng, "sop", py, puv)
    try:
        out = dec.synthesize(ly, luv, 128, 192)
        assert all(np.isfinite(p).all() for p in out)
    finally:
        dec.close()
