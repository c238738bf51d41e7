"""GPU parity of the synthesis / analysis networks, the tiling scheduler, the output stage and
the attention-block layers, against the CPU oracle (the reference's f32 path restated) on the
same seeded inputs and random-init weights, through the C ABI.

Gates: decoded planes in [0, 255] with PSNR >= 50 dB against the CPU
output and the 8-bit reconstruction within +-1 step on >= 99.9% of samples; intermediate
layer kernels within relative L2 1e-3. The output stage is bit-exact given identical planes.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo

REL_L2 = 1e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def psnr(a, b):
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return 99.0 if mse == 0 else 10 * np.log10(255.0 ** 2 / mse)


def eight_bit_gate(got, want):
    qg = zo.quantize_plane(got).astype(np.int32)
    qw = zo.quantize_plane(want).astype(np.int32)
    d = np.abs(qg - qw)
    return float(np.mean(d <= 1)), int(d.max())


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=8 << 30)
    yield e
    e.close()


_NETS = {}


def nets(eng, op):
    import zenjpegai_b200 as zj
    import synthetic as syn
    if op not in _NETS:
        py, puv = syn.synthesis_params(op, 2)
        _NETS[op] = (py, puv, zj.Network(eng, zj.SYN_Y, zo.OPS[op], py),
                     zj.Network(eng, zj.SYN_UV, zo.OPS[op], puv))
    return _NETS[op]


def run_primary(net, y_hat, h, w):
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import ctypes
    oh, ow = zj.synth_out_size(zj.SYN_Y, net.op, h, w)
    out = np.empty((1, oh, ow), np.float32)
    zj.check(_lib.lib().zjai_synthesis_primary(net.handle, ctypes.c_void_p(y_hat.ctypes.data),
                                               y_hat.shape[1], y_hat.shape[2], h, w,
                                               ctypes.c_void_p(out.ctypes.data), 0))
    return out


def run_secondary(net, yl, yc, h, w):
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import ctypes
    oh, ow = zj.synth_out_size(zj.SYN_UV, net.op, h, w)
    out = np.empty((2, oh, ow), np.float32)
    zj.check(_lib.lib().zjai_synthesis_secondary(
        net.handle, ctypes.c_void_p(yl.ctypes.data), yl.shape[1], yl.shape[2],
        ctypes.c_void_p(yc.ctypes.data), yc.shape[1], yc.shape[2], h, w,
        ctypes.c_void_p(out.ctypes.data), 0))
    return out


@pytest.mark.parametrize("op", ["sop", "bop", "hop"])
@pytest.mark.parametrize("h,w", [(128, 192), (120, 200)])
def test_synthesis_tile(eng, op, h, w):
    import synthetic as syn
    py, puv, ny, nuv = nets(eng, op)
    lh, lw = -(-h // 16), -(-w // 16)
    ly = syn.laplace_latent(7, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(7, "luv", (96, lh, lw), 1.5)
    gy = run_primary(ny, ly, h, w)
    wy = zo.synthesis_primary(zo.Checkpoint(py), zo.OPS[op], ly, h, w)
    guv = run_secondary(nuv, ly, luv, h, w)
    wuv = zo.synthesis_secondary(zo.Checkpoint(puv), zo.OPS[op], ly, luv, h, w)
    for got, want in ((gy, wy), (guv, wuv)):
        assert got.shape == want.shape
        p = psnr(got, want)
        frac, worst = eight_bit_gate(got, want)
        assert p >= 50.0, (op, p)
        assert frac >= 0.999, (op, frac, worst)


def _synth_gpu(eng, op, H, W, tile, overlap, sv=2, sh=2):
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import synthetic as syn
    py, puv, ny, nuv = nets(eng, op)
    lh, lw = -(-H // 16), -(-W // 16)
    ly = syn.laplace_latent(11, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(11, "luv", (96, lh, lw), 1.5)
    ch, cw = -(-H // sv), -(-W // sh)
    ry = np.zeros((H, W), np.float32)
    ru = np.zeros((ch, cw), np.float32)
    rv = np.zeros((ch, cw), np.float32)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    zj.check(_lib.lib().zjai_synthesize(eng.handle, ny.handle, nuv.handle, p(ly), p(luv), lh, lw,
                                        H, W, H, W, tile, overlap, sv, sh, p(ry), p(ru), p(rv),
                                        0, None))
    return (ry, ru, rv), (py, puv, ly, luv)


def _synth_both(eng, op, H, W, tile, overlap, sv=2, sh=2):
    got, (py, puv, ly, luv) = _synth_gpu(eng, op, H, W, tile, overlap, sv, sh)
    wy, wu, wv = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.OPS[op], ly, luv, H, W,
                               tile_size=tile, overlap=overlap, sv=sv, sh=sh)
    return got, (wy, wu, wv)


@pytest.mark.parametrize("op,H,W,tile,overlap", [
    ("sop", 200, 344, 128, 16),
    ("hop", 272, 400, 128, 32),
    ("bop", 136, 240, 0, 0),
])
def test_synthesize_tiled(eng, op, H, W, tile, overlap):
    got, want = _synth_both(eng, op, H, W, tile, overlap)
    for g, w in zip(got, want):
        assert g.shape == w.shape
        assert psnr(g, w) >= 50.0
        frac, worst = eight_bit_gate(g, w)
        assert frac >= 0.999, (frac, worst)


@pytest.mark.parametrize("op,H,W,tile,overlap,bits", [
    ("sop", 136, 200, 0, 0, 8),
    ("hop", 272, 400, 128, 32, 8),
    ("hop", 130, 142, 0, 0, 10),
])
def test_synthesize_fused_output(eng, op, H, W, tile, overlap, bits):
    """The fused output stage (zjai_synthesize_q: samples quantized in the final layers'
    epilogue) equals quantize_plane_par of the f32 planes zjai_synthesize writes, to the bit."""
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import synthetic as syn
    py, puv, ny, nuv = nets(eng, op)
    lh, lw = -(-H // 16), -(-W // 16)
    ly = syn.laplace_latent(12, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(12, "luv", (96, lh, lw), 1.5)
    ch, cw = -(-H // 2), -(-W // 2)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    f = [np.zeros(s, np.float32) for s in ((H, W), (ch, cw), (ch, cw))]
    zj.check(_lib.lib().zjai_synthesize(eng.handle, ny.handle, nuv.handle, p(ly), p(luv), lh, lw,
                                        H, W, H, W, tile, overlap, 2, 2, p(f[0]), p(f[1]),
                                        p(f[2]), 0, None))
    dt = np.uint8 if bits == 8 else np.uint16
    q = [np.zeros(a.shape, dt) for a in f]
    zj.check(_lib.lib().zjai_synthesize_q(eng.handle, ny.handle, nuv.handle, p(ly), p(luv), lh,
                                          lw, H, W, H, W, tile, overlap, 2, 2, bits, p(q[0]),
                                          p(q[1]), p(q[2]), 0, None))
    for got, plane in zip(q, f):
        assert np.array_equal(got.astype(np.uint16), zo.quantize_plane(plane, bits))


def test_synthesize_deterministic(eng):
    """Two runs of the same tiled HOP synthesis give identical planes (no atomics or
    scheduling-dependent reductions anywhere on the path; the crate asserts bit-identity across
    thread counts, tests/decode_ref.rs:378)."""
    a, _ = _synth_gpu(eng, "hop", 272, 400, 128, 32)
    b, _ = _synth_gpu(eng, "hop", 272, 400, 128, 32)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_output_stage_bit_exact(eng):
    """Given identical planes, the GPU output stage equals the oracle's to the bit
    (quantize_plane_par, bicubic 4:2:0 -> 4:4:4, BT.709, round half to even)."""
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import synthetic as syn
    h, w = 135, 241
    y = syn.uniform(3, "y", (h, w), -5.0, 260.0)
    u = syn.uniform(3, "u", ((h + 1) // 2, (w + 1) // 2), -5.0, 260.0)
    v = syn.uniform(3, "v", ((h + 1) // 2, (w + 1) // 2), -5.0, 260.0)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    q = np.empty(y.shape, np.uint8)
    zj.check(_lib.lib().zjai_quantize_plane(eng.handle, p(y), y.size, 8, p(q), 0))
    assert np.array_equal(q.astype(np.uint16), zo.quantize_plane(y))
    rgb = np.empty((h, w, 3), np.uint8)
    zj.check(_lib.lib().zjai_yuv_to_rgb(eng.handle, p(y), p(u), p(v), h, w, u.shape[0],
                                        u.shape[1], 8, p(rgb), 0))
    uu = zo.resize_bicubic(u[None], h, w)[0]
    vv = zo.resize_bicubic(v[None], h, w)[0]
    r, g, b = zo.to_rgb_planes(y, uu, vv)
    want = zo.quantize_rgb(r, g, b)
    assert np.array_equal(rgb.astype(np.uint16), want)


@pytest.mark.parametrize("c", [128, 64, 40, 200, 384])
def test_layer_norm(eng, c):
    # c <= 256: pixel-segment kernel (8 / 16 / 32 lanes per pixel, idle lanes at 40 and 200);
    # 384: warp-per-pixel kernel
    import synthetic as syn
    x = syn.normal(5, "x", (c, 23, 37), std=3.0, mean=0.5)
    wt = syn.normal(5, "w", (c,), std=0.1, mean=1.0)
    b = syn.normal(5, "b", (c,), std=0.05)
    assert rel_l2(eng.layer_norm(x, wt, b), zo.layer_norm_channels(x, wt, b)) < REL_L2


@pytest.mark.parametrize("c,h,w", [(384, 19, 33), (1024, 19, 33), (40, 70, 130), (8, 5, 3),
                                   (192, 131, 66)])
def test_depthwise(eng, c, h, w):
    # row-streaming kernel: 64-column strips, 64-row bands, 64-channel blocks (ragged at
    # 40 / 8 channels, 130 columns, 70 and 131 rows)
    import synthetic as syn
    x = syn.normal(6, "x", (c, h, w))
    wt = syn.normal(6, "w", (c, 1, 3, 3), std=0.3)
    got = eng.depthwise3x3(x, wt)
    want = zo.conv2d(x, wt, None, pad=(1, 1), groups=c)
    assert rel_l2(got, want) < REL_L2


@pytest.mark.parametrize("c,h,w", [(1024, 19, 33), (512, 70, 97), (48, 9, 40), (16, 3, 2)])
def test_depthwise_elu_gate(eng, c, h, w):
    # FFN depthwise + ELU gate fused: 32-column strips, two 64-channel slabs per block
    import synthetic as syn
    x = syn.normal(7, "x", (c, h, w))
    wt = syn.normal(7, "w", (c, 1, 3, 3), std=0.3)
    got = eng.depthwise3x3_elu_gate(x, wt)
    d = zo.conv2d(x, wt, None, pad=(1, 1), groups=c)
    want = zo.elu_gate(d[: c // 2], d[c // 2:])
    assert got.shape == (c // 2, h, w)
    assert rel_l2(got, want) < REL_L2


@pytest.mark.parametrize("dim,hidden,h,w", [
    (128, 512, 40, 52),  # HOP luma width: 8 chunks, two 64-channel slabs of K, ragged tiles
    (64, 256, 37, 29),   # HOP chroma width: 4 chunks, one slab
    (128, 512, 12, 16),  # exactly one tile
    (64, 256, 5, 7),     # smaller than a tile
    (128, 256, 26, 33),  # other hidden width
])
def test_transformer_ffn(eng, dim, hidden, h, w):
    # fused FFN kernel (project_in -> depthwise 3x3 + ELU gate -> project_out + residual in one
    # tcgen05 kernel) after the layer norm, against the oracle's layers composed
    import synthetic as syn
    x = syn.normal(9, "x", (dim, h, w))
    nw = syn.uniform(9, "nw", (dim,), 0.5, 1.5)
    nb = syn.normal(9, "nb", (dim,), std=0.1)
    wi = syn.normal(9, "wi", (2 * hidden, dim, 1, 1), std=dim ** -0.5)
    wd = syn.normal(9, "wd", (2 * hidden, 1, 3, 3), std=0.3)
    wo = syn.normal(9, "wo", (dim, hidden, 1, 1), std=hidden ** -0.5)
    got = eng.transformer_ffn(x, nw, nb, wi, wd, wo)
    t = zo.layer_norm_channels(x, nw, nb)
    t = zo.conv2d(t, wi)
    t = zo.conv2d(t, wd, None, pad=(1, 1), groups=2 * hidden)
    t = zo.elu_gate(t[:hidden], t[hidden:])
    t = zo.conv2d(t, wo)
    assert got.shape == x.shape
    # the FFN's own contribution (residual removed) within the layer tolerance
    assert rel_l2(got - x, t) < REL_L2


@pytest.mark.parametrize("dim,h,w", [(128, 40, 52), (64, 64, 64), (96, 17, 29)])
def test_channel_attention(eng, dim, h, w):
    # 128 / 64: register-tiled Gram and per-head apply (head width 32 / 16); 96: generic kernels
    import synthetic as syn
    qkv = syn.normal(8, "qkv", (3 * dim, h, w))
    t = syn.uniform(8, "t", (4,), 0.5, 2.0)
    got = eng.channel_attention(qkv, 4, t)
    want = zo.channel_attention(qkv, 4, t)
    assert rel_l2(got, want) < REL_L2


@pytest.mark.parametrize("op", ["bop", "hop"])
def test_analysis(eng, op):
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import synthetic as syn
    pa, pauv = syn.analysis_params(op, 4)
    h, w = 120, 200
    x = np.floor(syn.uniform(9, "rgb", (1, h, w), 0.0, 256.0)).astype(np.float32)
    xc = np.floor(syn.uniform(9, "c", (12, h // 2, w // 2), 0.0, 256.0)).astype(np.float32)
    na = zj.Network(eng, zj.ANA_Y, zo.OPS[op], pa)
    nc = zj.Network(eng, zj.ANA_UV, zo.OPS[op], pauv)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    got = np.empty((160, -(-h // 16), -(-w // 16)), np.float32)
    zj.check(_lib.lib().zjai_analysis_primary(na.handle, p(x), h, w, p(got), 0))
    want = zo.analysis_primary(zo.Checkpoint(pa), zo.OPS[op], x)
    assert rel_l2(got, want) < 5e-3
    gotc = np.empty((96, -(-h // 16), -(-w // 16)), np.float32)
    zj.check(_lib.lib().zjai_analysis_secondary(nc.handle, p(xc), h // 2, w // 2, p(gotc), 0))
    wantc = zo.analysis_secondary(zo.Checkpoint(pauv), zo.OPS[op], xc)
    assert rel_l2(gotc, wantc) < 5e-3


@pytest.mark.parametrize("op,h,w", [("bop", 75, 131), ("hop", 57, 93)])
def test_analysis_primary_odd_size(eng, op, h, w):
    # odd picture sizes: the luma input's first-layer taps past the last row / column replicate
    # it (normalize_pad's padding), those above / left of the picture are the conv's zeros
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    import synthetic as syn
    pa, _ = syn.analysis_params(op, 4)
    x = np.floor(syn.uniform(11, "odd", (1, h, w), 0.0, 256.0)).astype(np.float32)
    na = zj.Network(eng, zj.ANA_Y, zo.OPS[op], pa)
    got = np.empty((160, -(-h // 16), -(-w // 16)), np.float32)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    zj.check(_lib.lib().zjai_analysis_primary(na.handle, p(x), h, w, p(got), 0))
    want = zo.analysis_primary(zo.Checkpoint(pa), zo.OPS[op], x)
    assert rel_l2(got, want) < 5e-3


def test_model_errors(eng):
    """Missing / mis-shaped parameters fail like the crate's loaders (Error::Model)."""
    import zenjpegai_b200 as zj
    import synthetic as syn
    py, _ = syn.synthesis_params("sop", 2)
    bad = dict(py)
    del bad["conv3.bias"]
    with pytest.raises(zj.ZjaiError) as e:
        zj.Network(eng, zj.SYN_Y, zj.SOP, bad)
    assert e.value.status == 5 and "conv3.bias" in str(e.value)
    bad = dict(py)
    bad["conv4.weight"] = np.zeros((16, 31, 1, 1), np.float32)
    with pytest.raises(zj.ZjaiError) as e:
        zj.Network(eng, zj.SYN_Y, zj.SOP, bad)
    assert e.value.status == 5 and "expected" in str(e.value)


def test_cancel_and_reuse(eng):
    """The caller's stop flag (the crate's `enough::Stop`, reconstruct.rs:391) is polled
    between tiles and layers: a set flag returns ZJAI_CANCELLED and the context stays usable."""
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder
    import synthetic as syn
    py, puv, ny, nuv = nets(eng, "sop")
    dec = Decoder.__new__(Decoder)
    dec.engine, dec.op, dec.net_y, dec.net_uv = eng, zj.SOP, ny, nuv
    H, W = 128, 192
    ly = syn.laplace_latent(40, "c/ly", (160, H // 16, W // 16), 1.5)
    luv = syn.laplace_latent(40, "c/luv", (96, H // 16, W // 16), 1.5)
    with pytest.raises(zj.ZjaiError) as e:
        dec.synthesize(ly, luv, H, W, tile_size=64, overlap=16, cancel=ctypes.c_int(1))
    assert e.value.status == 4  # ZJAI_CANCELLED
    got = dec.synthesize(ly, luv, H, W, tile_size=64, overlap=16, cancel=ctypes.c_int(0))
    want = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.SOP, ly, luv, H, W,
                         tile_size=64, overlap=16)
    assert psnr(got[0], want[0]) >= 50.0


def test_arena_limit_and_bad_geometry():
    """Arena exhaustion fails with ZJAI_LIMIT_EXCEEDED (Error::LimitExceeded) and malformed tile
    geometry with ZJAI_INVALID_DATA (tiles.rs:71-76); the context remains usable."""
    import zenjpegai_b200 as zj
    from zenjpegai_b200.decoder import Decoder
    import synthetic as syn
    small = zj.Engine(0, arena_bytes=64 << 20)
    py, puv = syn.synthesis_params("hop", 3)
    dec = Decoder(small, "hop", py, puv)
    H, W = 1024, 1024
    ly = syn.laplace_latent(41, "l/ly", (160, 64, 64), 1.5)
    luv = syn.laplace_latent(41, "l/luv", (96, 64, 64), 1.5)
    with pytest.raises(zj.ZjaiError) as e:
        dec.synthesize(ly, luv, H, W)
    assert e.value.status == 3  # ZJAI_LIMIT_EXCEEDED
    with pytest.raises(zj.ZjaiError) as e:
        dec.synthesize(ly, luv, H, W, tile_size=16, overlap=16)
    assert e.value.status == 6  # ZJAI_INVALID_DATA
    out = dec.synthesize(ly[:, :4, :4].copy(), luv[:, :4, :4].copy(), 64, 64)
    assert np.isfinite(out[0]).all()
    dec.close()
    small.close()


@pytest.mark.parametrize("op,H,W,tile,overlap,bits", [
    ("hop", 272, 400, 128, 32, 8),
    ("sop", 136, 203, 0, 0, 8),
    ("bop", 96, 128, 0, 0, 10),
])
def test_synthesize_rgb(eng, op, H, W, tile, overlap, bits):
    """Synthesis straight to RGB (the f32 planes never leave the device) equals zjai_synthesize
    followed by zjai_yuv_to_rgb to the bit, and the oracle's RGB (output.rs on its planes)
    within one step on >= 99.9% of samples."""
    import ctypes
    import synthetic as syn
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    from zenjpegai_b200.decoder import Decoder
    py, puv, ny, nuv = nets(eng, op)
    dec = Decoder.__new__(Decoder)
    dec.engine, dec.op, dec.net_y, dec.net_uv = eng, zo.OPS[op], ny, nuv
    lh, lw = -(-H // 16), -(-W // 16)
    ly = syn.laplace_latent(13, "ly", (160, lh, lw), 1.5)
    luv = syn.laplace_latent(13, "luv", (96, lh, lw), 1.5)
    got = dec.synthesize_rgb(ly, luv, H, W, tile_size=tile, overlap=overlap, bit_depth=bits)
    y, u, v = dec.synthesize(ly, luv, H, W, tile_size=tile, overlap=overlap)
    dt = np.uint8 if bits == 8 else np.uint16
    two = np.empty((H, W, 3), dt)
    p = lambda a: ctypes.c_void_p(a.ctypes.data)
    zj.check(_lib.lib().zjai_yuv_to_rgb(eng.handle, p(y), p(u), p(v), H, W, u.shape[0],
                                        u.shape[1], bits, p(two), 0))
    assert np.array_equal(got, two)
    wy, wu, wv = zo.synthesize(zo.Checkpoint(py), zo.Checkpoint(puv), zo.OPS[op], ly, luv, H, W,
                               tile_size=tile, overlap=overlap)
    r, g, b = zo.to_rgb_planes(wy, zo.resize_bicubic(wu[None], H, W)[0],
                               zo.resize_bicubic(wv[None], H, W)[0])
    want = zo.quantize_rgb(r, g, b, bits)
    d = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert float(np.mean(d <= (1 if bits == 8 else 4))) >= 0.999
