"""The oracle's latent-domain networks (hyper-decoder, context model) against an independent
float64 numpy restatement of src/model/hyper_decoder.rs:94-113 and src/model/mcm.rs:161-257 /
:733-760 (the layer primitives themselves are pinned by the crate's nn vectors in
test_oracle_golden.py; this pins their composition: crop, activations, stage order, padded
positions, context concatenation)."""

import numpy as np
import pytest

import oracle as zo
import synthetic as syn


def conv64(x, w, b=None, pad=0, groups=1):
    c, h, ww = x.shape
    o, icg, kh, kw = w.shape
    xp = np.pad(x.astype(np.float64), ((0, 0), (pad, pad), (pad, pad)))
    oh, ow = h + 2 * pad - kh + 1, ww + 2 * pad - kw + 1
    out = np.zeros((o, oh, ow))
    ocg = o // groups
    for g in range(groups):
        wg = w[g * ocg:(g + 1) * ocg].astype(np.float64)
        xg = xp[g * icg:(g + 1) * icg]
        for ky in range(kh):
            for kx in range(kw):
                out[g * ocg:(g + 1) * ocg] += np.einsum("oc,chw->ohw", wg[:, :, ky, kx],
                                                        xg[:, ky:ky + oh, kx:kx + ow])
    if b is not None:
        out += b.astype(np.float64)[:, None, None]
    return out


def convt64(x, w, b, k=4, stride=2, pad=1):
    """PyTorch ConvTranspose2d (weight [in][out][k][k]) by scatter."""
    c, h, ww = x.shape
    o = w.shape[1]
    full = np.zeros((o, (h - 1) * stride + k, (ww - 1) * stride + k))
    for ky in range(k):
        for kx in range(k):
            contrib = np.einsum("co,chw->ohw", w[:, :, ky, kx].astype(np.float64), x)
            full[:, ky:ky + (h - 1) * stride + 1:stride, kx:kx + (ww - 1) * stride + 1:stride] += contrib
    oh, ow = (h - 1) * stride - 2 * pad + k, (ww - 1) * stride - 2 * pad + k
    return full[:, pad:pad + oh, pad:pad + ow] + b.astype(np.float64)[:, None, None]


def hyper64(p, z, out_h, out_w):
    t = conv64(z, p["hyper_decoder.conv1.weight"])
    t = convt64(t, p["hyper_decoder.conv2.weight"], p["hyper_decoder.conv2.bias"])
    t = np.clip(t[:, :out_h, :out_w], 0, 6)
    t = np.clip(conv64(t, p["hyper_decoder.conv3.weight"], p["hyper_decoder.conv3.bias"], 1), 0, 6)
    return conv64(t, p["hyper_decoder.conv4.weight"], p["hyper_decoder.conv4.bias"], 1)


def mcm64(p, res, psi):
    c, h, w = res.shape
    hh, hw = -(-h // 2), -(-w // 2)
    rp = np.zeros((c, 2 * hh, 2 * hw))
    rp[:, :h, :w] = res
    y = np.zeros((c, 2 * hh, 2 * hw))
    ctx = None
    for s, (py, px) in enumerate([(0, 0), (1, 1), (0, 1), (1, 0)]):
        psi_s = psi[s * c:(s + 1) * c].astype(np.float64)
        pre = "context.MCM.%d" % s
        if s == 0:
            x = psi_s
        else:
            t = conv64(ctx, p[pre + ".conv.0.weight"])
            t = conv64(t, p[pre + ".conv.1.weight"], p[pre + ".conv.1.bias"], 1, c // 32)
            x = np.concatenate([t, psi_s])
        f = pre + ".fusion_pred_net"
        m = np.maximum(conv64(x, p[f + ".conv1.weight"]), 0)
        m = np.maximum(conv64(m, p[f + ".conv2.weight"]), 0)
        m = conv64(m, p[f + ".conv3.weight"])
        stage = m + rp[:, py::2, px::2]
        y[:, py::2, px::2] = stage
        ctx = stage if ctx is None else np.concatenate([ctx, stage])
    return y[:, :h, :w]


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


@pytest.mark.parametrize("hz,wz,out_h,out_w", [(3, 4, 6, 8), (3, 4, 5, 7), (1, 1, 1, 2)])
def test_hyper_decoder_composition(hz, wz, out_h, out_w):
    p = syn.latent_params(11, 32, context=False)
    z = np.round(syn.laplace_latent(5, "z", (32, hz, wz), 2.0)).astype(np.float32)
    got = zo.hyper_decode(zo.Checkpoint(p), z, out_h, out_w)
    want = hyper64(p, z, out_h, out_w)
    assert got.shape == want.shape == (128, out_h, out_w)
    assert rel(got, want) < 1e-5


def test_hyper_decoder_rejects_oversized_crop():
    p = syn.latent_params(11, 32, context=False)
    z = np.zeros((32, 2, 2), np.float32)
    with pytest.raises(ValueError):
        zo.hyper_decode(zo.Checkpoint(p), z, 5, 4)


@pytest.mark.parametrize("h,w", [(8, 10), (9, 13), (1, 1), (2, 3)])
def test_context_model_composition(h, w):
    """Even and odd extents: positions past an odd edge read a zero residual but their stage
    value (the mean) still feeds the next stages' context."""
    p = syn.latent_params(12, 32, context=True)
    res = syn.laplace_latent(6, "r", (32, h, w), 1.0)
    psi = syn.normal(7, "psi", (128, -(-h // 2), -(-w // 2)))
    got = zo.context_decompress(zo.Checkpoint(p), res, psi)
    want = mcm64(p, res, psi)
    assert rel(got, want) < 1e-5


def test_no_context_model_is_upshuffle_plus_residual():
    """Without "context.MCM.*" the latent is upshuffle_psi(psi) + residual, one f32 add."""
    p = syn.latent_params(13, 96, context=False)
    h, w = 7, 10
    res = syn.laplace_latent(8, "r", (96, h, w), 1.0)
    psi = syn.normal(9, "psi", (384, 4, 5))
    got = zo.context_decompress(zo.Checkpoint(p), res, psi)
    lut = [0, 2, 3, 1]
    want = np.empty_like(res)
    for Y in range(h):
        for X in range(w):
            s = lut[(Y % 2) * 2 + X % 2]
            want[:, Y, X] = psi[s * 96:(s + 1) * 96, Y // 2, X // 2] + res[:, Y, X]
    assert np.array_equal(got, want)


def test_context_model_rejects_channels_not_multiple_of_32():
    p = syn.latent_params(14, 48, context=True)
    res = np.zeros((48, 4, 4), np.float32)
    psi = np.zeros((192, 2, 2), np.float32)
    with pytest.raises(ValueError):
        zo.context_decompress(zo.Checkpoint(p), res, psi)
