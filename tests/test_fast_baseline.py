"""The timed CPU baseline (oracle/fast.c, the crate's nn::fast convolution algorithm restated:
blocked NCHWc layout, register tiles of 8 positions x 8 channels, per-row threads, transposed
convs as parity phases) gives the same bits as the oracle's nn::reference loops, as the crate
asserts between its two paths (tests/fast_vs_reference.rs). CPU only."""

import numpy as np
import pytest

import oracle as zo


@pytest.fixture()
def fast():
    zo.set_fast(True)
    yield
    zo.set_fast(False)


def _both(fn):
    zo.set_fast(False)
    ref = fn()
    zo.set_fast(True)
    got = fn()
    return got, ref


@pytest.mark.parametrize("c,oc,h,w,k,stride,pad,groups,extra", [
    (160, 160, 11, 13, 3, 1, 1, 1, (0, 0, 0, 0)),   # HOP first-stage residual conv
    (128, 128, 17, 9, 3, 2, 1, 1, (0, 0, 0, 0)),    # stride 2 (CAB subscale, analysis)
    (128, 128, 10, 12, 3, 1, 1, 4, (0, 0, 0, 0)),   # grouped (HOP ResAU, 32 per group)
    (64, 64, 9, 15, 3, 1, 1, 4, (0, 0, 0, 0)),      # grouped, 16 per group (SOP / BOP ResAU)
    (128, 512, 7, 19, 1, 1, 0, 1, (0, 0, 0, 0)),    # 1x1 expansion
    (160, 256, 6, 7, 2, 1, 0, 1, (0, 0, 1, 1)),     # SOP upsampler 2x2 + extra pad
    (1, 128, 21, 23, 3, 2, 1, 1, (0, 0, 0, 0)),     # analysis conv1 (one input channel)
    (12, 128, 9, 10, 3, 2, 1, 1, (0, 0, 0, 0)),     # analysis secondary conv1
    (384, 384, 13, 11, 3, 1, 1, 384, (0, 0, 0, 0)),  # depthwise
    (64, 16, 12, 20, 1, 1, 0, 1, (0, 0, 0, 0)),     # narrow output (conv4)
    (40, 24, 5, 37, 3, 1, 1, 1, (0, 0, 0, 0)),      # channels not a multiple of 8
    (48, 48, 8, 8, 3, 1, 1, 3, (0, 0, 0, 0)),       # group size 16 (multiple of 8)
    (24, 24, 8, 8, 3, 1, 1, 6, (0, 0, 0, 0)),       # group size 4: reference loop fallback
])
def test_conv_bit_identical(c, oc, h, w, k, stride, pad, groups, extra):
    rng = np.random.default_rng(c * 7 + oc + k + groups)
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((oc, c // groups, k, k)) / np.sqrt(c * k * k / groups)).astype(np.float32)
    b = rng.standard_normal(oc).astype(np.float32)
    got, ref = _both(lambda: zo.conv2d(x, wt, b, stride=stride, pad=(pad, pad), groups=groups,
                                       extra=extra))
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("c,oc,h,w,k,pad,op", [
    (160, 128, 6, 9, 3, 1, 1), (128, 1, 11, 7, 3, 1, 1), (64, 8, 8, 5, 3, 1, 1),
    (160, 64, 9, 13, 4, 1, 0), (144, 64, 5, 6, 4, 1, 0), (20, 12, 3, 4, 3, 1, 1),
])
def test_convt_bit_identical(c, oc, h, w, k, pad, op):
    rng = np.random.default_rng(c + oc * 3 + k)
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c, oc, k, k)) / np.sqrt(c * k * k / 4)).astype(np.float32)
    b = rng.standard_normal(oc).astype(np.float32)
    got, ref = _both(lambda: zo.conv_transpose2d(x, wt, b, stride=2, pad=pad, out_pad=op))
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("op", ["sop", "hop"])
def test_network_bit_identical(op):
    import synthetic as syn
    py, puv = syn.synthesis_params(op, 2)
    h, w = 64, 96
    ly = syn.laplace_latent(5, "fb/ly", (160, h // 16, w // 16), 1.5)
    luv = syn.laplace_latent(5, "fb/luv", (96, h // 16, w // 16), 1.5)
    cky, ckuv = zo.Checkpoint(py), zo.Checkpoint(puv)
    got, ref = _both(lambda: (zo.synthesis_primary(cky, zo.OPS[op], ly, h, w),
                              zo.synthesis_secondary(ckuv, zo.OPS[op], ly, luv, h, w)))
    zo.set_fast(False)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)
