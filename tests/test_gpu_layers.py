"""GPU layer parity: the tcgen05 convolution and the other layer kernels against the CPU oracle
on the same seeded inputs, through the C ABI.

Tolerance: per-layer relative L2 error <= 1e-3. The GPU computes with
f16 operands (11-bit significand) and f32 accumulation; the oracle is the reference's f32
contract. The golden cases are also checked against the reference's torch outputs.
"""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "nn_vectors.npz"))
REL_L2 = 1e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0)
    yield e
    e.close()


@pytest.mark.parametrize("name,stride,pad,groups", [
    ("conv3x3_s1_p1_bias", 1, (1, 1), 1),
    ("conv3x3_s1_p1_g4_nobias", 1, (1, 1), 4),
    ("conv1x1_nobias", 1, (0, 0), 1),
    ("conv3x3_s2_p1_bias", 2, (1, 1), 1),
    ("conv2x2_s1_p0", 1, (0, 0), 1),
    ("conv1x3_p01_bias", 1, (0, 1), 1),
    ("conv3x1_p10_bias", 1, (1, 0), 1),
])
def test_conv_golden(eng, name, stride, pad, groups):
    x, w, y = GOLDEN[name + "/x"], GOLDEN[name + "/w"], GOLDEN[name + "/y"]
    b = GOLDEN[name + "/b"] if name + "/b" in GOLDEN.files else None
    got = eng.conv2d(np.ascontiguousarray(x), np.ascontiguousarray(w),
                     None if b is None else np.ascontiguousarray(b), stride=stride, pad=pad,
                     groups=groups)
    assert got.shape == y.shape
    assert rel_l2(got, y) < REL_L2
    assert rel_l2(got, zo.conv2d(x, w, b, stride=stride, pad=pad, groups=groups)) < REL_L2


@pytest.mark.parametrize("name,pad,op", [
    ("convt4x4_s2_p1_bias", 1, 0),
    ("convt3x3_s2_p1_op1_bias", 1, 1),
])
def test_convt_golden(eng, name, pad, op):
    x, w, y, b = (GOLDEN[name + "/" + k] for k in ("x", "w", "y", "b"))
    got = eng.conv_transpose2d(np.ascontiguousarray(x), np.ascontiguousarray(w),
                               np.ascontiguousarray(b), pad=pad, out_pad=op)
    assert got.shape == y.shape
    assert rel_l2(got, y) < REL_L2


# (cin, cout, h, w, k, stride, pad, groups, extra)
CASES = [
    (128, 128, 33, 45, 3, 1, 1, 1, None),     # odd sizes, kc 64
    (160, 160, 17, 30, 3, 1, 1, 1, None),     # 160 channels: 3 chunks, zero-filled tail
    (32, 32, 40, 50, 3, 1, 1, 2, None),       # kc 32, grouped (16 per group)
    (16, 48, 21, 19, 3, 1, 1, 1, None),       # kc 16
    (12, 128, 64, 48, 3, 2, 1, 1, None),      # analysis chroma conv1: stride 2, 12 channels
    (128, 128, 31, 29, 3, 2, 1, 1, None),     # stride 2, odd input
    (160, 256, 20, 24, 2, 1, 0, 1, (0, 0, 1, 1)),  # SOP upsample conv 2x2 + extra pad
    (128, 512, 16, 20, 1, 1, 0, 1, None),     # 1x1, N > 256 (two N tiles)
    (128, 1024, 9, 40, 1, 1, 0, 1, None),     # 1x1, four N tiles
    (256, 48, 10, 14, 3, 1, 1, 1, None),      # chroma combine
    (128, 128, 16, 16, 3, 1, 1, 4, None),     # HOP ResAU grouped
]


@pytest.mark.parametrize("case", CASES, ids=[str(c[:8]) for c in CASES])
def test_conv_random(eng, case):
    cin, cout, h, w, k, stride, pad, groups, extra = case
    rng = np.random.default_rng(hash(case) & 0xFFFF)
    x = rng.uniform(-1, 1, (cin, h, w)).astype(np.float32)
    kk = (k, k)
    wt = (rng.standard_normal((cout, cin // groups) + kk) / np.sqrt(cin // groups * k * k)
          ).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    got = eng.conv2d(x, wt, b, stride=stride, pad=(pad, pad), groups=groups, extra=extra)
    want = zo.conv2d(x, wt, b, stride=stride, pad=(pad, pad), groups=groups,
                     extra=extra or (0, 0, 0, 0))
    assert got.shape == want.shape
    assert rel_l2(got, want) < REL_L2


@pytest.mark.parametrize("cin,cout,h,w,k,op", [
    (160, 128, 12, 10, 3, 1), (128, 1, 20, 22, 3, 1), (64, 8, 16, 16, 3, 1),
    (160, 64, 9, 13, 4, 0), (144, 64, 8, 8, 4, 0),
])
def test_convt_random(eng, cin, cout, h, w, k, op):
    rng = np.random.default_rng(cin * 1000 + cout)
    x = rng.uniform(-1, 1, (cin, h, w)).astype(np.float32)
    wt = (rng.standard_normal((cin, cout, k, k)) / np.sqrt(cin * k * k / 4)).astype(np.float32)
    b = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    got = eng.conv_transpose2d(x, wt, b, pad=1, out_pad=op)
    want = zo.conv_transpose2d(x, wt, b, stride=2, pad=1, out_pad=op)
    assert got.shape == want.shape
    assert rel_l2(got, want) < REL_L2


def test_config1_conv_leaky(eng):
    """3x3 128->128 at 128x128, U(-1,1) input, N(0, 1/(9*128)) weights,
    N(0, 0.01^2) bias, seed 0, then LeakyReLU(0.01); compared elementwise with the oracle."""
    import synthetic as syn
    import zenjpegai_b200 as zj
    x = syn.uniform(0, "x", (128, 128, 128), -1.0, 1.0)
    w = syn.normal(0, "w", (128, 128, 3, 3), std=float(np.sqrt(1.0 / (9 * 128))))
    b = syn.normal(0, "b", (128,), std=0.01)
    got = eng.conv2d(x, w, b, pad=(1, 1), act=zj.ACT_LEAKY)
    want = zo.leaky_relu(zo.conv2d(x, w, b, pad=(1, 1)))
    assert rel_l2(got, want) < REL_L2
    assert np.max(np.abs(got - want)) < 1e-2


def test_device_timeout_then_recovery():
    """Failure detection without a GPU fault: with the convolution kernel's pipeline waits
    limited to 300 SM cycles (less than one TMA load takes to land), the first wait of every
    CTA runs out, the kernel records its status word, drains the copies and MMAs it has in
    flight, frees its TMEM and ends; the call reports ZJAI_DEVICE_TIMEOUT. The same context,
    back on the default limit, then computes the layer correctly."""
    import synthetic as syn
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=256 << 20)
    try:
        x = syn.uniform(30, "to/x", (128, 48, 64), -1.0, 1.0)
        w = syn.normal(30, "to/w", (128, 128, 3, 3), std=float(np.sqrt(1.0 / (9 * 128))))
        b = syn.normal(30, "to/b", (128,), std=0.01)
        e.set_wait_limit(300)
        with pytest.raises(zj.ZjaiError) as err:
            e.conv2d(x, w, b, pad=(1, 1))
        assert err.value.status == 8  # ZJAI_DEVICE_TIMEOUT
        assert "bounded wait" in str(err.value)
        e.set_wait_limit(0)
        got = e.conv2d(x, w, b, pad=(1, 1))
        assert rel_l2(got, zo.conv2d(x, w, b, pad=(1, 1))) < REL_L2
        e.sync()  # the status word was cleared by the failing call
    finally:
        e.close()
