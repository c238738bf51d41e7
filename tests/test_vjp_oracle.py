"""The oracle's RDLR layer VJPs (oracle/oracle.c `zo_conv2d_backward`,
`zo_conv_transpose2d_backward`, restating src/nn/reference.rs:238-336 through
src/nn/fast/layers.rs:72-90): pinned by the property the reference's own tests check
(`conv2d_backward_is_adjoint`, `conv_transpose2d_backward_is_adjoint`, reference.rs:437-505,
there through finite differences): the gradient is the adjoint of the layer,
<conv(x), d> = <x, conv_backward(d)>, checked here exactly in float64 sums over the oracle's own
f32 forward and backward."""

import numpy as np
import pytest

import oracle as zo


def rel(a, b):
    return abs(a - b) / max(abs(a), abs(b), 1e-30)


@pytest.mark.parametrize("c,oc,k,stride,pad,groups,extra,h,w", [
    (8, 12, 3, 1, 1, 1, None, 13, 11),
    (8, 8, 3, 1, 1, 4, None, 13, 11),
    (16, 16, 3, 1, 1, 16, None, 9, 10),      # depthwise
    (6, 10, 3, 2, 1, 1, None, 13, 11),       # stride 2, odd extent
    (6, 10, 3, 2, 1, 1, None, 12, 10),       # stride 2, even extent
    (8, 8, 3, 1, 1, 1, (1, 0, 2, 1), 10, 9),  # extra zero border
    (12, 20, 1, 1, 0, 1, None, 7, 9),        # 1x1
    (4, 6, 5, 1, 2, 2, None, 11, 8),
])
def test_conv2d_backward_is_the_adjoint(c, oc, k, stride, pad, groups, extra, h, w):
    rng = np.random.default_rng(c * 100 + oc + k + stride)
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    wt = rng.standard_normal((oc, c // groups, k, k)).astype(np.float32)
    y = zo.conv2d(x, wt, None, stride, (pad, pad), groups, extra or (0, 0, 0, 0))
    d = rng.standard_normal(y.shape).astype(np.float32)
    dx = zo.conv2d_backward(d, wt, h, w, stride, (pad, pad), groups, extra)
    assert dx.shape == x.shape
    a = float((y.astype(np.float64) * d).sum())
    b = float((x.astype(np.float64) * dx).sum())
    assert rel(a, b) < 1e-5, (a, b)


@pytest.mark.parametrize("c,oc,k,pad,out_pad,h,w", [
    (8, 6, 4, 1, 0, 9, 7), (8, 6, 3, 1, 1, 9, 7), (6, 8, 5, 2, 1, 10, 6), (4, 4, 3, 1, 0, 5, 5)])
def test_conv_transpose2d_backward_is_the_adjoint(c, oc, k, pad, out_pad, h, w):
    rng = np.random.default_rng(c + oc * 7 + k)
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    wt = rng.standard_normal((c, oc, k, k)).astype(np.float32)
    y = zo.conv_transpose2d(x, wt, None, 2, pad, out_pad)
    d = rng.standard_normal(y.shape).astype(np.float32)
    dx = zo.conv_transpose2d_backward(d, wt, h, w, 2, pad)
    a = float((y.astype(np.float64) * d).sum())
    b = float((x.astype(np.float64) * dx).sum())
    assert rel(a, b) < 1e-5, (a, b)


def test_conv2d_backward_of_a_one_hot_gradient_is_the_flipped_kernel():
    # a single d_out sample at (2, 3) of output channel 1 spreads w[1, :, ky, kx] over the input
    # pixels (2 + ky - 1, 3 + kx - 1)
    wt = np.arange(2 * 3 * 9, dtype=np.float32).reshape(2, 3, 3, 3)
    d = np.zeros((2, 6, 7), np.float32)
    d[1, 2, 3] = 1.0
    dx = zo.conv2d_backward(d, wt, 6, 7, 1, (1, 1), 1)
    want = np.zeros((3, 6, 7), np.float32)
    want[:, 1:4, 2:5] = wt[1]
    assert np.array_equal(dx, want)
