"""RDLR layer VJPs on the GPU through the C ABI (`zjai_conv2d_backward`,
`zjai_conv_transpose2d_backward`): the input gradients of the synthesis network's conv layer
shapes (3x3 residual-block convs, the grouped ResAU conv, 1x1 projections, depthwise 3x3, the
stride-2 CAB subscale conv, a zero-bordered conv, the upsampling transposed convs) against the
oracle's restatement of the crate's f32 loops. The GPU path runs them as convolutions with f16
operands (d_out scaled by a power of two first) and f32 accumulation: relative L2 within 2e-3,
also for gradients of 1e-7 magnitude, which unscaled f16 could not hold."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

import oracle as zo

TOL = 2e-3


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=1 << 30)
    yield e
    e.close()


def rel_l2(a, b):
    return float(np.linalg.norm((a - b).ravel()) / max(np.linalg.norm(b.ravel()), 1e-30))


def he(rng, shape, fan_in):
    return (rng.standard_normal(shape) * np.sqrt(2.0 / fan_in)).astype(np.float32)


@pytest.mark.parametrize("c,oc,k,stride,pad,groups,extra,h,w", [
    (128, 128, 3, 1, 1, 1, None, 40, 36),      # residual block conv
    (128, 128, 3, 1, 1, 4, None, 33, 30),      # ResAU grouped conv
    (128, 384, 1, 1, 0, 1, None, 32, 32),      # prep / qkv projection
    (384, 128, 1, 1, 0, 1, None, 24, 40),      # output projection
    (64, 64, 3, 1, 1, 64, None, 31, 29),       # depthwise
    (128, 128, 3, 2, 1, 1, None, 33, 29),      # CAB subscale, odd extent
    (160, 64, 3, 2, 1, 1, None, 32, 48),       # stride 2, even extent
    (64, 96, 3, 1, 1, 1, (0, 1, 1, 0), 30, 26),  # zero-bordered conv
    (96, 16, 3, 1, 1, 1, None, 27, 35),
])
@pytest.mark.parametrize("mag", [1.0, 1e-7])
def test_conv2d_backward(eng, c, oc, k, stride, pad, groups, extra, h, w, mag):
    rng = np.random.default_rng(c + oc + k * 10 + stride * 100 + h)
    wt = he(rng, (oc, c // groups, k, k), c // groups * k * k)
    H, W = h + (extra[0] + extra[2] if extra else 0), w + (extra[1] + extra[3] if extra else 0)
    oh, ow = (H + 2 * pad - k) // stride + 1, (W + 2 * pad - k) // stride + 1
    d = (rng.standard_normal((oc, oh, ow)) * mag).astype(np.float32)
    want = zo.conv2d_backward(d, wt, h, w, stride, (pad, pad), groups, extra)
    got = eng.conv2d_backward(d, wt, h, w, stride, (pad, pad), groups, extra)
    assert got.shape == want.shape
    assert rel_l2(got, want) < TOL


@pytest.mark.parametrize("c,oc,k,pad,out_pad,h,w", [
    (160, 64, 4, 1, 0, 17, 15),    # BOP / SOP upsampling convT 4x4
    (128, 128, 3, 1, 1, 16, 18),   # HOP upsampling convT 3x3
    (64, 64, 4, 1, 0, 32, 24),
    (128, 4, 3, 1, 1, 20, 21),     # final layer shape (few outputs)
])
@pytest.mark.parametrize("mag", [1.0, 1e-7])
def test_conv_transpose2d_backward(eng, c, oc, k, pad, out_pad, h, w, mag):
    rng = np.random.default_rng(c + oc + k + h)
    wt = he(rng, (c, oc, k, k), c * k * k)
    oh, ow = (h - 1) * 2 - 2 * pad + k + out_pad, (w - 1) * 2 - 2 * pad + k + out_pad
    d = (rng.standard_normal((oc, oh, ow)) * mag).astype(np.float32)
    want = zo.conv_transpose2d_backward(d, wt, h, w, 2, pad)
    got = eng.conv_transpose2d_backward(d, wt, h, w, pad)
    assert rel_l2(got, want) < TOL


def test_device_tensors_and_errors(eng):
    import torch
    import zenjpegai_b200 as zj
    rng = np.random.default_rng(3)
    wt = he(rng, (64, 32, 3, 3), 32 * 9)
    d = rng.standard_normal((64, 20, 22)).astype(np.float32)
    want = zo.conv2d_backward(d, wt, 20, 22, 1, (1, 1), 1)
    got = eng.conv2d_backward(torch.from_numpy(d).cuda(), torch.from_numpy(wt).cuda(), 20, 22,
                              1, (1, 1), 1)
    torch.cuda.synchronize()
    assert rel_l2(got.cpu().numpy(), want) < TOL
    # a d_out that is not the layer's output extent
    with pytest.raises(zj.ZjaiError) as e:
        eng.conv2d_backward(d, wt, 21, 22, 1, (1, 1), 1)
    assert e.value.status == zj._lib.INVALID_ARGUMENT
    with pytest.raises(zj.ZjaiError) as e:
        eng.conv2d_backward(d[:, :10, :11], wt, 20, 22, 2, (1, 1), 1, extra=(1, 0, 0, 0))
    assert e.value.status in (zj._lib.INVALID_ARGUMENT, zj._lib.UNSUPPORTED)
    # an all-zero gradient gives zeros
    z = eng.conv2d_backward(np.zeros_like(d), wt, 20, 22, 1, (1, 1), 1)
    assert not z.any()


@pytest.mark.parametrize("c,h,w", [(128, 40, 36), (64, 33, 47), (160, 24, 24)])
@pytest.mark.parametrize("mag", [1.0, 1e-7])
def test_residual_block_backward(eng, c, h, w, mag):
    rng = np.random.default_rng(c + h + w)
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    w1, w2 = he(rng, (c, c, 3, 3), c * 9), he(rng, (c, c, 3, 3), c * 9)
    b1 = (rng.standard_normal(c) * 0.1).astype(np.float32)
    tape = zo.conv2d(x, w1, b1, 1, (1, 1))
    d = (rng.standard_normal((c, h, w)) * mag).astype(np.float32)
    want = zo.residual_block_backward(d, tape, w1, w2)
    got = eng.residual_block_backward(d, tape, w1, w2)
    assert rel_l2(got, want) < TOL


@pytest.mark.parametrize("c,h,w", [(128, 32, 40), (64, 26, 18)])
@pytest.mark.parametrize("mag", [1.0, 1e-7])
def test_cab_backward(eng, c, h, w, mag):
    # a chain of eight conv VJPs per call: 3e-3 relative L2
    from test_vjp_oracle import cab_case, cab_forward_f64
    rng = np.random.default_rng(c + h + w)
    x, wts, bias = cab_case(rng, c, h, w)
    _, tape = cab_forward_f64(x, wts, bias)
    tape = {"trunk_pre": tape["trunk_pre"].astype(np.float32),
            "sig": tape["sig"].astype(np.float32),
            "rb_c1": [a.astype(np.float32) for a in tape["rb_c1"]],
            "mask_c1": [a.astype(np.float32) for a in tape["mask_c1"]]}
    d = (rng.standard_normal((c, h, w)) * mag).astype(np.float32)
    want = zo.cab_backward(d, tape, wts)
    got = eng.cab_backward(d, tape, wts)
    assert rel_l2(got, want) < 3e-3


def test_elu_gate_and_layer_norm_backward(eng):
    import torch
    rng = np.random.default_rng(9)
    a = (rng.standard_normal((64, 33, 29)) * 3).astype(np.float32)
    b = rng.standard_normal(a.shape).astype(np.float32)
    d = rng.standard_normal(a.shape).astype(np.float32)
    wa, wb = zo.elu_gate_backward(d, a, b)
    ga, gb = eng.elu_gate_backward(d, a, b)
    # the GPU's expf against the crate's exp: a few ulp
    assert np.allclose(ga, wa, rtol=1e-5, atol=1e-6) and np.allclose(gb, wb, rtol=1e-5, atol=1e-6)
    for c in (64, 128, 160):
        x = (rng.standard_normal((c, 37, 41)) * 2 + 0.3).astype(np.float32)
        wt = rng.standard_normal(c).astype(np.float32)
        dd = rng.standard_normal(x.shape).astype(np.float32)
        want = zo.layer_norm_backward(dd, x, wt)
        got = eng.layer_norm_backward(dd, x, wt)
        # the same f64 sums in channel order and the same f32 operations: equal up to the last
        # ulp of the division order
        assert np.allclose(got, want, rtol=1e-5, atol=1e-6)
        tg = eng.layer_norm_backward(torch.from_numpy(dd).cuda(), torch.from_numpy(x).cuda(),
                                     torch.from_numpy(wt).cuda())
        torch.cuda.synchronize()
        assert np.array_equal(tg.cpu().numpy(), got)


@pytest.mark.parametrize("dim,heads,h,w", [(128, 4, 37, 41), (64, 4, 64, 64), (256, 4, 20, 23)])
def test_channel_attention_backward(eng, dim, heads, h, w):
    rng = np.random.default_rng(dim + h)
    qkv = rng.standard_normal((3 * dim, h, w)).astype(np.float32)
    temp = rng.uniform(0.5, 2.0, heads).astype(np.float32)
    d = rng.standard_normal((dim, h, w)).astype(np.float32)
    attn = zo.channel_attention_weights(qkv, heads, temp)
    want = zo.channel_attention_backward(qkv, heads, temp, d)
    got = eng.channel_attention_backward(qkv, heads, temp, attn, d)
    # f64 sums on both sides in different orders: 1e-4 relative L2 per third (dq, dk, dv)
    for s in (slice(0, dim), slice(dim, 2 * dim), slice(2 * dim, 3 * dim)):
        assert rel_l2(got[s], want[s]) < 1e-4


@pytest.mark.parametrize("dim,hidden,heads,h,w", [(64, 128, 4, 24, 20), (128, 256, 4, 16, 18)])
def test_transformer_block_backward(eng, dim, hidden, heads, h, w):
    # a chain of five conv VJPs, two depthwise ones, the attention and two layer norms
    from test_vjp_oracle import tb_case, tb_forward_f64
    rng = np.random.default_rng(dim + hidden)
    wts = tb_case(rng, dim, hidden, heads)
    x = rng.standard_normal((dim, h, w)).astype(np.float32)
    _, tape = tb_forward_f64(x, wts, heads, hidden)
    qkv = tape["qkv"].astype(np.float32)
    tape32 = {"x_in": x, "qkv": qkv,
              "attn": zo.channel_attention_weights(qkv, heads, wts["temperature"]),
              "x_mid": tape["x_mid"].astype(np.float32), "gate": tape["gate"].astype(np.float32)}
    d = rng.standard_normal((dim, h, w)).astype(np.float32)
    want = zo.transformer_block_backward(d, heads, hidden, tape32, wts)
    got = eng.transformer_block_backward(d, heads, hidden, tape32, wts)
    assert rel_l2(got, want) < 3e-3
