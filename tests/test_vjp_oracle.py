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


def conv3x3_f64(x, w, b):
    """3x3 conv, padding 1, in float64 (the finite differences' forward)."""
    c, h, wd = x.shape
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1)))
    out = np.zeros((w.shape[0], h, wd)) + np.asarray(b, np.float64)[:, None, None]
    for ky in range(3):
        for kx in range(3):
            out += np.einsum("oc,chw->ohw", w[:, :, ky, kx].astype(np.float64),
                             xp[:, ky:ky + h, kx:kx + wd])
    return out


def test_residual_block_backward_matches_finite_differences():
    # ResidualBlock::backward (attention.rs:58-75) against the block's forward
    # conv2(relu(conv1(x) + b1)) + b2 + x: <d_out, F(x + e v) - F(x - e v)> / 2e = <d_x, v>
    # (the step small enough that no pre-activation crosses the ReLU's kink)
    rng = np.random.default_rng(11)
    c, h, w = 8, 12, 10
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    w1 = (rng.standard_normal((c, c, 3, 3)) * 0.2).astype(np.float32)
    w2 = (rng.standard_normal((c, c, 3, 3)) * 0.2).astype(np.float32)
    b1 = (rng.standard_normal(c) * 0.1).astype(np.float32)
    b2 = (rng.standard_normal(c) * 0.1).astype(np.float32)

    def forward(xx):
        t = conv3x3_f64(xx, w1, b1)
        return conv3x3_f64(np.maximum(t, 0), w2, b2) + xx, t

    y, tape = forward(x)
    d = rng.standard_normal(y.shape).astype(np.float32)
    dx = zo.residual_block_backward(d, tape.astype(np.float32), w1, w2)
    v = rng.standard_normal(x.shape).astype(np.float32)
    eps = 1e-3
    lhs = float((d * (forward(x + eps * v)[0] - forward(x - eps * v)[0])).sum()) / (2 * eps)
    rhs = float((dx.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-3, (lhs, rhs)
    # the skip alone: with zero conv weights the gradient is d_out
    z = np.zeros_like(w1)
    assert np.array_equal(zo.residual_block_backward(d, tape.astype(np.float32), z, z), d)


CAB_NAMES = ("trunk0.conv1", "trunk0.conv2", "trunk1.conv1", "trunk1.conv2", "subscale",
             "mask2.conv1", "mask2.conv2", "mask3.conv1", "mask3.conv2", "upscale")


def convT3_s2_f64(x, w, b):
    """`conv3x3_t` (attention.rs:77-80): transposed conv, kernel 3, stride 2, padding 1, output
    padding 1, weight [c][oc][3][3], in float64: input (iy, ix) feeds output
    (2 iy - 1 + ky, 2 ix - 1 + kx)."""
    c, h, wd = x.shape
    oc = w.shape[1]
    out = np.zeros((oc, 2 * h, 2 * wd)) + np.asarray(b, np.float64)[:, None, None]
    for ky in range(3):
        for kx in range(3):
            contrib = np.einsum("co,chw->ohw", w[:, :, ky, kx].astype(np.float64),
                                x.astype(np.float64))
            ys, xs = 2 * np.arange(h) - 1 + ky, 2 * np.arange(wd) - 1 + kx
            vy, vx = (ys >= 0) & (ys < 2 * h), (xs >= 0) & (xs < 2 * wd)
            out[:, ys[vy][:, None], xs[vx][None, :]] += contrib[:, vy][:, :, vx]
    return out


def cab_forward_f64(x, wts, bias):
    """`Cab::forward_tape` (attention.rs:146-180) in float64: output and tape."""
    def rb(xx, a, b):
        t = conv3x3_f64(xx, wts[a], bias[a])
        return conv3x3_f64(np.maximum(t, 0), wts[b], bias[b]) + xx, t
    t0, rb0 = rb(x, "trunk0.conv1", "trunk0.conv2")
    trunk, rb1 = rb(t0, "trunk1.conv1", "trunk1.conv2")
    m = conv3x3_f64(x, wts["subscale"], bias["subscale"])[:, ::2, ::2]  # stride 2, padding 1
    m, mc0 = rb(m, "mask2.conv1", "mask2.conv2")
    m, mc1 = rb(m, "mask3.conv1", "mask3.conv2")
    sig = 1.0 / (1.0 + np.exp(-convT3_s2_f64(m, wts["upscale"], bias["upscale"])))
    tape = {"trunk_pre": trunk, "sig": sig, "rb_c1": [rb0, rb1], "mask_c1": [mc0, mc1]}
    return trunk * sig + x, tape


def cab_case(rng, c, h, w):
    wts = {k: (rng.standard_normal((c, c, 3, 3)) * (0.6 / np.sqrt(9 * c))).astype(np.float32)
           for k in CAB_NAMES}
    bias = {k: (rng.standard_normal(c) * 0.05).astype(np.float32) for k in CAB_NAMES}
    x = rng.standard_normal((c, h, w)).astype(np.float32)
    return x, wts, bias


def test_cab_backward_matches_finite_differences():
    # Cab::backward (attention.rs:182-223) against finite differences of the CAB's forward
    rng = np.random.default_rng(21)
    x, wts, bias = cab_case(rng, 8, 12, 14)
    y, tape = cab_forward_f64(x, wts, bias)
    d = rng.standard_normal(y.shape).astype(np.float32)
    tape32 = {"trunk_pre": tape["trunk_pre"].astype(np.float32),
              "sig": tape["sig"].astype(np.float32),
              "rb_c1": [a.astype(np.float32) for a in tape["rb_c1"]],
              "mask_c1": [a.astype(np.float32) for a in tape["mask_c1"]]}
    dx = zo.cab_backward(d, tape32, wts)
    v = rng.standard_normal(x.shape).astype(np.float32)
    eps = 1e-3
    fp = cab_forward_f64(x + eps * v, wts, bias)[0]
    fm = cab_forward_f64(x - eps * v, wts, bias)[0]
    lhs = float((d * (fp - fm)).sum()) / (2 * eps)
    rhs = float((dx.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-3, (lhs, rhs)


def test_elu_gate_backward_is_the_derivative():
    # elu_gate_backward (math.rs:838-858) against the analytic derivative of elu(a) . b
    rng = np.random.default_rng(5)
    a = (rng.standard_normal(4096) * 3).astype(np.float32)
    b = rng.standard_normal(4096).astype(np.float32)
    d = rng.standard_normal(4096).astype(np.float32)
    da, db = zo.elu_gate_backward(d, a, b)
    a64, b64, d64 = a.astype(np.float64), b.astype(np.float64), d.astype(np.float64)
    want_a = np.where(a64 > 0, 1.0, np.exp(a64)) * b64 * d64
    want_b = np.where(a64 > 0, a64, np.expm1(a64)) * d64
    assert np.abs(da - want_a).max() < 1e-5 * (1 + np.abs(want_a).max())
    assert np.abs(db - want_b).max() < 1e-5 * (1 + np.abs(want_b).max())


def test_layer_norm_backward_matches_finite_differences():
    # layer_norm_channels_backward (math.rs:860-913) against finite differences of the channel
    # layer norm (math.rs:423-448) in float64
    rng = np.random.default_rng(6)
    c, h, w = 24, 7, 9
    x = (rng.standard_normal((c, h, w)) * 2 + 0.5).astype(np.float32)
    wt = rng.standard_normal(c).astype(np.float32)
    bs = rng.standard_normal(c).astype(np.float32)

    def ln(xx):
        m = xx.mean(0, keepdims=True)
        v = ((xx - m) ** 2).mean(0, keepdims=True)
        return (xx - m) / np.sqrt(v + 1e-5) * wt[:, None, None] + bs[:, None, None]

    d = rng.standard_normal((c, h, w)).astype(np.float32)
    dx = zo.layer_norm_backward(d, x, wt)
    v = rng.standard_normal(x.shape)
    eps = 1e-4
    x64 = x.astype(np.float64)
    lhs = float((d * (ln(x64 + eps * v) - ln(x64 - eps * v))).sum()) / (2 * eps)
    rhs = float((dx.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-4, (lhs, rhs)


def attention_f64(qkv, heads, temp):
    """`channel_attention` (math.rs:506-603) in float64: q, k rows L2-normalised over the
    pixels (norm clamped at 1e-12), per head softmax(T . q k^T) applied to v."""
    c3, h, w = qkv.shape
    dim, n = c3 // 3, h * w
    c = dim // heads
    x = qkv.reshape(c3, n).astype(np.float64)
    q, k, v = x[:dim], x[dim:2 * dim], x[2 * dim:]
    q = q / np.maximum(np.linalg.norm(q, axis=1, keepdims=True), 1e-12)
    k = k / np.maximum(np.linalg.norm(k, axis=1, keepdims=True), 1e-12)
    out = np.empty((dim, n))
    for hd in range(heads):
        s = slice(hd * c, (hd + 1) * c)
        a = temp[hd] * (q[s] @ k[s].T)
        a = np.exp(a - a.max(1, keepdims=True))
        a /= a.sum(1, keepdims=True)
        out[s] = a @ v[s]
    return out.reshape(dim, h, w)


@pytest.mark.parametrize("dim,heads,h,w", [(32, 4, 6, 7), (64, 2, 5, 9)])
def test_channel_attention_backward_matches_finite_differences(dim, heads, h, w):
    # channel_attention_backward (math.rs:668-836) against finite differences of the attention
    rng = np.random.default_rng(dim + heads)
    qkv = rng.standard_normal((3 * dim, h, w)).astype(np.float32)
    temp = (rng.uniform(0.5, 2.0, heads)).astype(np.float32)
    d = rng.standard_normal((dim, h, w)).astype(np.float32)
    dq = zo.channel_attention_backward(qkv, heads, temp, d)
    v = rng.standard_normal(qkv.shape)
    eps = 1e-4
    q64 = qkv.astype(np.float64)
    lhs = float((d * (attention_f64(q64 + eps * v, heads, temp) -
                      attention_f64(q64 - eps * v, heads, temp))).sum()) / (2 * eps)
    rhs = float((dq.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-4, (lhs, rhs)
    # and the oracle's attention forward is the float64 one
    assert np.abs(zo.channel_attention(qkv, heads, temp) - attention_f64(q64, heads, temp)).max() < 1e-5


def tb_forward_f64(x, wts, heads, hidden):
    """`TransformerBlock::forward_tape` (attention.rs:373-430) in float64: the block's output and
    its tape (x_in, qkv, x_mid, gate); layer norms over the channels (eps 1e-5), 1x1 and depthwise
    3x3 convs without bias."""
    def ln(t, wgt, b):
        m = t.mean(0, keepdims=True)
        v = ((t - m) ** 2).mean(0, keepdims=True)
        return (t - m) / np.sqrt(v + 1e-5) * wgt[:, None, None] + b[:, None, None]

    def pw(t, wgt):
        return np.einsum("oc,chw->ohw", wgt[:, :, 0, 0].astype(np.float64), t)

    def dw(t, wgt):
        c, h, w = t.shape
        tp = np.pad(t, ((0, 0), (1, 1), (1, 1)))
        out = np.zeros_like(t)
        for ky in range(3):
            for kx in range(3):
                out += wgt[:, 0, ky, kx][:, None, None].astype(np.float64) * tp[:, ky:ky + h, kx:kx + w]
        return out

    x = x.astype(np.float64)
    qkv = dw(pw(ln(x, wts["prep_norm"], wts["prep_norm_b"]), wts["prep_conv1"]), wts["prep_conv2"])
    a = attention_f64(qkv, heads, wts["temperature"])
    x_mid = x + pw(a, wts["attn_out"])
    gate = dw(pw(ln(x_mid, wts["ffn_norm"], wts["ffn_norm_b"]), wts["ffn_in"]), wts["ffn_dw"])
    x1, x2 = gate[:hidden], gate[hidden:]
    out = x_mid + pw(np.where(x1 > 0, x1, np.expm1(x1)) * x2, wts["ffn_out"])
    return out, {"x_in": x, "qkv": qkv, "x_mid": x_mid, "gate": gate}


def tb_case(rng, dim, hidden, heads):
    def w(*shape, fan):
        return (rng.standard_normal(shape) * (0.8 / np.sqrt(fan))).astype(np.float32)
    return {"prep_norm": (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32),
            "prep_norm_b": (0.1 * rng.standard_normal(dim)).astype(np.float32),
            "prep_conv1": w(3 * dim, dim, 1, 1, fan=dim), "prep_conv2": w(3 * dim, 1, 3, 3, fan=9),
            "temperature": rng.uniform(0.5, 2.0, heads).astype(np.float32),
            "attn_out": w(dim, dim, 1, 1, fan=dim),
            "ffn_norm": (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32),
            "ffn_norm_b": (0.1 * rng.standard_normal(dim)).astype(np.float32),
            "ffn_in": w(2 * hidden, dim, 1, 1, fan=dim), "ffn_dw": w(2 * hidden, 1, 3, 3, fan=9),
            "ffn_out": w(dim, hidden, 1, 1, fan=hidden)}


def test_transformer_block_backward_matches_finite_differences():
    # TransformerBlock::backward (attention.rs:435-480) against finite differences of the block
    rng = np.random.default_rng(31)
    dim, hidden, heads, h, w = 16, 24, 4, 6, 7
    wts = tb_case(rng, dim, hidden, heads)
    x = rng.standard_normal((dim, h, w)).astype(np.float32)
    y, tape = tb_forward_f64(x, wts, heads, hidden)
    qkv32 = tape["qkv"].astype(np.float32)
    tape32 = {"x_in": x, "qkv": qkv32,
              "attn": zo.channel_attention_weights(qkv32, heads, wts["temperature"]),
              "x_mid": tape["x_mid"].astype(np.float32), "gate": tape["gate"].astype(np.float32)}
    d = rng.standard_normal(y.shape).astype(np.float32)
    dx = zo.transformer_block_backward(d, heads, hidden, tape32, wts)
    v = rng.standard_normal(x.shape)
    eps = 1e-4
    lhs = float((d * (tb_forward_f64(x + eps * v, wts, heads, hidden)[0] -
                      tb_forward_f64(x - eps * v, wts, heads, hidden)[0])).sum()) / (2 * eps)
    rhs = float((dx.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-3, (lhs, rhs)


def tape32(tape, wts, heads):
    qkv = tape["qkv"].astype(np.float32)
    return {"x_in": tape["x_in"].astype(np.float32), "qkv": qkv,
            "attn": zo.channel_attention_weights(qkv, heads, wts["temperature"]),
            "x_mid": tape["x_mid"].astype(np.float32), "gate": tape["gate"].astype(np.float32)}


@pytest.mark.parametrize("resample", [True, False])
def test_tam_backward_matches_finite_differences(resample):
    # Tam::backward (attention.rs:578-600): us_conv's VJP, the two blocks', ds_conv's
    rng = np.random.default_rng(41 + resample)
    dim, hidden, heads, h, w = 16, 24, 4, 12, 10
    blocks = [tb_case(rng, dim, hidden, heads) for _ in range(2)]
    ds_w = (rng.standard_normal((dim, dim, 3, 3)) * (0.8 / np.sqrt(9 * dim))).astype(np.float32)
    us_w = (rng.standard_normal((dim, dim, 3, 3)) * (0.8 / np.sqrt(9 * dim))).astype(np.float32)
    zero = np.zeros(dim, np.float32)

    def forward(x):
        if resample:
            x = conv3x3_f64(x, ds_w, zero)[:, ::2, ::2]
        x, t0 = tb_forward_f64(x, blocks[0], heads, hidden)
        x, t1 = tb_forward_f64(x, blocks[1], heads, hidden)
        if resample:
            x = convT3_s2_f64(x, us_w, zero)
        return x, (t0, t1)

    x = rng.standard_normal((dim, h, w)).astype(np.float32)
    y, (t0, t1) = forward(x.astype(np.float64))
    d = rng.standard_normal(y.shape).astype(np.float32)
    dx = zo.tam_backward(d, heads, hidden, h, w, [tape32(t0, blocks[0], heads),
                                                  tape32(t1, blocks[1], heads)], blocks,
                         ds_w if resample else None, us_w if resample else None)
    v = rng.standard_normal(x.shape)
    eps = 1e-4
    x64 = x.astype(np.float64)
    lhs = float((d * (forward(x64 + eps * v)[0] - forward(x64 - eps * v)[0])).sum()) / (2 * eps)
    rhs = float((dx.astype(np.float64) * v).sum())
    assert rel(lhs, rhs) < 1e-3, (lhs, rhs)
