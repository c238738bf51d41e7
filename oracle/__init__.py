"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is a plain-C restatement of the reference crate's f32 CPU path (see `oracle.h`).
Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py` import this
module; the `zenjpegai_b200` package never does. Parity is pinned against the reference's own
golden vectors (`tests/golden/nn_vectors.npz`, converted by `tests/golden/make_golden.py`).
"""

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

SOP, BOP, HOP = 0, 1, 2
OPS = {"sop": SOP, "bop": BOP, "hop": HOP}


def build():
    """Compile the oracle library (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_f = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int
_i64 = ctypes.c_int64


class Param(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("ndim", _i), ("shape", _i * 4), ("data", _f)]


class Ckpt(ctypes.Structure):
    _fields_ = [("params", ctypes.POINTER(Param)), ("n", _i)]


class Tile(ctypes.Structure):
    _fields_ = [(k, _i) for k in (
        "img_x", "img_y", "img_w", "img_h", "lat_x", "lat_y", "lat_w", "lat_h",
        "core_x", "core_y", "core_w", "core_h", "off_x", "off_y")]


DUMP_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, _f, _i, _i, _i)


class ATile(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int) for k in (
        "img_x", "img_y", "img_w", "img_h", "lat_x", "lat_y", "lat_w", "lat_h",
        "core_x", "core_y", "core_w", "core_h", "off_x", "off_y")]


def _declare(L):
    L.zo_set_threads.argtypes = [_i]
    L.zo_preprocess_rgb.argtypes = [ctypes.c_void_p, _i, _i, _f, _f]
    L.zo_analysis_tiles.argtypes = [_i, _i, _i, _i, _i, ctypes.c_void_p, _i]
    L.zo_analyze_tiled.argtypes = [ctypes.c_void_p, _i, _i, _f, _i, _i, _f]
    L.zo_set_fast.argtypes = [_i]
    L.zo_set_output_clamp.argtypes = [_i]
    L.zo_conv2d_out_size.argtypes = [_i] * 7 + [ctypes.POINTER(_i)] * 3
    L.zo_conv2d.argtypes = [_f, _i, _i, _i, _f, _f, _i, _i, _i, _i, _i, _i, _i,
                            ctypes.POINTER(_i), _f]
    L.zo_conv_transpose2d_out_size.argtypes = [_i] * 6 + [ctypes.POINTER(_i)] * 2
    L.zo_conv_transpose2d.argtypes = [_f, _i, _i, _i, _f, _f, _i, _i, _i, _i, _i, _f]
    L.zo_pixel_shuffle.argtypes = [_f, _i, _i, _i, _i, _f]
    for n in ("zo_relu", "zo_relu6", "zo_sigmoid", "zo_denormalize"):
        getattr(L, n).argtypes = [_f, _i64]
    for n in ("zo_add", "zo_gate", "zo_mul", "zo_elu_gate"):
        getattr(L, n).argtypes = [_f, _f, _i64]
    L.zo_exp.argtypes = [ctypes.c_float]
    L.zo_exp.restype = ctypes.c_float
    L.zo_layer_norm_channels.argtypes = [_f, _i, _i, _i, _f, _f]
    L.zo_channel_attention.argtypes = [_f, _i, _i, _i, _i, _f, _f]
    L.zo_dot8.argtypes = [_f, _f, _i64]
    L.zo_dot8.restype = ctypes.c_double
    L.zo_set_dump.argtypes = [DUMP_FN]
    L.zo_synth_out_size.argtypes = [_i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]
    L.zo_synthesis_primary.argtypes = [ctypes.POINTER(Ckpt), _i, _f, _i, _i, _i, _i, _f]
    L.zo_synthesis_secondary.argtypes = [ctypes.POINTER(Ckpt), _i, _f, _i, _i, _f, _i, _i,
                                         _i, _i, _f]
    L.zo_analysis_primary.argtypes = [ctypes.POINTER(Ckpt), _i, _f, _i, _i, _f]
    L.zo_analysis_secondary.argtypes = [ctypes.POINTER(Ckpt), _i, _f, _i, _i, _f]
    L.zo_analysis_stage.argtypes = [ctypes.POINTER(Ckpt), _i, _i, _i, _f, _i, _i, _i, _f]
    L.zo_lef.argtypes = [_f, _i, _i, ctypes.POINTER(ctypes.c_int32), _i, _i, _i, _i, _i, _i, _f]
    L.zo_nearest_index.argtypes = [_i, _i, _i]
    L.zo_icci_filter.argtypes = [ctypes.c_void_p, ctypes.c_void_p, _i, _i, _f, _f, _f, _i, _i, _i, _i]
    L.zo_dwt2_block.argtypes = [_f, _f]
    L.zo_idwt2_block.argtypes = [_f, _f]
    L.zo_hyper_decode.argtypes = [ctypes.POINTER(Ckpt), _f, _i, _i, _i, _i, _i, _f]
    L.zo_context_decompress.argtypes = [ctypes.POINTER(Ckpt), _i, _f, _i, _i, _f, _f]
    L.zo_synthesis_tiles.argtypes = [_i] * 6 + [ctypes.POINTER(Tile), _i]
    L.zo_synthesize.argtypes = [ctypes.POINTER(Ckpt), ctypes.POINTER(Ckpt), _i, _f, _f] + \
        [_i] * 10 + [_f, _f, _f]
    L.zo_quantize_plane.argtypes = [_f, _i64, _i, ctypes.POINTER(ctypes.c_uint16)]
    L.zo_resize_bicubic.argtypes = [_f, _i, _i, _i, _i, _i, _f]
    L.zo_to_rgb_planes.argtypes = [_f, _f, _f, _i64]
    L.zo_quantize_rgb.argtypes = [_f, _f, _f, _i64, _i, ctypes.POINTER(ctypes.c_uint16)]
    L.zo_normalize.argtypes = [_f, _i64, _f]
    L.zo_pad_amount.argtypes = [_i, _i]
    L.zo_conv2d_backward.argtypes = [_f, _i, _i, _i, _f, _i, _i, _i, _i, _i, _i, _i,
                                     ctypes.POINTER(_i), _i, _i, _f]
    L.zo_conv_transpose2d_backward.argtypes = [_f, _i, _i, _i, _f, _i, _i, _i, _i, _i, _i, _f]
    L.zo_residual_block_backward.argtypes = [_f, _f, _i, _i, _i, _f, _f, _f]
    L.zo_cab_backward.argtypes = [_f, _i, _i, _i, _f * 4, _f * 2, _f * 10, _f]
    L.zo_elu_gate_backward.argtypes = [_f, _f, _f, _i64, _f, _f]
    L.zo_layer_norm_backward.argtypes = [_f, _f, _i, _i, _i, _f, _f]
    L.zo_channel_attention_weights.argtypes = [_f, _i, _i, _i, _i, _f, _f]
    L.zo_channel_attention_backward.argtypes = [_f, _i, _i, _i, _i, _f, _f, _f, _f]
    L.zo_transformer_block_backward.argtypes = [_f, _i, _i, _i, _i, _i, _f * 5, _f * 9, _f]
    L.zo_tam_backward.argtypes = [_f, _i, _i, _i, _i, _i, _i, _f * 5, _f * 5, _f * 9, _f * 9, _f,
                                  _f, _f]
    L.zo_efe_split_edge.argtypes = [ctypes.c_double, _i]
    L.zo_efe_linear.argtypes = [_f, _i, _i, _f, _f, _i, _i, _i, _i, _i, _i, _i, _i,
                                ctypes.POINTER(EfeLinearSet), _f, _f]
    L.zo_efe_nonlinear.argtypes = [_f, _i, _i, _f, _f, _i, _i, _i, _i, _i, _i,
                                   ctypes.POINTER(EfeNonlinearParams), _f, _f]


def _fp(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f)


def _c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n):
    lib().zo_set_threads(int(n))


def set_fast(on):
    """Convolutions on the restatement of the crate's nn::fast algorithm (fast.c: same bits,
    blocked layout and register tiles; the timed CPU baseline) or on the reference loops."""
    lib().zo_set_fast(1 if on else 0)


def set_output_clamp(on):
    """False: the synthesis outputs are x * 128 + 127.5 without the [0, 255] clamp."""
    lib().zo_set_output_clamp(1 if on else 0)


def get_fast():
    return bool(lib().zo_get_fast())


def conv2d(x, w, b=None, stride=1, pad=(0, 0), groups=1, extra=(0, 0, 0, 0)):
    """x [c,h,w], w [oc, c/groups, kh, kw] -> [oc, oh, ow] (reference.rs:92-133)."""
    x, w = _c32(x), _c32(w)
    c, h, wd = x.shape
    oc, _, kh, kw = w.shape
    ex = (_i * 4)(*extra)
    oh, ow = _i(), _i()
    lib().zo_conv2d_out_size(h, wd, kh, kw, stride, pad[0], pad[1], ex, oh, ow)
    out = np.empty((oc, oh.value, ow.value), np.float32)
    bb = _c32(b) if b is not None else None
    r = lib().zo_conv2d(_fp(x), c, h, wd, _fp(w), _fp(bb) if bb is not None else None, oc, kh,
                        kw, stride, pad[0], pad[1], groups, ex, _fp(out))
    if r:
        raise ValueError("oracle conv2d: bad geometry")
    return out


def conv_transpose2d(x, w, b=None, stride=2, pad=1, out_pad=0):
    """x [c,h,w], w [c, oc, k, k] (reference.rs:204-236)."""
    x, w = _c32(x), _c32(w)
    c, h, wd = x.shape
    _, oc, k, _ = w.shape
    oh, ow = _i(), _i()
    lib().zo_conv_transpose2d_out_size(h, wd, k, stride, pad, out_pad, oh, ow)
    out = np.empty((oc, oh.value, ow.value), np.float32)
    bb = _c32(b) if b is not None else None
    r = lib().zo_conv_transpose2d(_fp(x), c, h, wd, _fp(w),
                                  _fp(bb) if bb is not None else None, oc, k, stride, pad,
                                  out_pad, _fp(out))
    if r:
        raise ValueError("oracle conv_transpose2d: bad geometry")
    return out


def conv2d_backward(dout, w, h, wd, stride=1, pad=(0, 0), groups=1, extra=None):
    """Input gradient of `conv2d` (reference.rs:241-292, layers.rs:72-90): dout [oc, oh, ow],
    w [oc, c/groups, kh, kw] -> [c, h, wd] (h, wd: the layer input without its extra border)."""
    dout, w = _c32(dout), _c32(w)
    oc, oh, ow = dout.shape
    _, icg, kh, kw = w.shape
    c = icg * groups
    out = np.empty((c, h, wd), np.float32)
    ex = (_i * 4)(*extra) if extra is not None else None
    if lib().zo_conv2d_backward(_fp(dout), oc, oh, ow, _fp(w), c, kh, kw, stride, pad[0],
                                pad[1], groups, ex, h, wd, _fp(out)):
        raise ValueError("oracle conv2d_backward: bad geometry")
    return out


def conv_transpose2d_backward(dout, w, h, wd, stride=2, pad=1):
    """Input gradient of `conv_transpose2d` (reference.rs:294-336): dout [oc, oh, ow],
    w [c, oc, k, k] -> [c, h, wd]."""
    dout, w = _c32(dout), _c32(w)
    oc, oh, ow = dout.shape
    c, _, k, _ = w.shape
    out = np.empty((c, h, wd), np.float32)
    if lib().zo_conv_transpose2d_backward(_fp(dout), oc, oh, ow, _fp(w), c, k, stride, pad, h,
                                          wd, _fp(out)):
        raise ValueError("oracle conv_transpose2d_backward: bad geometry")
    return out


def residual_block_backward(dout, conv1_out, w1, w2):
    """`ResidualBlock::backward` (attention.rs:58-75): dout, conv1_out [c, h, w], conv weights
    [c, c, 3, 3] -> d_x [c, h, w]."""
    dout, t, w1, w2 = _c32(dout), _c32(conv1_out), _c32(w1), _c32(w2)
    c, h, w = dout.shape
    out = np.empty_like(dout)
    if lib().zo_residual_block_backward(_fp(dout), _fp(t), c, h, w, _fp(w1), _fp(w2), _fp(out)):
        raise ValueError("oracle residual_block_backward: bad geometry")
    return out


CAB_WEIGHTS = ("trunk0.conv1", "trunk0.conv2", "trunk1.conv1", "trunk1.conv2", "subscale",
               "mask2.conv1", "mask2.conv2", "mask3.conv1", "mask3.conv2", "upscale")


def cab_backward(dout, tape, weights):
    """`Cab::backward` (attention.rs:182-223): dout [c, h, w]; tape {"trunk_pre", "sig",
    "rb_c1": [2], "mask_c1": [2]}; weights {name in CAB_WEIGHTS: [c, c, 3, 3]} -> d_x."""
    dout = _c32(dout)
    c, h, w = dout.shape
    ts = [_c32(tape["trunk_pre"]), _c32(tape["sig"]), _c32(tape["rb_c1"][0]),
          _c32(tape["rb_c1"][1])]
    ms = [_c32(m) for m in tape["mask_c1"]]
    ws = [_c32(weights[k]) for k in CAB_WEIGHTS]
    out = np.empty_like(dout)
    if lib().zo_cab_backward(_fp(dout), c, h, w, (_f * 4)(*[_fp(a) for a in ts]),
                             (_f * 2)(*[_fp(a) for a in ms]), (_f * 10)(*[_fp(a) for a in ws]),
                             _fp(out)):
        raise ValueError("oracle cab_backward: bad geometry")
    return out


def elu_gate_backward(d, a, b):
    """`elu_gate_backward` (math.rs:838-858): (d_a, d_b) of y = elu(a) . b."""
    d, a, b = _c32(d), _c32(a), _c32(b)
    da, db = np.empty_like(d), np.empty_like(d)
    lib().zo_elu_gate_backward(_fp(d), _fp(a), _fp(b), d.size, _fp(da), _fp(db))
    return da, db


def layer_norm_backward(d, x, weight):
    """`layer_norm_channels_backward` (math.rs:860-913): d, x [c, h, w], weight [c] -> d_x."""
    d, x = _c32(d), _c32(x)
    c, h, w = x.shape
    out = np.empty_like(x)
    if lib().zo_layer_norm_backward(_fp(d), _fp(x), c, h, w, _fp(_c32(weight)), _fp(out)):
        raise ValueError("oracle layer_norm_backward: bad shape")
    return out


def channel_attention_weights(qkv, heads, temperature):
    """The forward's softmax weights [dim, dim / heads] (the attention VJP's tape)."""
    qkv, t = _c32(qkv), _c32(temperature)
    c3, h, w = qkv.shape
    attn = np.empty((c3 // 3, c3 // 3 // heads), np.float32)
    if lib().zo_channel_attention_weights(_fp(qkv), c3, h, w, heads, _fp(t), _fp(attn)):
        raise ValueError("oracle channel_attention_weights: channel / head counts")
    return attn


def channel_attention_backward(qkv, heads, temperature, dout):
    """`channel_attention_backward` (math.rs:668-836) with the forward's softmax weights as the
    tape: qkv [3 dim, h, w], dout [dim, h, w] -> dqkv [3 dim, h, w]."""
    qkv, dout, t = _c32(qkv), _c32(dout), _c32(temperature)
    c3, h, w = qkv.shape
    dim = c3 // 3
    attn = np.empty((dim, dim // heads), np.float32)
    out = np.empty_like(qkv)
    if lib().zo_channel_attention_weights(_fp(qkv), c3, h, w, heads, _fp(t), _fp(attn)) or \
            lib().zo_channel_attention_backward(_fp(qkv), c3, h, w, heads, _fp(t), _fp(attn),
                                                _fp(dout), _fp(out)):
        raise ValueError("oracle channel_attention_backward: channel / head counts")
    return out


TB_TAPE = ("x_in", "qkv", "attn", "x_mid", "gate")
TB_WEIGHTS = ("prep_norm", "prep_conv1", "prep_conv2", "temperature", "attn_out", "ffn_norm",
              "ffn_in", "ffn_dw", "ffn_out")


def transformer_block_backward(dout, heads, hidden, tape, weights):
    """`TransformerBlock::backward` (attention.rs:435-480): dout [dim, h, w]; tape and weights
    dicts keyed by TB_TAPE / TB_WEIGHTS -> d_x [dim, h, w]."""
    dout = _c32(dout)
    dim, h, w = dout.shape
    ts = [_c32(tape[k]) for k in TB_TAPE]
    ws = [_c32(weights[k]) for k in TB_WEIGHTS]
    out = np.empty_like(dout)
    if lib().zo_transformer_block_backward(_fp(dout), dim, hidden, heads, h, w,
                                           (_f * 5)(*[_fp(a) for a in ts]),
                                           (_f * 9)(*[_fp(a) for a in ws]), _fp(out)):
        raise ValueError("oracle transformer_block_backward: shapes")
    return out


def tam_backward(dout, heads, hidden, h, w, tapes, weights, ds_w=None, us_w=None):
    """`Tam::backward` (attention.rs:578-600): dout at the TAM's output, tapes / weights of its
    two blocks (dicts as transformer_block_backward takes), ds_w / us_w the resampling convs
    (None: no resampling) -> d_x [dim, h, w]."""
    dout = _c32(dout)
    dim = dout.shape[0]
    keep = []

    def arr(a):
        a = _c32(a)
        keep.append(a)
        return _fp(a)
    tp = [(_f * 5)(*[arr(t[k]) for k in TB_TAPE]) for t in tapes]
    wp = [(_f * 9)(*[arr(wd[k]) for k in TB_WEIGHTS]) for wd in weights]
    rs = ds_w is not None
    out = np.empty((dim, h, w), np.float32)
    if lib().zo_tam_backward(_fp(dout), dim, hidden, heads, h, w, int(rs), tp[0], tp[1], wp[0],
                             wp[1], arr(ds_w) if rs else None, arr(us_w) if rs else None,
                             _fp(out)):
        raise ValueError("oracle tam_backward: shapes")
    return out


def pixel_shuffle(x, r):
    x = _c32(x)
    c, h, w = x.shape
    out = np.empty((c // (r * r), h * r, w * r), np.float32)
    if lib().zo_pixel_shuffle(_fp(x), c, h, w, r, _fp(out)):
        raise ValueError("pixel_shuffle")
    return out


def _unary(name, x):
    y = _c32(x).copy()
    getattr(lib(), name)(_fp(y), y.size)
    return y


def relu(x):
    return _unary("zo_relu", x)


def relu6(x):
    return _unary("zo_relu6", x)


def sigmoid(x):
    return _unary("zo_sigmoid", x)


def denormalize(x):
    return _unary("zo_denormalize", x)


def _binary(name, a, b):
    y = _c32(a).copy()
    b = _c32(b)
    assert y.size == b.size
    getattr(lib(), name)(_fp(y), _fp(b), y.size)
    return y


def add(a, b):
    return _binary("zo_add", a, b)


def gate(x, m):
    return _binary("zo_gate", x, m)


def mul(a, b):
    return _binary("zo_mul", a, b)


def elu_gate(a, b):
    return _binary("zo_elu_gate", a, b)


def exp(x):
    return np.array([lib().zo_exp(float(v)) for v in np.asarray(x, np.float32).ravel()],
                    np.float32).reshape(np.shape(x))


def leaky_relu(x, slope=0.01):
    """torch.nn.functional.leaky_relu (not a reference op; used by the BASELINE configs)."""
    x = _c32(x)
    return np.where(x > 0, x, x * np.float32(slope)).astype(np.float32)


def layer_norm_channels(x, w, b):
    y = _c32(x).copy()
    c, h, wd = y.shape
    lib().zo_layer_norm_channels(_fp(y), c, h, wd, _fp(_c32(w)), _fp(_c32(b)))
    return y


def channel_attention(qkv, heads, temperature):
    qkv = _c32(qkv)
    c3, h, w = qkv.shape
    out = np.empty((c3 // 3, h, w), np.float32)
    if lib().zo_channel_attention(_fp(qkv), c3, h, w, heads, _fp(_c32(temperature)), _fp(out)):
        raise ValueError("channel_attention")
    return out


def dot8(a, b):
    a, b = _c32(a), _c32(b)
    return lib().zo_dot8(_fp(a), _fp(b), a.size)


class Checkpoint:
    """Named f32 tensors handed to the C oracle (keeps the numpy buffers alive)."""

    def __init__(self, params):
        self.arrays = {k: _c32(v) for k, v in params.items()}
        n = len(self.arrays)
        self._p = (Param * n)()
        self._names = []
        for i, (k, v) in enumerate(self.arrays.items()):
            nm = k.encode()
            self._names.append(nm)
            self._p[i].name = nm
            self._p[i].ndim = v.ndim
            for d in range(4):
                self._p[i].shape[d] = v.shape[d] if d < v.ndim else 0
            self._p[i].data = _fp(v)
        self.ck = Ckpt(self._p, n)


_dump_keep = []


def set_dump(fn):
    """fn(name, array) per intermediate map, or None."""
    if fn is None:
        cb = DUMP_FN()
    else:
        def _cb(name, data, c, h, w):
            fn(name.decode(), np.ctypeslib.as_array(data, shape=(c, h, w)).copy())
        cb = DUMP_FN(_cb)
    _dump_keep[:] = [cb]
    lib().zo_set_dump(cb)


def synth_out_size(op, secondary, h, w):
    oh, ow = _i(), _i()
    lib().zo_synth_out_size(op, int(secondary), h, w, oh, ow)
    return oh.value, ow.value


def synthesis_primary(ck, op, y_hat, h, w):
    y_hat = _c32(y_hat)
    assert y_hat.shape[0] == 160
    oh, ow = synth_out_size(op, 0, h, w)
    out = np.empty((1, oh, ow), np.float32)
    lib().zo_synthesis_primary(ctypes.byref(ck.ck), op, _fp(y_hat), y_hat.shape[1],
                               y_hat.shape[2], h, w, _fp(out))
    return out


def synthesis_secondary(ck, op, y_luma, y_chroma, h, w):
    y_luma, y_chroma = _c32(y_luma), _c32(y_chroma)
    oh, ow = synth_out_size(op, 1, h, w)
    out = np.empty((2, oh, ow), np.float32)
    r = lib().zo_synthesis_secondary(ctypes.byref(ck.ck), op, _fp(y_luma), y_luma.shape[1],
                                     y_luma.shape[2], _fp(y_chroma), y_chroma.shape[1],
                                     y_chroma.shape[2], h, w, _fp(out))
    if r:
        raise ValueError("synthesis_secondary")
    return out


def analysis_primary(ck, op, x):
    x = _c32(x)
    _, h, w = x.shape
    out = np.empty((160, -(-h // 16), -(-w // 16)), np.float32)
    if lib().zo_analysis_primary(ctypes.byref(ck.ck), op, _fp(x), h, w, _fp(out)):
        raise ValueError("analysis_primary")
    return out


def analysis_stage(ck, op, secondary, stage, x, h, w):
    """Analysis stage `stage` (1..4) of an h x w picture on its input x (the picture for stage
    1, else the previous stage's 128-channel map): act1, act2, act3 or the latent."""
    x = _c32(x)
    d = {1: 2, 2: 4, 3: 8}.get(stage, 16 if not secondary else 8)
    cout = 128 if stage < 4 else (96 if secondary else 160)
    out = np.empty((cout, -(-h // d), -(-w // d)), np.float32)
    if lib().zo_analysis_stage(ctypes.byref(ck.ck), op, int(bool(secondary)), stage, _fp(x),
                               x.shape[0], h, w, _fp(out)):
        raise ValueError("analysis_stage")
    return out


def analysis_secondary(ck, op, x):
    x = _c32(x)
    _, h, w = x.shape
    out = np.empty((96, -(-h // 8), -(-w // 8)), np.float32)
    if lib().zo_analysis_secondary(ctypes.byref(ck.ck), op, _fp(x), h, w, _fp(out)):
        raise ValueError("analysis_secondary")
    return out


def lef(luma, scale_log, channel, model_id, bit_depth=8):
    """LEF sharpening (src/filters/lef.rs:100-171) of luma [h, w] (or [1, h, w])."""
    y = _c32(luma).reshape(luma.shape[-2:])
    s = np.ascontiguousarray(scale_log, dtype=np.int32)
    c, sh, sw = s.shape
    out = np.empty_like(y)
    if lib().zo_lef(_fp(y), y.shape[0], y.shape[1], s.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                    c, sh, sw, channel, model_id, bit_depth, _fp(out)):
        raise ValueError("LEF: model_id / channel / bit depth / extent out of range")
    return out


_u32p = ctypes.POINTER(ctypes.c_uint32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class EfeLinearSet(ctypes.Structure):
    _fields_ = [("cand", _i * 2), ("filter_len", _i * 2), ("min_symbol", _i),
                ("chroma_codes", _u32p * 2), ("luma_codes", _u32p * 2)]


class EfeNonlinearParams(ctypes.Structure):
    _fields_ = [("min_symbol", _i), ("tile_width", _i), ("tile_height", _i), ("ntiles", _i),
                ("luma_min", _u16p), ("luma_max", _u16p), ("codes", _u32p * 2),
                ("ncodes", _i * 2), ("mask_bs", _i), ("mask_h", _i), ("mask_w", _i),
                ("mask", _u8p * 2)]


class EfeError(ValueError):
    """A filter call the crate rejects; `status` is its zjai_status number (1 invalid
    argument, 2 unsupported, 6 invalid data)."""

    def __init__(self, status):
        super().__init__(f"EFE: status {status}")
        self.status = status


def _arr(a, dtype, ptype, keep):
    if a is None:
        return None
    a = np.ascontiguousarray(a, dtype=dtype).ravel()
    keep.append(a)
    return a.ctypes.data_as(ptype)


def _efe_linear_set(st, keep):
    """ctypes set from {"cand": [c_u, c_v] (-1 / None: plane not filtered), "filter_len",
    "min_symbol", "chroma": [codes_u, codes_v], "luma": [codes_u, codes_v]}."""
    s = EfeLinearSet()
    for p in range(2):
        c = st["cand"][p]
        s.cand[p] = -1 if c is None else int(c)
        s.filter_len[p] = int(st["filter_len"][p])
        s.chroma_codes[p] = _arr(st["chroma"][p], np.uint32, _u32p, keep)
        s.luma_codes[p] = _arr(st["luma"][p], np.uint32, _u32p, keep)
    s.min_symbol = int(st.get("min_symbol", 0))
    return s


def efe_split_edge(fraction, s):
    return lib().zo_efe_split_edge(float(fraction), int(s))


def efe_linear(y, u, v, fmt, mean, st):
    """EFE linear (src/filters/efe_linear.rs:403-460) with one coded set `st`; fmt = (s_ver,
    s_hor, c_ver, c_hor); mean = the two B1 codes. Returns the filtered (u, v)."""
    y, u, v = _c32(y), _c32(u), _c32(v)
    keep = []
    s = _efe_linear_set(st, keep)
    ou, ov = np.empty_like(u), np.empty_like(v)
    r = lib().zo_efe_linear(_fp(y), y.shape[0], y.shape[1], _fp(u), _fp(v), u.shape[0],
                            u.shape[1], *fmt, int(mean[0]), int(mean[1]), ctypes.byref(s),
                            _fp(ou), _fp(ov))
    if r:
        raise EfeError(r)
    return ou, ov


def _efe_nonlinear_params(prm, keep):
    """ctypes parameters from {"min_symbol", "tile_width", "tile_height", "luma_min",
    "luma_max", "codes": [u, v] (None: off), "mask_bs", "masks": [u, v] ([my, mx] arrays or
    None)}."""
    q = EfeNonlinearParams()
    q.min_symbol = int(prm.get("min_symbol", 0))
    q.tile_width = int(prm.get("tile_width", 0))
    q.tile_height = int(prm.get("tile_height", 0))
    lmin, lmax = prm.get("luma_min"), prm.get("luma_max")
    q.ntiles = 0 if lmin is None else min(len(lmin), len(lmax))
    q.luma_min = _arr(lmin, np.uint16, _u16p, keep)
    q.luma_max = _arr(lmax, np.uint16, _u16p, keep)
    codes = prm.get("codes", [None, None])
    masks = prm.get("masks", [None, None])
    geo = next((np.asarray(m).shape for m in masks if m is not None), (0, 0))
    q.mask_bs = int(prm.get("mask_bs", 0))
    q.mask_h, q.mask_w = int(geo[0]), int(geo[1])
    for p in range(2):
        q.codes[p] = _arr(codes[p], np.uint32, _u32p, keep)
        q.ncodes[p] = 0 if codes[p] is None else int(np.asarray(codes[p]).size)
        q.mask[p] = _arr(masks[p], np.uint8, _u8p, keep)
    return q


def efe_nonlinear(y, u, v, fmt, prm, alt=None):
    """EFE non-linear (src/filters/efe_nonlinear.rs:190-237): returns the filtered (u, v);
    alt = the EFE linear filter's alternative (u, v) or None."""
    y = _c32(y)
    u, v = _c32(u).copy(), _c32(v).copy()
    keep = []
    q = _efe_nonlinear_params(prm, keep)
    au, av = (None, None) if alt is None else (_c32(alt[0]), _c32(alt[1]))
    r = lib().zo_efe_nonlinear(_fp(y), y.shape[0], y.shape[1], _fp(u), _fp(v), u.shape[0],
                               u.shape[1], *fmt, ctypes.byref(q),
                               None if au is None else _fp(au), None if av is None else _fp(av))
    if r:
        raise EfeError(r)
    return u, v


def nearest_index(i, src, dst):
    return lib().zo_nearest_index(i, src, dst)


def icci_filter(ck_y, ck_uv, use_u, use_v, y, u, v, tile=0, overlap=0):
    """eICCI (src/filters/icci.rs) of a 4:4:4 picture: filtered copies of y, u, v [h, w]."""
    y, u, v = (np.array(_c32(p), copy=True) for p in (y, u, v))
    h, w = y.shape
    r = lib().zo_icci_filter(ctypes.byref(ck_y.ck) if ck_y is not None else None,
                             ctypes.byref(ck_uv.ck) if ck_uv is not None else None,
                             int(use_u), int(use_v), _fp(y), _fp(u), _fp(v), h, w, tile, overlap)
    if r:
        raise ValueError("eICCI: malformed tiling")
    return y, u, v


def dwt2_block(p):
    out = np.empty(16, np.float32)
    lib().zo_dwt2_block(_fp(_c32(p).reshape(16)), _fp(out))
    return out


def idwt2_block(s):
    out = np.empty(16, np.float32)
    lib().zo_idwt2_block(_fp(_c32(s).reshape(16)), _fp(out))
    return out.reshape(4, 4)


def hyper_decode(ck, z, out_h, out_w):
    """HyperDecoder::forward_f32 (hyper_decoder.rs:94-113): z [c, hz, wz] -> psi
    [4c, out_h, out_w]."""
    z = _c32(z)
    c, hz, wz = z.shape
    psi = np.empty((4 * c, out_h, out_w), np.float32)
    if lib().zo_hyper_decode(ctypes.byref(ck.ck), _fp(z), c, hz, wz, out_h, out_w, _fp(psi)):
        raise ValueError("hyper_decode: crop larger than the upsampled map")
    return psi


def context_decompress(ck, residual, psi):
    """The latent y_hat from the dequantised residual [c, h, w] and psi [4c, ceil(h/2),
    ceil(w/2)] (reconstruct.rs:200-212): the context model (mcm.rs:161-257) when `ck` has one,
    else upshuffle_psi + residual."""
    residual, psi = _c32(residual), _c32(psi)
    c, h, w = residual.shape
    if psi.shape != (4 * c, -(-h // 2), -(-w // 2)):
        raise ValueError("context_decompress: residual / psi shape mismatch")
    y = np.empty_like(residual)
    if lib().zo_context_decompress(ctypes.byref(ck.ck), c, _fp(residual), h, w, _fp(psi),
                                   _fp(y)):
        raise ValueError("context_decompress: channel count must be a multiple of 32")
    return y


def synthesis_tiles(height, width, lh, lw, tile_size, overlap):
    n = lib().zo_synthesis_tiles(height, width, lh, lw, tile_size, overlap, None, 0)
    if n <= 0:
        raise ValueError("malformed synthesis tiling")
    arr = (Tile * n)()
    lib().zo_synthesis_tiles(height, width, lh, lw, tile_size, overlap, arr, n)
    return [{k: getattr(t, k) for k, _ in Tile._fields_} for t in arr]


def synthesize(ck_y, ck_uv, op, y_hat_y, y_hat_uv, height, width, out_h=None, out_w=None,
               tile_size=0, overlap=0, sv=2, sh=2):
    y_hat_y, y_hat_uv = _c32(y_hat_y), _c32(y_hat_uv)
    _, lh, lw = y_hat_y.shape
    out_h = height if out_h is None else out_h
    out_w = width if out_w is None else out_w
    ch, cw = -(-out_h // sv), -(-out_w // sh)
    ry = np.zeros((out_h, out_w), np.float32)
    ru = np.zeros((ch, cw), np.float32)
    rv = np.zeros((ch, cw), np.float32)
    r = lib().zo_synthesize(ctypes.byref(ck_y.ck), ctypes.byref(ck_uv.ck), op, _fp(y_hat_y),
                            _fp(y_hat_uv), lh, lw, height, width, out_h, out_w, tile_size,
                            overlap, sv, sh, _fp(ry), _fp(ru), _fp(rv))
    if r:
        raise ValueError("synthesize")
    return ry, ru, rv


def quantize_plane(x, bit_depth=8):
    x = _c32(x)
    out = np.empty(x.shape, np.uint16)
    lib().zo_quantize_plane(_fp(x), x.size, bit_depth,
                            out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)))
    return out


def resize_bicubic(x, out_h, out_w):
    x = _c32(x)
    c, h, w = x.shape
    out = np.empty((c, out_h, out_w), np.float32)
    if lib().zo_resize_bicubic(_fp(x), c, h, w, out_h, out_w, _fp(out)):
        raise ValueError("resize_bicubic")
    return out


def to_rgb_planes(y, u, v):
    r, g, b = _c32(y).copy(), _c32(u).copy(), _c32(v).copy()
    lib().zo_to_rgb_planes(_fp(r), _fp(g), _fp(b), r.size)
    return r, g, b


def quantize_rgb(r, g, b, bit_depth=8):
    r, g, b = _c32(r), _c32(g), _c32(b)
    out = np.empty(r.shape + (3,), np.uint16)
    lib().zo_quantize_rgb(_fp(r), _fp(g), _fp(b), r.size, bit_depth,
                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)))
    return out


def pad_amount(n, d):
    return lib().zo_pad_amount(n, d)


def preprocess_rgb(rgb):
    """`preprocess_rgb` (colour.rs:535-541): uint8 RGB [h, w, 3] -> (luma [1, h, w],
    chroma [12, ph / 2, pw / 2]) in [0, 255]."""
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w, _ = rgb.shape
    luma = np.empty((1, h, w), np.float32)
    chroma = np.empty((12, (h + h % 2) // 2, (w + w % 2) // 2), np.float32)
    lib().zo_preprocess_rgb(rgb.ctypes.data, h, w, _fp(luma), _fp(chroma))
    return luma, chroma


def analysis_tiles(ccs, h, w, lh, lw):
    """`analysis_tiles` (encoder/tiles.rs:51-156) as a list of dicts."""
    n = lib().zo_analysis_tiles(ccs, h, w, lh, lw, None, 0)
    if n <= 0:
        raise ValueError("malformed analysis tiling")
    arr = (ATile * n)()
    lib().zo_analysis_tiles(ccs, h, w, lh, lw, ctypes.cast(arr, ctypes.c_void_p), n)
    return [{k: getattr(t, k) for k, _ in ATile._fields_} for t in arr]


def analyze_tiled(ck, op, ccs, x):
    """Tiled analysis of component ccs: x [1 or 12, h, w] -> latent [160 or 96, ., .]."""
    x = _c32(x)
    _, h, w = x.shape
    d = 8 if ccs else 16
    out = np.empty((96 if ccs else 160, -(-h // d), -(-w // d)), np.float32)
    if lib().zo_analyze_tiled(ctypes.byref(ck.ck), op, ccs, _fp(x), h, w, _fp(out)):
        raise ValueError("analyze_tiled")
    return out
