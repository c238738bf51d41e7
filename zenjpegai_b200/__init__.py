"""zenjpegai_b200 — B200 (sm_100a) engine for the JPEG AI synthesis / analysis networks.

Python host side over the C ABI of `include/zjai.h` (library `libzjai.so`, built by
`zenjpegai_b200/build.py`). It mirrors the reference crate's interfaces for this path:

* `Engine` — the crate's `Engine` (src/nn/fast/mod.rs:127-169): here a CUDA context on one
  GPU (stream, device arena, kernel status word).
* `nn` layer calls — `ConvLayer` / `ConvTransposeLayer` / `math::*` (src/nn/fast/layers.rs,
  math.rs) on planar `[c, h, w]` f32 tensors.
* `SynthesisPrimary`, `SynthesisSecondary`, `AnalysisPrimary`, `AnalysisSecondary` — the
  network types of src/model/{synthesis,analysis}.rs: `load(params, op, engine)` +
  `forward(...)`.
* `synthesize` / `synthesis_tiles` — src/decoder/reconstruct.rs:274-464 and
  src/tools/tiles.rs:39-119.
* `LatentModel` — the float networks of src/model/common.rs `CommonModel`: the hyper-decoder
  (hyper_decoder.rs) and the optional context model (mcm.rs), with reconstruct.rs:107-230's
  one-region latent reconstruction.

Arrays are numpy float32 (host memory) or torch CUDA float32 tensors (device memory of the
engine's GPU). Errors raise `ZjaiError` whose `.status` mirrors the crate's `Error` variant.
There is no CPU fallback: without the CUDA library this package does not import.
"""

import ctypes

import numpy as np

from . import _lib
from ._lib import (ACT_LEAKY, ACT_NONE, ACT_RELU, ACT_RELU6, ACT_SIGMOID, ANA_UV, ANA_Y, BOP,
                   HOP, ICCI, LATENT, SOP, SYN_UV, SYN_Y, ZjaiError, check)

__all__ = ["Engine", "ZjaiError", "SOP", "BOP", "HOP", "SYN_Y", "SYN_UV", "ANA_Y", "ANA_UV",
           "ACT_NONE", "ACT_RELU", "ACT_LEAKY", "ACT_SIGMOID", "ACT_RELU6", "Network", "Stage",
           "LatentModel", "LATENT", "ICCI",
           "synthesis_tiles", "synth_out_size", "version"]

_lib.lib()  # load now: importing the package without its CUDA library is an error


def version():
    return _lib.lib().zjai_version().decode()


def _is_torch(a):
    return type(a).__module__.startswith("torch")


def _arg(a, want_shape=None, writable=False):
    """(pointer, mem) of a numpy host array or a torch CUDA tensor (float32, contiguous)."""
    if _is_torch(a):
        import torch
        if a.dtype != torch.float32 or not a.is_contiguous():
            raise ZjaiError(_lib.INVALID_ARGUMENT, "tensor must be contiguous float32")
        if want_shape is not None and tuple(a.shape) != tuple(want_shape):
            raise ZjaiError(_lib.INVALID_ARGUMENT, "shape %s, expected %s"
                            % (tuple(a.shape), tuple(want_shape)))
        if not a.is_cuda:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "torch tensors must be CUDA tensors")
        return ctypes.c_void_p(a.data_ptr()), _lib.MEM_DEVICE
    if not isinstance(a, np.ndarray) or a.dtype != np.float32 or not a.flags.c_contiguous:
        raise ZjaiError(_lib.INVALID_ARGUMENT, "array must be a contiguous float32 ndarray")
    if want_shape is not None and tuple(a.shape) != tuple(want_shape):
        raise ZjaiError(_lib.INVALID_ARGUMENT, "shape %s, expected %s"
                        % (a.shape, tuple(want_shape)))
    return ctypes.c_void_p(a.ctypes.data), _lib.MEM_HOST


def _like(x, shape):
    if _is_torch(x):
        import torch
        return torch.empty(shape, dtype=torch.float32, device=x.device)
    return np.empty(shape, np.float32)


class Engine:
    """A CUDA context on one GPU (the crate's `Engine`, GPU kind)."""

    def __init__(self, device=0, arena_bytes=0):
        h = ctypes.c_void_p()
        check(_lib.lib().zjai_ctx_create(int(device), int(arena_bytes), ctypes.byref(h)))
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            _lib.lib().zjai_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, cuda_stream_ptr):
        check(_lib.lib().zjai_ctx_set_stream(self.handle, ctypes.c_void_p(cuda_stream_ptr)))

    def sync(self):
        check(_lib.lib().zjai_ctx_sync(self.handle))

    def set_output_clamp(self, clamp):
        """False: synthesis planes without the final [0, 255] clamp (diagnostics)."""
        check(_lib.lib().zjai_ctx_set_output_clamp(self.handle, 1 if clamp else 0))

    def set_wait_limit(self, cycles):
        """Limit of the convolution kernel's pipeline waits in SM cycles (0: default)."""
        check(_lib.lib().zjai_ctx_set_wait_limit(self.handle, int(cycles)))

    def set_graphs(self, enable):
        """Replay repeated device calls of the tiled synthesis as CUDA graphs (captured on the
        second call with the same arguments)."""
        check(_lib.lib().zjai_ctx_set_graphs(self.handle, 1 if enable else 0))

    def set_probe(self, name, buf):
        """Capture the intermediate map `name` ("ana.act1" ..) of later network runs into `buf`
        (a float32 CUDA tensor, planar [n, c, h, w] or larger); buf None removes it."""
        if buf is None:
            check(_lib.lib().zjai_ctx_set_probe(self.handle, name.encode(), None, 0))
            return
        p, mem = _arg(buf)
        if mem != _lib.MEM_DEVICE:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "a probe buffer must be a CUDA tensor")
        check(_lib.lib().zjai_ctx_set_probe(self.handle, name.encode(), p, buf.numel()))

    @property
    def launch_count(self):
        return int(_lib.lib().zjai_ctx_launch_count(self.handle))

    # ---- nn layer interface (src/nn/fast/layers.rs, math.rs) ------------------------------
    def conv2d(self, x, weight, bias=None, stride=1, pad=(0, 0), groups=1, extra=None,
               act=ACT_NONE, out=None):
        c, h, w = x.shape
        oc, _, kh, kw = weight.shape
        ex = extra or (0, 0, 0, 0)
        oh = (h + ex[0] + ex[2] + 2 * pad[0] - kh) // stride + 1
        ow = (w + ex[1] + ex[3] + 2 * pad[1] - kw) // stride + 1
        if out is None:
            out = _like(x, (oc, oh, ow))
        px, mem = _arg(x)
        pw, m2 = _arg(weight)
        pb = _arg(bias)[0] if bias is not None else None
        po, m3 = _arg(out, (oc, oh, ow))
        if len({mem, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        exa = (ctypes.c_int * 4)(*ex)
        check(_lib.lib().zjai_conv2d(self.handle, px, c, h, w, pw, pb, oc, kh, kw, stride,
                                     pad[0], pad[1], groups, exa, act, po, mem))
        return out

    def conv_transpose2d(self, x, weight, bias=None, pad=1, out_pad=0, out=None):
        c, h, w = x.shape
        _, oc, k, _ = weight.shape
        oh = (h - 1) * 2 + k + out_pad - 2 * pad
        ow = (w - 1) * 2 + k + out_pad - 2 * pad
        if out is None:
            out = _like(x, (oc, oh, ow))
        px, mem = _arg(x)
        pw, _ = _arg(weight)
        pb = _arg(bias)[0] if bias is not None else None
        po, _ = _arg(out, (oc, oh, ow))
        check(_lib.lib().zjai_conv_transpose2d(self.handle, px, c, h, w, pw, pb, oc, k, pad,
                                               out_pad, po, mem))
        return out

    def conv2d_backward(self, dout, weight, h, w, stride=1, pad=(0, 0), groups=1, extra=None,
                        out=None):
        """Input gradient of `conv2d` (`ConvLayer::backward`, the RDLR VJP): dout [oc, oh, ow]
        of the layer on an input [c, h, w] -> [c, h, w]."""
        oc, oh, ow = dout.shape
        _, icg, kh, kw = weight.shape
        c = icg * groups
        if out is None:
            out = _like(dout, (c, h, w))
        pd, mem = _arg(dout)
        pw, m2 = _arg(weight)
        po, m3 = _arg(out, (c, h, w))
        if len({mem, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        exa = (ctypes.c_int * 4)(*extra) if extra else None
        check(_lib.lib().zjai_conv2d_backward(self.handle, pd, oc, oh, ow, pw, c, kh, kw, stride,
                                              pad[0], pad[1], groups, exa, h, w, po, mem))
        return out

    def conv_transpose2d_backward(self, dout, weight, h, w, pad=1, out=None):
        """Input gradient of the stride-2 `conv_transpose2d` (`ConvTransposeLayer::backward`):
        dout [oc, oh, ow], weight [c, oc, k, k] -> [c, h, w]."""
        oc, oh, ow = dout.shape
        c, _, k, _ = weight.shape
        if out is None:
            out = _like(dout, (c, h, w))
        pd, mem = _arg(dout)
        pw, m2 = _arg(weight)
        po, m3 = _arg(out, (c, h, w))
        if len({mem, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_conv_transpose2d_backward(self.handle, pd, oc, oh, ow, pw, c, k, pad,
                                                        h, w, po, mem))
        return out

    def residual_block_backward(self, dout, conv1_out, w1, w2, out=None):
        """`ResidualBlock::backward` (the RDLR VJP of conv3x3 -> ReLU -> conv3x3 + x): dout and
        the tape conv1_out [c, h, w], conv weights [c, c, 3, 3] -> d_x [c, h, w]."""
        c, h, w = dout.shape
        if out is None:
            out = _like(dout, (c, h, w))
        pd, mem = _arg(dout)
        pt, m1 = _arg(conv1_out, (c, h, w))
        p1, m2 = _arg(w1, (c, c, 3, 3))
        p2, m3 = _arg(w2, (c, c, 3, 3))
        po, m4 = _arg(out, (c, h, w))
        if len({mem, m1, m2, m3, m4}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_residual_block_backward(self.handle, pd, pt, c, h, w, p1, p2, po,
                                                      mem))
        return out

    def elu_gate_backward(self, d, a, b):
        """`elu_gate_backward` (math.rs:838-858): (d_a, d_b) of y = elu(a) . b."""
        pd, mem = _arg(d)
        pa, m1 = _arg(a, tuple(d.shape))
        pb, m2 = _arg(b, tuple(d.shape))
        oa, ob = _like(d, tuple(d.shape)), _like(d, tuple(d.shape))
        if len({mem, m1, m2}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        n = int(np.prod(d.shape))
        check(_lib.lib().zjai_elu_gate_backward(self.handle, pd, pa, pb, n, _arg(oa)[0],
                                                _arg(ob)[0], mem))
        return oa, ob

    def layer_norm_backward(self, d, x, weight, out=None):
        """`layer_norm_channels_backward` (math.rs:860-913): d, x [c, h, w], weight [c]."""
        c, h, w = x.shape
        out = _like(x, (c, h, w)) if out is None else out
        pd, mem = _arg(d, (c, h, w))
        px, m1 = _arg(x)
        pw, m2 = _arg(weight, (c,))
        po, m3 = _arg(out, (c, h, w))
        if len({mem, m1, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_layer_norm_backward(self.handle, pd, px, c, h, w, pw, po, mem))
        return out

    def channel_attention_backward(self, qkv, heads, temperature, attn, dout, out=None):
        """`channel_attention_backward` (math.rs:668-836): qkv [3 dim, h, w], the forward's
        softmax weights attn [dim, dim / heads], dout [dim, h, w] -> dqkv [3 dim, h, w]."""
        c3, h, w = qkv.shape
        out = _like(qkv, (c3, h, w)) if out is None else out
        pq, mem = _arg(qkv)
        pt, m1 = _arg(temperature, (heads,))
        pa, m2 = _arg(attn, (c3 // 3, c3 // 3 // heads))
        pd, m3 = _arg(dout, (c3 // 3, h, w))
        po, m4 = _arg(out, (c3, h, w))
        if len({mem, m1, m2, m3, m4}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_channel_attention_backward(self.handle, pq, c3, h, w, heads, pt, pa,
                                                         pd, po, mem))
        return out

    def transformer_block_backward(self, dout, heads, hidden, tape, weights, out=None):
        """`TransformerBlock::backward` (attention.rs:435-480): dout [dim, h, w]; tape {"x_in",
        "qkv", "attn", "x_mid", "gate"}; weights {"prep_norm", "prep_conv1", "prep_conv2",
        "temperature", "attn_out", "ffn_norm", "ffn_in", "ffn_dw", "ffn_out"} -> d_x."""
        dim, h, w = dout.shape
        out = _like(dout, (dim, h, w)) if out is None else out
        pd, mem = _arg(dout)
        po, m = _arg(out, (dim, h, w))
        mems = {mem, m}
        t, wt = _lib.TbTape(), _lib.TbWeights()
        for k, _ in _lib.TbTape._fields_:
            p, m = _arg(tape[k])
            setattr(t, k, p)
            mems.add(m)
        for k, _ in _lib.TbWeights._fields_:
            p, m = _arg(weights[k])
            setattr(wt, k, p)
            mems.add(m)
        if len(mems) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_transformer_block_backward(self.handle, pd, dim, hidden, heads, h,
                                                         w, ctypes.byref(t), ctypes.byref(wt),
                                                         po, mem))
        return out

    CAB_WEIGHTS = ("trunk0.conv1", "trunk0.conv2", "trunk1.conv1", "trunk1.conv2", "subscale",
                   "mask2.conv1", "mask2.conv2", "mask3.conv1", "mask3.conv2", "upscale")

    def cab_backward(self, dout, tape, weights, out=None):
        """`Cab::backward` (the RDLR VJP of x + trunk(x) . sigmoid(mask(x))): dout [c, h, w];
        tape {"trunk_pre", "sig", "rb_c1": [2 arrays], "mask_c1": [2 arrays at h/2 x w/2]};
        weights {name in CAB_WEIGHTS: [c, c, 3, 3]} -> d_x [c, h, w]."""
        c, h, w = dout.shape
        if out is None:
            out = _like(dout, (c, h, w))
        pd, mem = _arg(dout)
        po, m = _arg(out, (c, h, w))
        mems = {mem, m}
        t = _lib.CabTape()
        for name in ("trunk_pre", "sig"):
            p, m = _arg(tape[name], (c, h, w))
            setattr(t, name, p)
            mems.add(m)
        for i in range(2):
            p, m = _arg(tape["rb_c1"][i], (c, h, w))
            t.rb_c1[i] = p
            mems.add(m)
            p, m = _arg(tape["mask_c1"][i], (c, h // 2, w // 2))
            t.mask_c1[i] = p
            mems.add(m)
        wts = _lib.CabWeights()
        ptr = {}
        for k in self.CAB_WEIGHTS:
            ptr[k], m = _arg(weights[k], (c, c, 3, 3))
            mems.add(m)
        for i in range(2):
            for j in range(2):
                wts.trunk[i][j] = ptr["trunk%d.conv%d" % (i, j + 1)]
            wts.mask2[i] = ptr["mask2.conv%d" % (i + 1)]
            wts.mask3[i] = ptr["mask3.conv%d" % (i + 1)]
        wts.subscale, wts.upscale = ptr["subscale"], ptr["upscale"]
        if len(mems) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_cab_backward(self.handle, pd, c, h, w, ctypes.byref(t),
                                           ctypes.byref(wts), po, mem))
        return out

    def layer_norm(self, x, weight, bias, out=None):
        c, h, w = x.shape
        out = _like(x, x.shape) if out is None else out
        px, mem = _arg(x)
        check(_lib.lib().zjai_layer_norm(self.handle, px, c, h, w, _arg(weight)[0],
                                         _arg(bias)[0], _arg(out, x.shape)[0], mem))
        return out

    def channel_attention(self, qkv, heads, temperature, out=None):
        c3, h, w = qkv.shape
        out = _like(qkv, (c3 // 3, h, w)) if out is None else out
        px, mem = _arg(qkv)
        check(_lib.lib().zjai_channel_attention(self.handle, px, c3, h, w, heads,
                                                _arg(temperature)[0],
                                                _arg(out, (c3 // 3, h, w))[0], mem))
        return out

    def depthwise3x3(self, x, weight, out=None):
        c, h, w = x.shape
        out = _like(x, x.shape) if out is None else out
        px, mem = _arg(x)
        check(_lib.lib().zjai_depthwise3x3(self.handle, px, c, h, w, _arg(weight)[0],
                                           _arg(out, x.shape)[0], mem))
        return out

    def depthwise3x3_elu_gate(self, x, weight, out=None):
        """The FFN's depthwise conv then `math::elu_gate` (attention.rs:347-355), fused:
        [c, h, w] -> [c/2, h, w]."""
        c, h, w = x.shape
        shape = (c // 2, h, w)
        out = _like(x, shape) if out is None else out
        px, mem = _arg(x)
        check(_lib.lib().zjai_depthwise3x3_elu_gate(self.handle, px, c, h, w, _arg(weight)[0],
                                                    _arg(out, shape)[0], mem))
        return out

    def transformer_ffn(self, x, norm_weight, norm_bias, w_in, w_dw, w_out, out=None):
        """The feed-forward half of `TransformerBlock::forward` (attention.rs:346-371):
        x + W_out . gate(dw3x3(W_in . layer_norm(x))) for x [c, h, w], w_in [2 hidden, c(,1,1)],
        w_dw [2 hidden(,1), 3, 3], w_out [c, hidden(,1,1)]."""
        c, h, w = x.shape
        hidden = w_in.shape[0] // 2
        out = _like(x, (c, h, w)) if out is None else out
        px, mem = _arg(x)
        check(_lib.lib().zjai_transformer_ffn(
            self.handle, px, c, h, w, hidden, _arg(norm_weight)[0], _arg(norm_bias)[0],
            _arg(w_in)[0], _arg(w_dw)[0], _arg(w_out)[0], _arg(out, (c, h, w))[0], mem))
        return out


def synth_out_size(kind, op, h, w):
    oh, ow = ctypes.c_int(), ctypes.c_int()
    check(_lib.lib().zjai_synth_out_size(kind, op, h, w, ctypes.byref(oh), ctypes.byref(ow)))
    return oh.value, ow.value


def synthesis_tiles(height, width, latent_h, latent_w, tile_size=0, overlap=0):
    """`synthesis_tiles` (src/tools/tiles.rs:39-119): list of tile dicts."""
    n = ctypes.c_int()
    check(_lib.lib().zjai_synthesis_tiles(height, width, latent_h, latent_w, tile_size,
                                          overlap, None, 0, ctypes.byref(n)))
    arr = (_lib.Tile * n.value)()
    check(_lib.lib().zjai_synthesis_tiles(height, width, latent_h, latent_w, tile_size,
                                          overlap, arr, n.value, ctypes.byref(n)))
    return [{k: getattr(t, k) for k, _ in _lib.Tile._fields_} for t in arr]


def _param_array(params):
    """ctypes array of zjai_param over float32 copies of `params` (name -> array), and the
    objects that must stay alive while it is used."""
    arrs = {k: np.ascontiguousarray(v, dtype=np.float32) for k, v in params.items()}
    ps = (_lib.Param * max(1, len(arrs)))()
    keep = [arrs]
    for i, (k, v) in enumerate(arrs.items()):
        nm = k.encode()
        keep.append(nm)
        ps[i].name = nm
        ps[i].ndim = v.ndim
        for d in range(4):
            ps[i].shape[d] = v.shape[d] if d < v.ndim else 0
        ps[i].data = v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    return ps, len(arrs), keep


class Network:
    """A synthesis / analysis network with GPU-resident packed weights
    (`SynthesisPrimary::load` etc.). `params` maps checkpoint names to float32 arrays."""

    def __init__(self, engine, kind, op, params):
        self.engine = engine
        self.kind = kind
        self.op = op
        ps, n, keep = _param_array(params)
        h = ctypes.c_void_p()
        check(_lib.lib().zjai_net_create(engine.handle, kind, op, ps, n, ctypes.byref(h)))
        self.handle = h

    def close(self):
        if self.handle:
            _lib.lib().zjai_net_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Stage(Network):
    """A conv stage (zjai_stage_create): conv k x k (+ `act`, + depth-to-space `shuffle`) then
    the residual blocks `res.<i>` with `res_act` between their convs."""

    def __init__(self, engine, params, shuffle=1, act=ACT_NONE, res_act=ACT_RELU):
        self.engine = engine
        self.kind, self.op = 4, 0
        w = params["conv.weight"]
        self.cin = int(w.shape[1])
        self.cout = int(w.shape[0]) // (shuffle * shuffle)
        self.shuffle = shuffle
        ps, n, keep = _param_array(params)
        h = ctypes.c_void_p()
        check(_lib.lib().zjai_stage_create(engine.handle, shuffle, act, res_act, ps, n,
                                           ctypes.byref(h)))
        self.handle = h

    def forward(self, x, out=None):
        c, h, w = x.shape
        shape = (self.cout, h * self.shuffle, w * self.shuffle)
        if out is None:
            out = _like(x, shape)
        px, mem = _arg(x)
        po, m2 = _arg(out, shape)
        if mem != m2:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_stage_forward(self.handle, px, c, h, w, po, mem))
        return out


class LatentModel(Network):
    """The latent-domain float networks of one component (`CommonModel`, common.rs:34-131):
    `HyperDecoder` and, when `params` hold "context.MCM.*", the `ContextModel`. C is the
    checkpoint's channel count (160 luma, 96 chroma)."""

    def __init__(self, engine, params):
        super().__init__(engine, LATENT, 0, params)
        self.chs = int(params["hyper_decoder.conv1.weight"].shape[0])
        self.has_context = "context.MCM.0.fusion_pred_net.conv1.weight" in params

    def hyper_decode(self, z_hat, out_h, out_w, out=None):
        """`HyperDecoder::forward_f32` (hyper_decoder.rs:94-113): z_hat [C, hz, wz] -> psi
        [4C, out_h, out_w]."""
        c, hz, wz = z_hat.shape
        shape = (4 * self.chs, out_h, out_w)
        if out is None:
            out = _like(z_hat, shape)
        pz, mem = _arg(z_hat, (self.chs, hz, wz))
        po, m2 = _arg(out, shape)
        if mem != m2:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_hyper_decode(self.handle, pz, hz, wz, out_h, out_w, po, mem))
        return out

    def decompress(self, residual, psi, out=None):
        """y_hat [C, h, w] from the residual [C, h, w] and psi [4C, ceil(h/2), ceil(w/2)]
        (reconstruct.rs:200-212: the context model, or upshuffle_psi + residual)."""
        c, h, w = residual.shape
        if out is None:
            out = _like(residual, (c, h, w))
        pr, mem = _arg(residual, (self.chs, h, w))
        pp, m2 = _arg(psi, (4 * self.chs, -(-h // 2), -(-w // 2)))
        po, m3 = _arg(out, (self.chs, h, w))
        if len({mem, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_context_decompress(self.handle, pr, h, w, pp, po, mem))
        return out

    def reconstruct(self, z_hat, residual, with_psi=False):
        """One region of `reconstruct_latent` (reconstruct.rs:107-230): (y_hat, psi or None)."""
        c, hz, wz = z_hat.shape
        _, h, w = residual.shape
        y = _like(residual, (self.chs, h, w))
        psi = _like(residual, (4 * self.chs, -(-h // 2), -(-w // 2))) if with_psi else None
        pz, mem = _arg(z_hat, (self.chs, hz, wz))
        pr, m2 = _arg(residual, (self.chs, h, w))
        py, m3 = _arg(y)
        pp = _arg(psi)[0] if with_psi else None
        if len({mem, m2, m3}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
        check(_lib.lib().zjai_reconstruct_latent(self.handle, pz, hz, wz, pr, h, w, pp, py, mem))
        return y, psi
