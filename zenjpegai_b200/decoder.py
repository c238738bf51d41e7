"""Decoder / Encoder front ends of the GPU path, mirroring the crate's public API for the part
of the pipeline this engine replaces.

`Decoder` stands in for `zenjpegai::Decoder` (src/decoder/api.rs:38-458) from the point where the
entropy stage has produced the latents: `synthesize` is `synthesize_with`
(src/decoder/reconstruct.rs:274-331), `finish_yuv` / `finish_rgb` are the output stage
(src/decoder/output.rs). Entropy decoding stays on the host and is not part of this package.
`Encoder.analyze` stands in for the analysis transforms the crate's `Encoder` runs
(src/model/analysis.rs) on pre-processed planes.

Arrays are numpy float32 (host) or torch CUDA tensors (device), as in the package root.
"""

import ctypes

import numpy as np

from . import _lib
from ._lib import ZjaiError, check
from . import Engine, Network, SYN_Y, SYN_UV, ANA_Y, ANA_UV, synthesis_tiles, _arg

OPS = {"sop": _lib.SOP, "bop": _lib.BOP, "hop": _lib.HOP}


def _op(op):
    return OPS[op] if isinstance(op, str) else int(op)


def _cdiv(a, b):
    return -(-a // b)


def _ptr(a):
    """Address of an integer sample plane (torch tensor or numpy array)."""
    return ctypes.c_void_p(a.data_ptr() if hasattr(a, "data_ptr") else a.ctypes.data)


class Decoder:
    """Synthesis networks of one operating point, loaded once (the crate's model cache,
    api.rs:135-157) and reused for every picture."""

    def __init__(self, engine, op, params_y, params_uv):
        self.engine = engine
        self.op = _op(op)
        self.net_y = Network(engine, SYN_Y, self.op, params_y)
        self.net_uv = Network(engine, SYN_UV, self.op, params_uv)

    def close(self):
        self.net_y.close()
        self.net_uv.close()

    def _planes(self, like, out_h, out_w, sv, sh, bit_depth=None):
        """Zeroed output planes: f32, or the integer samples of `bit_depth` (uint8 for 8 bits,
        else uint16; int16 storage for torch, which has no uint16)."""
        ch, cw = _cdiv(out_h, sv), _cdiv(out_w, sh)
        if type(like).__module__.startswith("torch"):
            import torch
            dt = (torch.float32 if bit_depth is None else
                  torch.uint8 if bit_depth == 8 else torch.int16)
            z = lambda s: torch.zeros(s, dtype=dt, device=like.device)
        else:
            dt = np.float32 if bit_depth is None else np.uint8 if bit_depth == 8 else np.uint16
            z = lambda s: np.zeros(s, dt)
        return z((out_h, out_w)), z((ch, cw)), z((ch, cw))

    def synthesize(self, y_hat_y, y_hat_uv, height, width, out_h=None, out_w=None,
                   tile_size=0, overlap=0, sv=2, sh=2, out=None, cancel=None, bit_depth=None):
        """Whole picture: latents [160, lh, lw] / [96, lh, lw] -> planes (y, u, v) in [0, 255]
        (`synthesize_with`, reconstruct.rs:274-331). `cancel` is an optional ctypes c_int
        polled between tiles and layers (the crate's `Stop`). With `bit_depth`, the planes are
        the quantized samples (`quantize_plane_par`, output.rs:330-342) written by the final
        layers directly (the fused output stage)."""
        out_h = height if out_h is None else out_h
        out_w = width if out_w is None else out_w
        _, lh, lw = y_hat_y.shape
        ry, ru, rv = out if out is not None else self._planes(y_hat_y, out_h, out_w, sv, sh,
                                                              bit_depth)
        py, mem = _arg(y_hat_y, (160, lh, lw))
        puv, _ = _arg(y_hat_uv, (96, lh, lw))
        stop = ctypes.byref(cancel) if cancel is not None else None
        if bit_depth is None:
            check(_lib.lib().zjai_synthesize(
                self.engine.handle, self.net_y.handle, self.net_uv.handle, py, puv, lh, lw,
                height, width, out_h, out_w, tile_size, overlap, sv, sh, _arg(ry)[0],
                _arg(ru)[0], _arg(rv)[0], mem, stop))
        else:
            check(_lib.lib().zjai_synthesize_q(
                self.engine.handle, self.net_y.handle, self.net_uv.handle, py, puv, lh, lw,
                height, width, out_h, out_w, tile_size, overlap, sv, sh, bit_depth,
                _ptr(ry), _ptr(ru), _ptr(rv), mem, stop))
        return ry, ru, rv

    def synthesize_tiles(self, y_hat_y, y_hat_uv, tiles, out_h, out_w, sv=2, sh=2, out=None,
                         cancel=None, bit_depth=None):
        """Only the listed tiles (a shard of `synthesis_tiles`); planes outside their cores
        are left as they are. `bit_depth`: quantized sample planes as in `synthesize`."""
        _, lh, lw = y_hat_y.shape
        ry, ru, rv = out if out is not None else self._planes(y_hat_y, out_h, out_w, sv, sh,
                                                              bit_depth)
        arr = (_lib.Tile * max(1, len(tiles)))()
        for i, t in enumerate(tiles):
            for k, _ in _lib.Tile._fields_:
                setattr(arr[i], k, int(t[k]))
        py, mem = _arg(y_hat_y, (160, lh, lw))
        puv, _ = _arg(y_hat_uv, (96, lh, lw))
        stop = ctypes.byref(cancel) if cancel is not None else None
        if bit_depth is None:
            check(_lib.lib().zjai_synthesize_tiles(
                self.engine.handle, self.net_y.handle, self.net_uv.handle, py, puv, lh, lw, arr,
                len(tiles), out_h, out_w, sv, sh, _arg(ry)[0], _arg(ru)[0], _arg(rv)[0], mem,
                stop))
        else:
            check(_lib.lib().zjai_synthesize_tiles_q(
                self.engine.handle, self.net_y.handle, self.net_uv.handle, py, puv, lh, lw, arr,
                len(tiles), out_h, out_w, sv, sh, bit_depth, _ptr(ry), _ptr(ru), _ptr(rv), mem,
                stop))
        return ry, ru, rv

    def synthesize_rgb(self, y_hat_y, y_hat_uv, height, width, tile_size=0, overlap=0,
                       bit_depth=8, cancel=None):
        """Whole picture straight to interleaved RGB [h, w, 3] (synthesis, then bicubic
        4:2:0 -> 4:4:4, BT.709 and rounding on the device; output.rs:124-262, 407-438)."""
        _, lh, lw = y_hat_y.shape
        if type(y_hat_y).__module__.startswith("torch"):
            import torch
            out = torch.empty((height, width, 3), dtype=torch.uint8 if bit_depth == 8
                              else torch.int16, device=y_hat_y.device)
        else:
            out = np.empty((height, width, 3), np.uint8 if bit_depth == 8 else np.uint16)
        py, mem = _arg(y_hat_y, (160, lh, lw))
        puv, _ = _arg(y_hat_uv, (96, lh, lw))
        stop = ctypes.byref(cancel) if cancel is not None else None
        check(_lib.lib().zjai_synthesize_rgb(
            self.engine.handle, self.net_y.handle, self.net_uv.handle, py, puv, lh, lw, height,
            width, tile_size, overlap, bit_depth, _ptr(out), mem, stop))
        return out

    def synthesize_batch(self, y_hat_y, y_hat_uv, height, width, tile_size=0, overlap=0, sv=1,
                         sh=1, bit_depth=8, out=None, cancel=None):
        """n independent pictures of one size in one call: latents [n, 160, lh, lw] /
        [n, 96, lh, lw] -> planes ([n, h, w], [n, ch, cw], [n, ch, cw]) of quantized samples
        (bit_depth 8..16) or f32 (bit_depth 0)."""
        n, _, lh, lw = y_hat_y.shape
        ch, cw = _cdiv(height, sv), _cdiv(width, sh)
        if out is None:
            if type(y_hat_y).__module__.startswith("torch"):
                import torch
                dt = (torch.float32 if bit_depth == 0 else
                      torch.uint8 if bit_depth == 8 else torch.int16)
                z = lambda s: torch.zeros(s, dtype=dt, device=y_hat_y.device)
            else:
                dt = np.float32 if bit_depth == 0 else np.uint8 if bit_depth == 8 else np.uint16
                z = lambda s: np.zeros(s, dt)
            out = (z((n, height, width)), z((n, ch, cw)), z((n, ch, cw)))
        ry, ru, rv = out
        py, mem = _arg(y_hat_y)
        puv, _ = _arg(y_hat_uv)
        stop = ctypes.byref(cancel) if cancel is not None else None
        check(_lib.lib().zjai_synthesize_batch(
            self.engine.handle, self.net_y.handle, self.net_uv.handle, n, py, puv, lh, lw,
            height, width, height, width, tile_size, overlap, sv, sh, bit_depth, _ptr(ry),
            _ptr(ru), _ptr(rv), mem, stop))
        return ry, ru, rv

    # ---- output stage (src/decoder/output.rs) -------------------------------------------
    def quantize_plane(self, x, bit_depth=8, out=None):
        """`quantize_plane_par` (output.rs:330-342); uint8 for 8-bit, else uint16."""
        dt = np.uint8 if bit_depth == 8 else np.uint16
        if out is None:
            if type(x).__module__.startswith("torch"):
                import torch
                out = torch.empty(tuple(x.shape), dtype=torch.uint8 if bit_depth == 8
                                  else torch.int16, device=x.device)
            else:
                out = np.empty(x.shape, dt)
        px, mem = _arg(x)
        po = ctypes.c_void_p(out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data)
        n = int(np.prod(tuple(x.shape)))
        check(_lib.lib().zjai_quantize_plane(self.engine.handle, px, n, bit_depth, po, mem))
        return out

    def yuv_to_rgb(self, y, u, v, bit_depth=8, out=None):
        """Bicubic 4:2:0 -> 4:4:4, BT.709, round half to even (output.rs:103-262, 407-438):
        interleaved RGB [h, w, 3]."""
        h, w = y.shape
        ch, cw = u.shape
        if out is None:
            if type(y).__module__.startswith("torch"):
                import torch
                out = torch.empty((h, w, 3), dtype=torch.uint8 if bit_depth == 8
                                  else torch.int16, device=y.device)
            else:
                out = np.empty((h, w, 3), np.uint8 if bit_depth == 8 else np.uint16)
        py, mem = _arg(y)
        po = ctypes.c_void_p(out.data_ptr() if hasattr(out, "data_ptr") else out.ctypes.data)
        check(_lib.lib().zjai_yuv_to_rgb(self.engine.handle, py, _arg(u)[0], _arg(v)[0], h, w,
                                         ch, cw, bit_depth, po, mem))
        return out


class Encoder:
    """Analysis transforms (src/model/analysis.rs) of one operating point (BOP / HOP)."""

    def __init__(self, engine, op, params_y, params_uv):
        self.engine = engine
        self.op = _op(op)
        self.net_y = Network(engine, ANA_Y, self.op, params_y)
        self.net_uv = Network(engine, ANA_UV, self.op, params_uv)

    def close(self):
        self.net_y.close()
        self.net_uv.close()

    def analyze(self, luma, chroma12):
        """luma [1, h, w] and chroma [12, h/2, w/2] in [0, 255] -> latents
        ([160, ceil(h/16), ceil(w/16)], [96, ceil(h2/8), ceil(w2/8)])."""
        _, h, w = luma.shape
        _, h2, w2 = chroma12.shape
        if type(luma).__module__.startswith("torch"):
            import torch
            ly = torch.empty((160, _cdiv(h, 16), _cdiv(w, 16)), device=luma.device)
            luv = torch.empty((96, _cdiv(h2, 8), _cdiv(w2, 8)), device=luma.device)
        else:
            ly = np.empty((160, _cdiv(h, 16), _cdiv(w, 16)), np.float32)
            luv = np.empty((96, _cdiv(h2, 8), _cdiv(w2, 8)), np.float32)
        px, mem = _arg(luma)
        check(_lib.lib().zjai_analysis_primary(self.net_y.handle, px, h, w, _arg(ly)[0], mem))
        check(_lib.lib().zjai_analysis_secondary(self.net_uv.handle, _arg(chroma12)[0], h2, w2,
                                                 _arg(luv)[0], mem))
        return ly, luv

    def analyze_rgb(self, rgb, out=None):
        """n 8-bit RGB pictures [n, h, w, 3] (numpy uint8 or a torch CUDA uint8 tensor) ->
        latents ([n, 160, ceil(h/16), ceil(w/16)], [n, 96, ceil(ceil(h/2)/8), ...]):
        `preprocess_rgb` and both analysis transforms, tiled like the crate's encoder."""
        n, h, w, _ = rgb.shape
        h2, w2 = _cdiv(h, 2), _cdiv(w, 2)
        shapes = ((n, 160, _cdiv(h, 16), _cdiv(w, 16)), (n, 96, _cdiv(h2, 8), _cdiv(w2, 8)))
        if out is None:
            if type(rgb).__module__.startswith("torch"):
                import torch
                out = tuple(torch.empty(s, device=rgb.device) for s in shapes)
            else:
                out = tuple(np.empty(s, np.float32) for s in shapes)
        ly, luv = out
        mem = _lib.MEM_DEVICE if type(rgb).__module__.startswith("torch") else _lib.MEM_HOST
        if mem == _lib.MEM_HOST:
            rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        check(_lib.lib().zjai_analyze_rgb(self.engine.handle, self.net_y.handle,
                                          self.net_uv.handle, n, _ptr(rgb), h, w, _ptr(ly),
                                          _ptr(luv), mem))
        return ly, luv


def preprocess_rgb(engine, rgb):
    """`colour::preprocess_rgb` on the GPU: uint8 RGB [h, w, 3] (host) -> (luma [1, h, w],
    chroma [12, ceil(h/2), ceil(w/2)]), bit-exact with the crate."""
    rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
    h, w, _ = rgb.shape
    luma = np.empty((1, h, w), np.float32)
    chroma = np.empty((12, _cdiv(h, 2), _cdiv(w, 2)), np.float32)
    check(_lib.lib().zjai_preprocess_rgb(engine.handle, _ptr(rgb), h, w, _ptr(luma),
                                         _ptr(chroma), _lib.MEM_HOST))
    return luma, chroma
