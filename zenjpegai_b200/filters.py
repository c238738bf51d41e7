"""Enhancement post-filters on reconstructed planes (src/filters/), over the C ABI: the EFE
linear and non-linear chroma filters (src/filters/efe_linear.rs, efe_nonlinear.rs;
`zjai_efe_linear`, `zjai_efe_nonlinear`), eICCI (src/filters/icci.rs, networks
src/model/icci.rs; `zjai_icci_filter`) and LEF, the luma edge filter (src/filters/lef.rs;
`zjai_lef`), in the crate's order (src/filters/mod.rs:52-73): EFE linear, eICCI, EFE
non-linear, LEF."""

import ctypes

import numpy as np

from . import _arg, _is_torch, _lib, _like
from ._lib import ZjaiError, check


def lef(engine, luma, scale_log, channel, model_id, bit_depth=8, out=None):
    """LEF sharpening of luma [h, w] (float32, [0, 255]) steered by channel `channel` of the
    luma sigma-index map scale_log [c, sh, sw] (int32). Host numpy arrays or CUDA tensors
    (both arguments on the same side); returns the filtered plane."""
    h, w = luma.shape[-2:]
    if out is None:
        out = _like(luma, tuple(luma.shape))
    pl, mem = _arg(luma)
    po, m2 = _arg(out, tuple(luma.shape))
    if _is_torch(scale_log):
        import torch
        if scale_log.dtype != torch.int32 or not scale_log.is_contiguous() or not scale_log.is_cuda:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "scale_log must be a contiguous int32 CUDA tensor")
        ps, m3 = ctypes.c_void_p(scale_log.data_ptr()), _lib.MEM_DEVICE
    else:
        scale_log = np.ascontiguousarray(scale_log, dtype=np.int32)
        ps, m3 = ctypes.c_void_p(scale_log.ctypes.data), _lib.MEM_HOST
    if len({mem, m2, m3}) != 1:
        raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
    c, sh, sw = scale_log.shape
    check(_lib.lib().zjai_lef(engine.handle, pl, h, w, ps, c, sh, sw, channel, model_id,
                              bit_depth, po, mem))
    return out


def icci_network(engine, params):
    """One network of the eICCI bank (`IcciNet::load`) from its checkpoint's tensors."""
    from . import ICCI, Network
    return Network(engine, ICCI, 0, params)


def icci(engine, net_y, net_uv, y, u, v, use_u=True, use_v=True, tile=0, overlap=0):
    """eICCI of a 4:4:4 picture, in place on y, u, v [h, w] (float32 [0, 255], numpy or CUDA
    tensors); net_y / net_uv from `icci_network` or None (that part not filtered)."""
    h, w = y.shape[-2:]
    py, mem = _arg(y)
    pu, m2 = _arg(u, tuple(y.shape))
    pv, m3 = _arg(v, tuple(y.shape))
    if len({mem, m2, m3}) != 1:
        raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
    check(_lib.lib().zjai_icci_filter(engine.handle, net_y.handle if net_y else None,
                                      net_uv.handle if net_uv else None, int(use_u), int(use_v),
                                      py, pu, pv, h, w, tile, overlap, mem))
    return y, u, v


def _codes(a, dtype, ptype, keep):
    if a is None:
        return None
    a = np.ascontiguousarray(a, dtype=dtype).ravel()
    keep.append(a)
    return a.ctypes.data_as(ptype)


def _efe_set(st, keep):
    """`EfeLinearSet` (src/header.rs:623-639) from a dict: "cand" [u, v] (None or -1: plane not
    filtered), "filter_len" [u, v], "min_symbol", "chroma" [u, v] and "luma" [u, v] weight codes
    (per region, in the split's order; arrays of any shape, flattened)."""
    s = _lib.EfeLinearSet()
    for p in range(2):
        c = st["cand"][p]
        s.cand[p] = -1 if c is None else int(c)
        s.filter_len[p] = int(st["filter_len"][p])
        s.chroma_codes[p] = _codes(st["chroma"][p], np.uint32, _lib._u32p, keep)
        s.luma_codes[p] = _codes(st["luma"][p], np.uint32, _lib._u32p, keep)
    s.min_symbol = int(st.get("min_symbol", 0))
    return s


def _planes(y, u, v):
    h, w = y.shape[-2:]
    py, mem = _arg(y)
    pu, m2 = _arg(u)
    pv, m3 = _arg(v, tuple(u.shape))
    if len({mem, m2, m3}) != 1:
        raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
    return h, w, py, pu, pv, mem


def efe_linear(engine, y, u, v, fmt, mean, filter_set, out=None):
    """EFE linear (`efe_linear::filter_plane` over both chroma planes) with one coded set.
    y [h, w], u / v [ch, cw] float32 in [0, 255] (numpy or CUDA tensors); fmt = (s_ver, s_hor,
    c_ver, c_hor); mean = the two B1 codes. Returns the filtered (u, v) (new arrays, or `out`)."""
    h, w, py, pu, pv, mem = _planes(y, u, v)
    ch, cw = u.shape[-2:]
    if out is None:
        out = (_like(u, tuple(u.shape)), _like(v, tuple(v.shape)))
    po_u, m4 = _arg(out[0], tuple(u.shape))
    po_v, m5 = _arg(out[1], tuple(u.shape))
    if len({mem, m4, m5}) != 1:
        raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
    keep = []
    st = _efe_set(filter_set, keep)
    check(_lib.lib().zjai_efe_linear(engine.handle, py, h, w, pu, pv, ch, cw, *fmt, int(mean[0]),
                                     int(mean[1]), ctypes.byref(st), po_u, po_v, mem))
    return out


def efe_nonlinear(engine, y, u, v, fmt, params, alt=None):
    """EFE non-linear (`efe_nonlinear::apply`) in place on u / v [ch, cw]: the tile network
    where params["codes"][p] is given, then the on/off switch towards alt = (alt_u, alt_v)
    where params["masks"][0] is given. params: "min_symbol", "tile_width", "tile_height",
    "luma_min", "luma_max", "codes" [u, v], "mask_bs", "masks" [u, v] ([my, mx] arrays)."""
    h, w, py, pu, pv, mem = _planes(y, u, v)
    ch, cw = u.shape[-2:]
    pa_u = pa_v = None
    if alt is not None:
        pa_u, m4 = _arg(alt[0], tuple(u.shape))
        pa_v, m5 = _arg(alt[1], tuple(u.shape))
        if len({mem, m4, m5}) != 1:
            raise ZjaiError(_lib.INVALID_ARGUMENT, "mixed host and device arguments")
    keep = []
    q = _lib.EfeNonlinearParams()
    q.min_symbol = int(params.get("min_symbol", 0))
    q.tile_width = int(params.get("tile_width", 0))
    q.tile_height = int(params.get("tile_height", 0))
    lmin, lmax = params.get("luma_min"), params.get("luma_max")
    q.ntiles = 0 if lmin is None else min(len(lmin), len(lmax))
    q.luma_min = _codes(lmin, np.uint16, _lib._u16p, keep)
    q.luma_max = _codes(lmax, np.uint16, _lib._u16p, keep)
    codes = params.get("codes", [None, None])
    masks = params.get("masks", [None, None])
    geo = next((np.asarray(m).shape for m in masks if m is not None), (0, 0))
    q.mask_bs = int(params.get("mask_bs", 0))
    q.mask_h, q.mask_w = int(geo[0]), int(geo[1])
    for p in range(2):
        q.codes[p] = _codes(codes[p], np.uint32, _lib._u32p, keep)
        q.ncodes[p] = 0 if codes[p] is None else int(np.asarray(codes[p]).size)
        q.mask[p] = _codes(masks[p], np.uint8, _lib._u8p, keep)
    check(_lib.lib().zjai_efe_nonlinear(engine.handle, py, h, w, pu, pv, ch, cw, *fmt,
                                        ctypes.byref(q), pa_u, pa_v, mem))
    return u, v
