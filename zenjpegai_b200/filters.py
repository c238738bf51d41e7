"""Enhancement post-filters on reconstructed planes (src/filters/): LEF, the luma edge filter
(src/filters/lef.rs), and eICCI (src/filters/icci.rs, networks src/model/icci.rs), over the C
ABI (`zjai_lef`, `zjai_icci_filter`)."""

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
