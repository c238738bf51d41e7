"""Networks loaded from weight files (zjai_ckpt_params -> zjai_net_create) on the GPU: a
synthesis network read from a `.pth` file gives the same planes as the same parameters passed
directly, and a latent model read from a packed file with f16 weights (the ZJB2 form) matches
the oracle run on the f16-rounded weights."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

import oracle as zo
import synthetic as syn


@pytest.fixture(scope="module")
def eng():
    import zenjpegai_b200 as zj
    e = zj.Engine(0, arena_bytes=2 << 30)
    yield e
    e.close()


def test_synthesis_from_pth(eng, tmp_path):
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import weights as W
    py, _ = syn.synthesis_params("sop", 2)
    path = tmp_path / "y.pth"
    torch.save({k: torch.from_numpy(v) for k, v in py.items()}, path)
    lat = syn.laplace_latent(7, "ly", (160, 4, 6), 2.0)
    outs = []
    for params in (py, W.Checkpoint(str(path)).params()):
        net = zj.Network(eng, zj.SYN_Y, zj.SOP, params)
        try:
            outs.append(net_forward(net, lat))
        finally:
            net.close()
    assert np.array_equal(outs[0], outs[1])


def net_forward(net, lat):
    import ctypes
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import _lib
    c, lh, lw = lat.shape
    h, w = 16 * lh, 16 * lw
    oh, ow = ctypes.c_int(), ctypes.c_int()
    zj.check(_lib.lib().zjai_synth_out_size(zj.SYN_Y, zj.SOP, h, w, ctypes.byref(oh), ctypes.byref(ow)))
    out = np.empty((1, oh.value, ow.value), np.float32)
    zj.check(_lib.lib().zjai_synthesis_primary(net.handle, ctypes.c_void_p(lat.ctypes.data), lh, lw,
                                               h, w, ctypes.c_void_p(out.ctypes.data), 0))
    return out


def test_latent_model_from_f16_packed(eng):
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import weights as W
    from test_weights_io import write_zjm
    p = syn.latent_params(31, 96, context=False)
    half = {k: v.astype(np.float16) for k, v in p.items()}
    ck = W.Checkpoint(write_zjm(half))
    params = ck.params()
    m = zj.LatentModel(eng, params)
    try:
        z = np.round(syn.laplace_latent(3, "z", (96, 5, 7), 2.0)).astype(np.float32)
        got = m.hyper_decode(z, 10, 13)
        want = zo.hyper_decode(zo.Checkpoint({k: v.astype(np.float32) for k, v in half.items()}),
                               z, 10, 13)
        rel = np.linalg.norm(got - want) / np.linalg.norm(want)
        assert rel < 2e-3
    finally:
        m.close()


def test_load_synthesis_from_model_dir(eng, tmp_path):
    """load_synthesis through a ModelDir laid out like the reference's models/ directory."""
    import zenjpegai_b200 as zj
    from zenjpegai_b200 import weights as W
    py, _ = syn.synthesis_params("sop", 2)
    rel = W.synthesis_path(1, 0, zj.SOP)
    (tmp_path / rel).parent.mkdir(parents=True)
    torch.save({k: torch.from_numpy(v) for k, v in py.items()}, tmp_path / rel)
    lat = syn.laplace_latent(8, "ly", (160, 3, 5), 2.0)
    a = W.load_synthesis(eng, W.ModelDir(str(tmp_path)), 1, zj.SOP, 0)
    b = zj.Network(eng, zj.SYN_Y, zj.SOP, py)
    try:
        assert np.array_equal(net_forward(a, lat), net_forward(b, lat))
    finally:
        a.close()
        b.close()
